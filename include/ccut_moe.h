/*
 * ccut_moe.h -- C ABI of the B200 (sm_100a) quantized MoE expert forward.
 *
 * Drop-in boundary for CostCut-Infer's MoE expert path.  The reference is pure Python
 * (numpy + numba) and has no native FFI; each entry point below replaces one Python
 * function on the path and is bound from Python with ctypes (ccut_b200/_lib.py).
 * Reference paths are relative to the reference's python/ directory.
 *
 * Conventions
 *   - Every pointer argument is a DEVICE pointer unless stated otherwise.
 *   - Every entry point returns CCUT_OK (0) or a CCUT_ERR_* code; none aborts or traps.
 *   - Work is enqueued on `stream` (a cudaStream_t); nothing synchronises the host unless
 *     stated.  Calls on the same stream are ordered; calls that share a workspace must not
 *     overlap on different streams.
 *   - Workspaces are caller-allocated, sized by the matching *_workspace_bytes function.
 *     Zero-fill a workspace before its first use and keep it for one entry point: its first
 *     bytes hold the status word and the work counters of the decode GEMM's dynamic
 *     schedule, which every call leaves at zero.
 *   - Activations are bf16 bit patterns (uint16_t); routing ids are int32.
 *   - Hidden, intermediate and every matrix dimension must be multiples of 128.
 */
#ifndef CCUT_MOE_H
#define CCUT_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define CCUT_API __attribute__((visibility("default")))
#else
#define CCUT_API
#endif

typedef struct CUstream_st* ccut_stream_t; /* == cudaStream_t */

/* Status codes.  The Python shim maps them onto the exception classes the reference
 * raises: INVALID/WORKSPACE -> ValueError (ccut/quant/weight_only.py:46,53,
 * ccut/quant/method.py:42), UNSUPPORTED -> NotImplementedError (ccut/quant/method.py:115,
 * ccut/models/generic.py:198, ccut/quant/fp8.py:48), TIMEOUT -> TimeoutError
 * (ccut/experts/reader.py:327), CUDA/NCCL -> RuntimeError. */
enum {
  CCUT_OK = 0,
  CCUT_ERR_INVALID = 1,
  CCUT_ERR_UNSUPPORTED = 2,
  CCUT_ERR_CUDA = 3,
  CCUT_ERR_WORKSPACE = 4,
  CCUT_ERR_TIMEOUT = 5,
  CCUT_ERR_NCCL = 6
};

/* Weight formats (the reference registers formats as QuantKey names,
 * ccut/quant/spec.py:72-149).  AWQ_INT4_G128 and FP8_E4M3_B128 are new keys.  FP8_E4M3_CH is
 * the reference's own FP8 (fp8_static_channel_sym / fp8_dynamic_token_sym /
 * fp8_static_tensor_sym: e4m3 with an fp32 scale per output channel, ccut/quant/kernels.py:
 * 150-171) and INT4_SYM_G128 its signed int4 (int4_w4a16_sym, ccut/quant/kernels.py:277-295);
 * both take one fp32 scale per output channel per 128-k group, so a per-channel (or
 * per-tensor) scale is that scale repeated along K, and a per-input scale must be constant
 * within each 128-k group. */
enum {
  CCUT_FMT_AWQ_INT4_G128 = 1, /* AWQ: qweight int32 [K,N/8], qzeros int32 [K/128,N/8], scales fp16 [K/128,N] */
  CCUT_FMT_FP8_E4M3_B128 = 2, /* DeepSeek fp8: weight e4m3 [N,K], scale fp32 [N/128,K/128] */
  CCUT_FMT_FP8_E4M3_CH = 3,   /* weight e4m3 [N,K], scale fp32 [K/128,N] */
  CCUT_FMT_INT4_SYM_G128 = 4  /* signed int4 v as q = v + 8 in qweight int32 [K,N/8], scale fp32 [K/128,N] */
};

/* Packed tile layouts (same byte size).  ROWS feeds the tcgen05 kernel (one output channel
 * per row, dequantized into tensor memory; the gate and up matrices of w13 are fused into
 * shared 128-row blocks); FRAGS feeds the mma.sync kernel (pre-arranged register fragments). */
enum { CCUT_LAYOUT_ROWS = 0, CCUT_LAYOUT_FRAGS = 1 };

/* Expert-GEMM kernel policy.  TC: tcgen05 (tensor-memory) kernel on the ROWS layout, best
 * when many rows share an expert (prefill).  MMA: mma.sync kernel on the FRAGS layout, best
 * for decode-sized batches.  AUTO: MMA when FRAGS weights are present and the batch gives
 * fewer than CCUT_TC_MIN_ROWS rows per routed expert, else TC. */
enum { CCUT_KERNEL_AUTO = 0, CCUT_KERNEL_TC = 1, CCUT_KERNEL_MMA = 2 };
#define CCUT_TC_MIN_ROWS 64

/* AWQ nibble order inside a 32-bit word. */
enum { CCUT_NIBBLES_AWQ = 0, CCUT_NIBBLES_SEQUENTIAL = 1 };

/* Routing modes (ccut/blocks/moe.py:71-89 for 0 and 1; 2 has no reference counterpart). */
enum {
  CCUT_ROUTE_SOFTMAX_TOPK = 0,  /* norm_topk_prob=False: softmax over E, then top-k */
  CCUT_ROUTE_TOPK_SOFTMAX = 1,  /* norm_topk_prob=True: top-k of logits, softmax over k */
  CCUT_ROUTE_SIGMOID_GROUP = 2  /* DeepSeek-V3 grouped sigmoid top-k */
};

enum { CCUT_OUT_BF16 = 0, CCUT_OUT_F32 = 1 };

typedef struct {
  int mode;             /* CCUT_ROUTE_* */
  int top_k;            /* 1..16 */
  int n_group;          /* sigmoid_group: number of expert groups (E % n_group == 0) */
  int topk_group;       /* sigmoid_group: groups kept */
  float routed_scaling; /* sigmoid_group: weight multiplier */
  const float* bias;    /* sigmoid_group: [E] selection bias, or NULL */
} ccut_route_params;

/* One MoE layer resident in HBM (replaces the reference's streamed expert reader,
 * ccut/experts/reader.py:86-334, and the per-call segment reads of
 * ccut/models/generic.py:389-400).  Shared experts (ccut/models/generic.py:380-385) are
 * stored after the routed ones as `num_shared_slices` slices of width `inter` each. */
#define CCUT_MAX_SHARED_SLICES 32

typedef struct {
  int format;            /* CCUT_FMT_* */
  int kernel;            /* CCUT_KERNEL_* */
  int hidden;            /* H */
  int inter;             /* I, routed expert intermediate size */
  int num_experts;       /* E */
  int num_shared_slices; /* shared-expert intermediate / I (0 = no shared expert), <= CCUT_MAX_SHARED_SLICES */
  float shared_gate;     /* multiplier of the shared-expert output (ccut/blocks/moe.py:177-179) */
  const void* w13;       /* ROWS layout: packed gate/up of E + slices experts, ccut_w13_bytes() each */
  const void* w2;        /* ROWS layout: packed down, ccut_w2_bytes() each */
  const void* w13_frags; /* FRAGS layout of the same weights, or NULL (then only the TC kernel runs) */
  const void* w2_frags;
  const float* router;   /* fp32 [E, H] router weight (gate_w in ccut/models/generic.py:361) */
} ccut_moe_layer;

/* ---- misc ---------------------------------------------------------------------- */
CCUT_API const char* ccut_strerror(int code);
CCUT_API int ccut_abi_version(void);

/* ---- packing: checkpoint layout (device) -> kernel tile layout (device) ---------- */
/* Bytes of one packed matrix of K inputs x N outputs. */
CCUT_API size_t ccut_packed_matrix_bytes(int format, int K, int N);
/* Bytes of one expert's packed gate+up (K = H, N = I) and down (K = I, N = H). */
CCUT_API size_t ccut_w13_bytes(int format, int hidden, int inter);
CCUT_API size_t ccut_w2_bytes(int format, int hidden, int inter);

/* Pack one matrix.  `nmat` = 2 packs gate (slot 0) and up (slot 1) into one buffer of
 * 2 * ccut_packed_matrix_bytes() (FRAGS: interleaved blocks; ROWS: fused 128-row blocks of
 * 64 gate + 64 up channels); `nmat` = 1 packs a lone matrix.
 * AWQ: q = qweight [K, N/8], z = qzeros [K/128, N/8], s = scales fp16 [K/128, N].
 * FP8 (B128): q = weight e4m3 [N, K], z unused (NULL), s = scale fp32 [N/128, K/128].
 * FP8 (CH): q = weight e4m3 [N, K], z unused (NULL), s = scale fp32 [K/128, N].
 * INT4 (SYM): q = qweight [K, N/8] of v + 8 (nibble order as for AWQ), z unused (NULL),
 * s = scale fp32 [K/128, N].
 * Replaces the load-time layout handling of ccut/quant/method.py:35-43 (create_weights). */
CCUT_API int ccut_pack_matrix(int format, int layout, const void* q, const void* z, const void* s, int K,
                              int N, int nibble_order, void* dst, int nmat, int slot, ccut_stream_t stream);

/* Debug export: packed matrix -> fp32 [K, N] (in, out), bit-identical to the checkpoint
 * dequant ((q - z) * s for AWQ, (q - 8) * s for INT4 (SYM); e4m3 * scale for FP8, NaN codes
 * -> NaN).
 * Replaces ccut/quant/kernels.py:150-171 (fp8_dequant_mat) / :276-295 (int4_dequant_row). */
CCUT_API int ccut_dequant_matrix(int format, int layout, const void* packed, int K, int N, int nmat,
                                 int slot, float* out, ccut_stream_t stream);

/* ---- routing (ccut/models/generic.py:361-362, ccut/blocks/moe.py:46-89) ----------- */
/* Workspace bytes for ccut_moe_route / ccut_moe_topk with T tokens and E experts. */
CCUT_API size_t ccut_route_workspace_bytes(int T, int E, int H);
/* logits = x @ router^T in fp32, then top-k per `rp`.  ids int32 [T, k], weights fp32
 * [T, k], logits fp32 [T, E] (may be NULL).  Ids are ordered by descending score; ties go
 * to the lowest expert index. */
CCUT_API int ccut_moe_route(const uint16_t* x, const float* router, int T, int H, int E,
                   const ccut_route_params* rp, int32_t* ids, float* weights, float* logits,
                   void* workspace, size_t ws_bytes, ccut_stream_t stream);
/* Top-k on precomputed fp32 logits [T, E] (the topk_softmax call of
 * ccut/blocks/moe.py:71-89). */
CCUT_API int ccut_moe_topk(const float* logits, int T, int E, const ccut_route_params* rp,
                  int32_t* ids, float* weights, ccut_stream_t stream);

/* ---- token permutation (ccut/models/generic.py:367-371, ccut/blocks/moe.py:164-170) - */
/* Sort the T*k (token, slot) pairs by expert, stable in (token, slot) order, and append
 * `num_shared_slices` blocks of all T tokens.  Outputs (R = T*k + slices*T rows):
 *   offsets   int32 [E + slices + 1]  first row of each expert
 *   row_token int32 [R]               token of each row
 *   row_weight fp32 [R]               routing weight of each row (shared_gate for shared)
 *   pair_row  int32 [T*k]             row of pair (t, j)
 * Ids must lie in [0, E).  `workspace` holds ccut_permute_workspace_bytes(E) bytes. */
CCUT_API size_t ccut_permute_workspace_bytes(int E);
CCUT_API int ccut_moe_permute(const int32_t* ids, const float* weights, int T, int k, int E,
                     int num_shared_slices, float shared_gate, int32_t* offsets,
                     int32_t* row_token, float* row_weight, int32_t* pair_row,
                     void* workspace, size_t ws_bytes, ccut_stream_t stream);

/* No reference counterpart: ccut_moe_permute with no workspace argument, for hosts that
 * cannot allocate device memory (a C / FFI caller with no device allocator, or a fixed
 * memory plan that forbids allocation while steps run).  Its per-expert counters live in
 * a file-scope device array of CCUT_PERMUTE_STATIC_MAX_EXPERTS int32 per device; it
 * allocates nothing.  E above that limit fails with CCUT_ERR_UNSUPPORTED.  Outputs and
 * errors are otherwise those of ccut_moe_permute.  The first call on a device (that device
 * current) looks up the array's address; make it before any stream capture.  Calls that
 * overlap on one device share the array and race: serialise them. */
#define CCUT_PERMUTE_STATIC_MAX_EXPERTS 256
CCUT_API int ccut_moe_permute_static(const int32_t* ids, const float* weights, int T, int k, int E,
                            int num_shared_slices, float shared_gate, int32_t* offsets,
                            int32_t* row_token, float* row_weight, int32_t* pair_row,
                            ccut_stream_t stream);

/* ---- expert FFN (ccut/blocks/moe.py:122-141, ccut/quant/kernels.py:219-231) ------- */
/* Workspace bytes of ccut_moe_expert_ffn (intermediate activations) for R rows. */
CCUT_API size_t ccut_expert_ffn_workspace_bytes(const ccut_moe_layer* L, int T, int k);
/* y_rows fp32 [R, H] = row_weight[r] * down(silu(x_r @ Wg) * (x_r @ Wu)) for every row
 * produced by ccut_moe_permute, using each row's expert.  `x` is bf16 [T, H]. */
CCUT_API int ccut_moe_expert_ffn(const ccut_moe_layer* L, const uint16_t* x, int T, int k,
                        const int32_t* offsets, const int32_t* row_token,
                        const float* row_weight, float* y_rows, void* workspace,
                        size_t ws_bytes, ccut_stream_t stream);
/* Same call restricted to formats (fails with CCUT_ERR_UNSUPPORTED otherwise): _w4a16 takes
 * the int4 formats (AWQ_INT4_G128, INT4_SYM_G128; the reference's "w4a16" compute path),
 * _fp8b128 FP8_E4M3_B128, _w8a16 FP8_E4M3_CH (the reference's "w8a16" path of per-channel FP8,
 * ccut/quant/method.py:109-111). */
CCUT_API int ccut_moe_expert_ffn_w4a16(const ccut_moe_layer* L, const uint16_t* x, int T, int k,
                              const int32_t* offsets, const int32_t* row_token,
                              const float* row_weight, float* y_rows, void* workspace,
                              size_t ws_bytes, ccut_stream_t stream);
CCUT_API int ccut_moe_expert_ffn_fp8b128(const ccut_moe_layer* L, const uint16_t* x, int T, int k,
                                const int32_t* offsets, const int32_t* row_token,
                                const float* row_weight, float* y_rows, void* workspace,
                                size_t ws_bytes, ccut_stream_t stream);
CCUT_API int ccut_moe_expert_ffn_w8a16(const ccut_moe_layer* L, const uint16_t* x, int T, int k,
                              const int32_t* offsets, const int32_t* row_token,
                              const float* row_weight, float* y_rows, void* workspace,
                              size_t ws_bytes, ccut_stream_t stream);

/* The two halves of ccut_moe_expert_ffn, for callers that schedule them separately.
 * gate/up: h_rows [R, I] = silu(x_r @ Wg) * (x_r @ Wu), f16 (both formats)
 * (ccut/blocks/moe.py:128-136); down: y_rows fp32 [R, H] = row_weight[r] * h_r @ Wd
 * (ccut/blocks/moe.py:137, ccut/models/generic.py:377-378). */
CCUT_API size_t ccut_gate_up_workspace_bytes(const ccut_moe_layer* L, int T);
CCUT_API int ccut_moe_gate_up(const ccut_moe_layer* L, const uint16_t* x, int T, int k,
                              const int32_t* offsets, const int32_t* row_token, uint16_t* h_rows,
                              void* workspace, size_t ws_bytes, ccut_stream_t stream);
/* Workspace bytes that let ccut_moe_down balance its work over the SMs (dynamic
 * schedule of the decode GEMM); a smaller workspace (at least 256 bytes) runs the static
 * schedule. */
CCUT_API size_t ccut_down_workspace_bytes(const ccut_moe_layer* L);
CCUT_API int ccut_moe_down(const ccut_moe_layer* L, const uint16_t* h_rows, int T, int k,
                           const int32_t* offsets, const float* row_weight, float* y_rows,
                           void* workspace, size_t ws_bytes, ccut_stream_t stream);

/* ---- combine (ccut/blocks/moe.py:172-173, ccut/models/generic.py:377-385) --------- */
/* out[t] = sum_j y_rows[pair_row[t, j]] + sum_s y_rows[T*k + s*T + t], summed in that
 * order in fp32; written as bf16 or fp32 per `out_dtype`. */
CCUT_API int ccut_moe_combine(const float* y_rows, const int32_t* pair_row, int T, int k, int H,
                     int num_shared_slices, void* out, int out_dtype, ccut_stream_t stream);

/* ---- whole layer (ccut/models/generic.py:348-386, moe_forward) --------------------- */
CCUT_API size_t ccut_moe_forward_workspace_bytes(const ccut_moe_layer* L, int T, int top_k);
/* route -> permute -> expert FFN -> combine.  ids / weights (may be NULL) receive the
 * routing decision. */
CCUT_API int ccut_moe_forward(const ccut_moe_layer* L, const ccut_route_params* rp, const uint16_t* x,
                     int T, void* out, int out_dtype, int32_t* ids, float* weights,
                     void* workspace, size_t ws_bytes, ccut_stream_t stream);

/* ---- quant linear (ccut/quant/method.py:45-58, QuantizeMethodBase.apply) ----------- */
/* y fp32 [M, N] = x [M, K] @ W, W a packed (nmat = 1) matrix; x bf16 [M, K]. */
CCUT_API size_t ccut_quant_linear_workspace_bytes(int format, int M, int K);
CCUT_API int ccut_quant_linear(int format, int layout, const void* packed, int K, int N,
                               const uint16_t* x, int M, float* y, void* workspace, size_t ws_bytes,
                               ccut_stream_t stream);

/* ---- attention and normalisation blocks of the full model (ccut/blocks/attn_gqa.py,
 * ccut/blocks/norm.py) ---------------------------------------------------------------- */
/* GQA attention (ccut/blocks/attn_gqa.py:127-153, gqa_attention_fast, as called by
 * ccut/models/generic.py:343).  q bf16 [batch, heads, seq, head_dim], k / v bf16
 * [batch, kv_heads, kv_len, head_dim] (16-byte aligned rows), out [batch, heads, seq,
 * head_dim] bf16 or fp32 (out_dtype).  Query head h reads kv head h / (heads / kv_heads).
 * causal_start >= 0 masks as build_causal_mask(seq, causal_start) (:65-73): query i sees kv
 * positions <= causal_start + i; -1: no mask.  scale <= 0 means 1/sqrt(head_dim); softcap
 * > 0 applies tanh(s / softcap) * softcap to the scaled scores (the softcap of
 * gqa_attention, :76-124).  head_dim 64 or 128.  `workspace` holds the per-split partial
 * results (ccut_gqa_attention_workspace_bytes). */
CCUT_API size_t ccut_gqa_attention_workspace_bytes(int batch, int heads, int kv_heads, int seq, int kv_len,
                                                   int head_dim);
CCUT_API int ccut_gqa_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, int batch, int heads,
                                int kv_heads, int seq, int kv_len, int head_dim, int causal_start, float scale,
                                float softcap, void* out, int out_dtype, void* workspace, size_t ws_bytes,
                                ccut_stream_t stream);
/* RMSNorm (ccut/blocks/norm.py:14-26): y = x * (mean(x^2) + eps)^-1/2 * weight per row, in
 * fp32.  x [rows, dim] bf16 or fp32 (x_dtype, CCUT_OUT_BF16 / CCUT_OUT_F32), weight fp32
 * [dim] or NULL (no affine), out [rows, dim] in out_dtype. */
CCUT_API int ccut_rms_norm(const void* x, int x_dtype, const float* weight, int rows, int dim, float eps,
                           void* out, int out_dtype, ccut_stream_t stream);
/* Rotary position embedding, half rotation (ccut/blocks/rope.py:130-175, apply_rope), on
 * one of q or k: x [batch, heads, seq, head_dim] (x_dtype), positions int32 [batch, seq],
 * inv_freq fp32 [head_dim / 2] (as build_rope returns it); the pair (i, i + head_dim/2) is
 * rotated by positions * inv_freq[i] after x is multiplied by `scale` (the attention factor
 * the reference applies to q under yarn / linear scaling; 1 for k). */
CCUT_API int ccut_apply_rope(const void* x, int x_dtype, int batch, int heads, int seq, int head_dim,
                             const float* inv_freq, const int32_t* positions, float scale, void* out,
                             int out_dtype, ccut_stream_t stream);
/* ccut_gqa_attention for a batch of sequences whose caches live in one pool (the decode step of
 * several requests in one launch; the reference attends per request,
 * ccut/models/generic.py:304-345): the k / v of batch row b are slot slots[b] (int32, device)
 * of k_pool / v_pool, slots slot_stride elements apart (a multiple of 8, at least kv_heads *
 * max_len * head_dim), kv head h at h * max_len * head_dim inside a slot; row b's query i sees
 * positions <= starts[b] + i (int32, device).  A slot outside [0, num_slots) or a negative
 * start reads nothing and gives zero rows.  The workspace is that of ccut_gqa_attention with
 * kv_len = max_len. */
CCUT_API int ccut_gqa_attention_pool(const uint16_t* q, const uint16_t* k_pool, const uint16_t* v_pool,
                                     const int32_t* slots, const int32_t* starts, int batch, int heads, int kv_heads,
                                     int seq, int max_len, int head_dim, long long slot_stride, int num_slots,
                                     float scale, float softcap, void* out, int out_dtype, void* workspace,
                                     size_t ws_bytes, ccut_stream_t stream);
/* MLA attention in the latent space (ccut/blocks/attn_mla.py:85-167, mla_decode /
 * mla_prefill, with the up-projections outside): q fp32 [batch, seq * heads, rank + rope_dim],
 * row s * heads + h = (q_nope of head h times k_up_h^T, the rotated q_pe); kv bf16 [batch,
 * kv_len, rank + rope_dim], per position (the latent c, the rotated k_pe); out [batch, seq *
 * heads, rank] (out_dtype) = softmax(q . kv^T * scale) @ kv[:, :rank], the latent output the
 * caller multiplies by v_up_h.  causal_start >= 0: query s sees positions <= causal_start +
 * s (mla_prefill's rule with causal_start = start_pos); -1: every position (mla_decode).
 * rank 512 and rope_dim 64 (DeepSeek-V2 / V3); scale > 0; q and kv 16-byte aligned.
 * Workspace: 256 bytes, or ccut_mla_attention_workspace_bytes when the kv range is split. */
CCUT_API size_t ccut_mla_attention_workspace_bytes(int batch, int heads, int seq, int kv_len);
CCUT_API int ccut_mla_attention(const float* q, const uint16_t* kv, int batch, int heads, int seq, int kv_len,
                                int rank, int rope_dim, int causal_start, float scale, void* out, int out_dtype,
                                void* workspace, size_t ws_bytes, ccut_stream_t stream);
/* ccut_mla_attention over a pool of latent caches (mla_decode, ccut/blocks/attn_mla.py:83-124,
 * for the requests of one engine step at once): batch row b attends over slot slots[b]
 * (int32, device) of kv_pool, whose slots are slot_stride elements apart (>= max_len *
 * (rank + rope_dim), a multiple of 8) and hold max_len rows each, with causal offset
 * starts[b] (int32, device): query s sees positions <= starts[b] + s.  A slot outside
 * [0, num_slots) or a negative start reads nothing and gives zero rows.  One launch serves a
 * decode batch of sequences of different lengths.  Workspace:
 * ccut_mla_attention_workspace_bytes(batch, heads, seq, max_len). */
CCUT_API int ccut_mla_attention_pool(const float* q, const uint16_t* kv_pool, const int32_t* slots,
                                     const int32_t* starts, int batch, int heads, int seq, int max_len, int rank,
                                     int rope_dim, long long slot_stride, int num_slots, float scale, void* out,
                                     int out_dtype, void* workspace, size_t ws_bytes, ccut_stream_t stream);

/* ---- diagnostics ------------------------------------------------------------------- */
/* Device-side status word kept at the start of every workspace: a kernel whose bounded
 * wait expired stores CCUT_ERR_TIMEOUT there instead of hanging.  Reads it (synchronises
 * `stream`) and clears it. */
CCUT_API int ccut_workspace_status(void* workspace, ccut_stream_t stream);
/* No reference counterpart (the reference's only timeout is the host-side one of
 * ccut/experts/reader.py:320-331).  Test of the kernels' bounded device waits: one small
 * launch waits, with the same wait routines the kernels use and a limit of budget_cycles SM
 * clocks (at most the kernels' own ~1 s), on one mbarrier that completes and on one that
 * nothing ever arrives on.  The second wait runs out, stores CCUT_ERR_TIMEOUT in the status
 * word of `workspace` (at least 256 bytes, zero-filled) and the kernel returns; int 1 of the
 * workspace receives the outcome bits (1: the completed wait succeeded; 2 and 4: the waits on
 * the idle barrier succeeded, which they must not).  Read the status with
 * ccut_workspace_status. */
CCUT_API int ccut_debug_wait_expiry(void* workspace, long long budget_cycles, ccut_stream_t stream);

/* ---- expert parallelism over NCCL (no reference counterpart: the reference runs a
 * layer's experts in one process, ccut/models/generic.py:364-385,
 * ccut/experts/pipeline.py:123-190) -------------------------------------------------- */
/* One process per GPU.  Rank r holds the routed experts [lo_r, hi_r) -- contiguous blocks of
 * E_global experts whose sizes differ by at most one, lo_r = r * (E/P) + min(r, E % P) -- and
 * every shared expert.  Ranks may carry different token counts T_local, all at most the
 * T_cap every rank sized its workspace for.  A token row goes once to each rank that owns one
 * of its experts, and one fp32 partial row per (token, rank) comes back; the exchange moves
 * fixed segments of T_cap rows per pair of ranks (rows past a segment's count carry ids -1;
 * partial rows travel as bf16, one rounding of each, as the layer's bf16 output has),
 * so that no count has to reach the host and a step never waits on it.  ccut_ep_init is
 * collective and returns once every rank has joined: distribute the unique id through a
 * channel with a timeout (e.g. a torch.distributed broadcast) so that a missing rank fails
 * there.  `timeout_s` bounds the host waits of ccut_ep_destroy. */
typedef struct ccut_ep ccut_ep;
/* Size of the NCCL unique id (host bytes) that rank 0 creates and every rank passes to
 * ccut_ep_init. */
CCUT_API size_t ccut_ep_unique_id_bytes(void);
CCUT_API int ccut_ep_unique_id(void* id_out);
/* Collective over `world` ranks (at most 64); uses the current CUDA device. */
CCUT_API int ccut_ep_init(const void* unique_id, int rank, int world, double timeout_s, ccut_ep** out);
CCUT_API int ccut_ep_destroy(ccut_ep* ep);
/* Workspace of ccut_moe_ep_dispatch / ccut_moe_ep_combine (the plan of a dispatch, which its
 * combine reads back). */
CCUT_API size_t ccut_moe_ep_exchange_workspace_bytes(int world, int T_cap, int H, int k);
/* Dispatch: the local tokens x bf16 [T_local, H] with their routing ids int32 [T_local, k]
 * (global expert ids) and weights fp32 [T_local, k] go to the ranks that own their experts.
 * Received rows land in one segment of T_cap rows per source rank (rank s at s * T_cap), in
 * the source's token order, each with its k ids made local to this rank (-1 for experts
 * elsewhere) and its k weights; rows past what a source sent carry ids -1:
 * x_recv bf16 [world * T_cap, H], ids_recv int32 [world * T_cap, k], w_recv fp32
 * [world * T_cap, k]; *recv_rows (host int) = world * T_cap, which recv_capacity must reach
 * (else CCUT_ERR_WORKSPACE).  Collective: every rank calls it, also with T_local = 0. */
CCUT_API int ccut_moe_ep_dispatch(ccut_ep* ep, const uint16_t* x, const int32_t* ids, const float* weights,
                                  int T_local, int T_cap, int H, int k, int num_experts_global, uint16_t* x_recv,
                                  int32_t* ids_recv, float* w_recv, int recv_capacity, int* recv_rows,
                                  void* workspace, size_t ws_bytes, ccut_stream_t stream);
/* Combine: y_recv bf16 [world * T_cap, H], one partial output per row the last dispatch on
 * this workspace received (in its order; rows with no local expert are ignored by their
 * source), goes back to the row's source; y_local fp32 [T_local, H] = for each local token the
 * fp32 sum of its partial rows in rank order (0 for a token routed to no expert).  Same
 * workspace as that dispatch.  Collective. */
CCUT_API int ccut_moe_ep_combine(ccut_ep* ep, const uint16_t* y_recv, int T_local, int T_cap, int H, int k,
                                 float* y_local, void* workspace, size_t ws_bytes, ccut_stream_t stream);
/* Whole expert-parallel layer: route (against L->router, fp32 [E_global, H]), dispatch, the
 * received rows through the local grouped FFN, combine, shared experts (on a second stream,
 * overlapping the exchange); out [T_local, H] bf16 or fp32.  L describes this rank's experts:
 * num_experts = hi_r - lo_r routed experts (global ids expert_lo = lo_r ..), then the shared
 * slices.  Every rank must call it, also with T_local = 0. */
CCUT_API size_t ccut_moe_ep_forward_workspace_bytes(const ccut_moe_layer* L, int num_experts_global,
                                                    int world, int T_cap, int top_k);
CCUT_API int ccut_moe_ep_forward(ccut_ep* ep, const ccut_moe_layer* L, int expert_lo,
                                 int num_experts_global, const ccut_route_params* rp,
                                 const uint16_t* x, int T_local, int T_cap, void* out, int out_dtype,
                                 void* workspace, size_t ws_bytes, ccut_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* CCUT_MOE_H */
