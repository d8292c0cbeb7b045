"""Decoder stack on the GPU: the reference's generic layer forward run on this package's kernels.

Follows ``model_forward_layer`` and ``full_attn_forward`` (``ccut/models/generic.py:304-345``,
``:403-447``) for ``full_attn`` layers with a MoE or dense FFN, and the step layout of the same
module (``ccut/models/generic.py:9-18``): embedding rows, the layers, the final RMSNorm and
``lm_head``.  For ``seq`` new tokens of one sequence at absolute positions ``p .. p + seq - 1``
each layer computes

====================================  ==================================================
``x = rms_norm(h, ln1)``              ``ccut_rms_norm`` on the fp32 residual, then bf16
``q | k | v = x @ [Wq; Wk; Wv]^T``    one bf16 GEMM (torch, cuBLAS), bf16 out
``q, k = q_norm(q), k_norm(k)``       ``ccut_rms_norm`` in bf16 (optional; the weight spans
                                      the whole projection or one head)
``q, k = rope(q, k, p ..)``           ``ccut_apply_rope``, then bf16
``K[:, p:], V[:, p:] = k, v``         the sequence's bf16 cache ``[kv_heads, max_len, d]``
``o = attention(q, K, V)``            ``ccut_gqa_attention`` over the cache buffer with
                                      ``causal_start = p``: query ``i`` reads positions
                                      ``<= p + i`` only, so the buffer needs no compaction
``h += o @ Wo^T``                     bf16 GEMM, added to the fp32 residual
``h += ffn(rms_norm(h, ln2))``        ``MoeLayer`` / ``DenseFfn`` (bf16 in, fp32 out)
====================================  ==================================================

``MlaDecoderLayer`` is the same layer with multi-head latent attention (DeepSeek-V2 / V3,
the reference's MLA blocks ``ccut/blocks/attn_mla.py`` assembled into a layer): one GEMM
gives ``q`` (or ``q_a``) and ``kv_a = [c, k_pe]``, ``c`` goes through ``kv_a_layernorm``,
RoPE turns ``q_pe`` / ``k_pe`` only, the cache keeps one bf16 row ``[c, k_pe_rot]`` (576
elements) per position, and ``ccut_mla_attention`` runs in the latent space between two
batched GEMMs (``q_nope`` folded through ``k_up``, the output unfolded through ``v_up``).

The step ends with ``logits = rms_norm(h, final_norm) @ lm_head^T`` in fp32 (``lm_head``
is kept as an fp32 copy).  ``forward_batch`` runs several sequences in one pass: their tokens
are stacked for the projections, norms, RoPE (each token at its own position) and the FFN, so
a MoE block reads its experts once for the whole batch; attention runs per sequence over its
own cache.  Every block gets its documented layout; the reference's layer
passes q as ``[1, seq, heads, d]`` to blocks that take ``[batch, heads, seq, d]``, which is
the same computation for one token and one kv head only.

Nothing here runs on the host: the norms, RoPE and attention go through the C-ABI library
(``_lib.call`` raises if it is missing), the FFN through ``MoeLayer`` / ``DenseFfn``.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from ccut_b200 import _lib
from ccut_b200.blocks.attn_mla import _latent_attention as _mla_attend
from ccut_b200.blocks.norm import rms_norm
from ccut_b200.blocks.rope import apply_rope
from ccut_b200.layer import _ptr, _stream
from ccut_b200.quant import QuantLinear
from ccut_b200.rope_tables import rope_table, yarn_mscale, yarn_rope_table

__all__ = ["DecoderLayer", "KvCache", "KvPool", "MlaDecoderLayer", "MoeDecoder", "rope_table", "yarn_mscale",
           "yarn_rope_table"]


def _tensor(a, dev: torch.device, dtype: torch.dtype) -> torch.Tensor:
    t = a if isinstance(a, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
    return t.to(device=dev, dtype=dtype).contiguous()


def _is_projection(w) -> bool:
    """A projection object: ``in_features``, ``out_features`` and ``__call__(x bf16 [M, in])``
    returning ``[M, out]`` (``quant.QuantLinear``)."""
    return callable(w) and hasattr(w, "in_features") and hasattr(w, "out_features")


def _project(w, x: torch.Tensor) -> torch.Tensor:
    """x bf16 [M, in] through a bf16 weight [out, in] (cuBLAS, bf16 out), a projection object
    (its own output type), or a list of either (outputs side by side, fp32)."""
    if isinstance(w, torch.Tensor):
        return F.linear(x, w)
    if isinstance(w, list):
        return torch.cat([_project(p, x).float() for p in w], dim=1)
    return w(x)


class KvCache:
    """One sequence's bf16 k (rotated) / v cache, ``[layers, kv_heads, max_len, head_dim]`` each;
    ``length`` positions are valid.  ``values=False`` keeps k only (``v`` None): the latent cache
    of MLA layers, ``[layers, 1, max_len, kv_lora_rank + qk_rope_head_dim]``."""

    def __init__(self, layers: int, kv_heads: int, max_len: int, head_dim: int, device="cuda", values: bool = True):
        if max_len <= 0:
            raise ValueError("max_len must be positive")
        self.k = torch.zeros((layers, kv_heads, max_len, head_dim), dtype=torch.bfloat16, device=device)
        self.v = torch.zeros_like(self.k) if values else None
        self.max_len = int(max_len)
        self.length = 0
        self.pool, self.slot = None, -1

    @classmethod
    def in_pool(cls, pool: "KvPool", slot: int) -> "KvCache":
        """The cache of slot ``slot`` of ``pool`` (views of the pool's tensors), empty."""
        if not 0 <= slot < pool.slots:
            raise ValueError(f"slot {slot} outside the pool's {pool.slots}")
        c = cls.__new__(cls)
        c.k, c.v = pool.k[slot], (pool.v[slot] if pool.v is not None else None)
        c.max_len, c.length, c.pool, c.slot = pool.max_len, 0, pool, int(slot)
        return c

    def truncate(self, n: int) -> None:
        """Keep the first ``n`` positions (later ones are overwritten by the next forward)."""
        if not 0 <= n <= self.length:
            raise ValueError(f"cannot truncate {self.length} cached positions to {n}")
        self.length = int(n)


class KvPool:
    """The caches of up to ``slots`` sequences in one allocation, ``[slots, layers, kv_heads,
    max_len, head_dim]`` bf16 for k and for v: a decode step over several of them is one
    attention launch per layer (``ccut_gqa_attention_pool``).  ``values=False`` keeps k only:
    the latent caches of MLA layers, ``[slots, layers, 1, max_len, 576]``
    (``ccut_mla_attention_pool``)."""

    def __init__(self, slots: int, layers: int, kv_heads: int, max_len: int, head_dim: int, device="cuda",
                 values: bool = True):
        if slots <= 0 or max_len <= 0:
            raise ValueError("slots and max_len must be positive")
        self.k = torch.zeros((slots, layers, kv_heads, max_len, head_dim), dtype=torch.bfloat16, device=device)
        self.v = torch.zeros_like(self.k) if values else None
        self.slots, self.max_len = int(slots), int(max_len)

    def cache(self, slot: int) -> KvCache:
        return KvCache.in_pool(self, slot)


def _attend_pool(q: torch.Tensor, pool: KvPool, layer: int, slots: torch.Tensor, starts: torch.Tensor,
                 softcap: float | None) -> torch.Tensor:
    """q ``[B, heads, S, d]`` bf16; batch row b attends over slot ``slots[b]`` of ``pool`` at
    ``layer`` with causal offset ``starts[b]`` -> ``[B, heads, S, d]`` bf16."""
    if not q.is_cuda:
        raise ValueError("attention runs on CUDA tensors only")
    B, H, S, d = q.shape
    Hkv, L = pool.k.shape[2], pool.k.shape[3]
    lib = _lib.load()
    nbytes = lib.ccut_gqa_attention_workspace_bytes(B, H, Hkv, S, L, d)
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=q.device)
    out = torch.empty((B, H, S, d), dtype=torch.bfloat16, device=q.device)
    with torch.cuda.device(q.device):
        _lib.call("ccut_gqa_attention_pool", _ptr(q), _ptr(pool.k[0, layer]), _ptr(pool.v[0, layer]), _ptr(slots),
                  _ptr(starts), B, H, Hkv, S, L, d, int(pool.k.stride(0)), pool.slots, 0.0, float(softcap or 0.0),
                  _ptr(out), _lib.OUT_BF16, _ptr(ws), ws.numel(), _stream())
    return out


def _mla_attend_pool(q: torch.Tensor, pool: KvPool, layer: int, slots: torch.Tensor, starts: torch.Tensor,
                     scale: float) -> torch.Tensor:
    """q fp32 ``[B, heads, 576]``, one query row per sequence; row b attends over slot
    ``slots[b]`` of the latent pool at ``layer``, positions ``<= starts[b]`` -> the latent output
    ``[B * heads, 512]`` fp32 (``ccut_mla_attention_pool``)."""
    if not q.is_cuda:
        raise ValueError("attention runs on CUDA tensors only")
    B, H, _ = q.shape
    L = pool.k.shape[3]
    lib = _lib.load()
    nbytes = lib.ccut_mla_attention_workspace_bytes(B, H, 1, L)
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=q.device)
    out = torch.empty((B * H, 512), dtype=torch.float32, device=q.device)
    with torch.cuda.device(q.device):
        _lib.call("ccut_mla_attention_pool", _ptr(q), _ptr(pool.k[0, layer]), _ptr(slots), _ptr(starts), B, H, 1, L,
                  512, 64, int(pool.k.stride(0)), pool.slots, float(scale), _ptr(out), _lib.OUT_F32, _ptr(ws),
                  ws.numel(), _stream())
    return out


def _attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, start_pos: int, softcap: float | None) -> torch.Tensor:
    """q ``[1, heads, seq, d]`` bf16, k / v ``[kv_heads, max_len, d]`` bf16 cache buffers ->
    ``[1, heads, seq, d]`` bf16 (``ccut_gqa_attention`` with ``causal_start = start_pos``)."""
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise ValueError("attention runs on CUDA tensors only")
    _, H, S, d = q.shape
    Hkv, L = k.shape[0], k.shape[1]
    lib = _lib.load()
    nbytes = lib.ccut_gqa_attention_workspace_bytes(1, H, Hkv, S, L, d)
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=q.device)
    out = torch.empty((1, H, S, d), dtype=torch.bfloat16, device=q.device)
    with torch.cuda.device(q.device):
        _lib.call("ccut_gqa_attention", _ptr(q), _ptr(k), _ptr(v), 1, H, Hkv, S, L, d, int(start_pos), 0.0,
                  float(softcap or 0.0), _ptr(out), _lib.OUT_BF16, _ptr(ws), ws.numel(), _stream())
    return out


class DecoderLayer:
    """One ``full_attn`` decoder layer.

    ``ln1`` / ``ln2`` [H]; ``wq`` [heads * d, H], ``wk`` / ``wv`` [kv_heads * d, H], ``wo``
    [H, heads * d] (checkpoint ``[out, in]`` layout, converted to bf16), or projection objects
    of those shapes (``quant.QuantLinear``: kept in their AWQ / FP8 format and run by
    ``ccut_quant_linear``; three of them for q / k / v are fused into one); ``q_norm`` / ``k_norm``
    None, ``[heads * d]`` / ``[kv_heads * d]`` (over the whole projection, the reference's
    ``rms_norm(q.reshape(seq, -1), w)``) or ``[d]`` (per head); ``ffn`` any object with
    ``forward(x_bf16 [T, H], out_dtype) -> [T, H]`` (``MoeLayer``, ``DenseFfn``)."""

    def __init__(self, ln1, wq, wk, wv, wo, ln2, ffn, q_norm=None, k_norm=None, *, heads: int, kv_heads: int,
                 head_dim: int, device="cuda"):
        dev = torch.device(device)
        if head_dim not in (64, 128):
            raise NotImplementedError(f"head dim {head_dim} (have 64, 128)")
        if heads <= 0 or kv_heads <= 0 or heads % kv_heads:
            raise ValueError(f"heads ({heads}) must be a positive multiple of kv_heads ({kv_heads})")
        self.heads, self.kv_heads, self.head_dim = int(heads), int(kv_heads), int(head_dim)
        self.ln1, self.ln2 = _tensor(ln1, dev, torch.float32), _tensor(ln2, dev, torch.float32)
        H = self.ln1.numel()
        self.hidden = H
        shapes = {"wq": (heads * head_dim, H), "wk": (kv_heads * head_dim, H), "wv": (kv_heads * head_dim, H),
                  "wo": (H, heads * head_dim)}
        mats = {}
        for name, m in zip(shapes, (wq, wk, wv, wo)):
            if _is_projection(m):
                if (m.out_features, m.in_features) != shapes[name]:
                    raise ValueError(f"{name} must map {shapes[name][1]} to {shapes[name][0]} features, got "
                                     f"{m.in_features} -> {m.out_features}")
                mats[name] = m
                continue
            t = _tensor(m, dev, torch.bfloat16)
            if tuple(t.shape) != shapes[name]:
                raise ValueError(f"{name} must be {shapes[name]}, got {tuple(t.shape)}")
            mats[name] = t
        if self.ln2.numel() != H:
            raise ValueError("ln1 and ln2 must have the same size")
        qkv = [mats["wq"], mats["wk"], mats["wv"]]
        if all(isinstance(p, torch.Tensor) for p in qkv):
            self.wqkv = torch.cat(qkv, 0).contiguous()
        elif all(isinstance(p, QuantLinear) for p in qkv):
            self.wqkv = QuantLinear.cat(qkv)
        else:
            self.wqkv = qkv
        self.wo = mats["wo"]
        self.q_norm = self._norm_w(q_norm, heads, dev, "q_norm")
        self.k_norm = self._norm_w(k_norm, kv_heads, dev, "k_norm")
        self.ffn = ffn
        self.device = dev

    @property
    def cache_layout(self) -> tuple:
        """What this layer keeps per position: ``(kind, kv_heads, width)``."""
        return ("gqa", self.kv_heads, self.head_dim)

    @property
    def rope_dim(self) -> int:
        return self.head_dim

    def _norm_w(self, w, n: int, dev, name: str):
        if w is None:
            return None
        t = _tensor(w, dev, torch.float32)
        if t.numel() not in (n * self.head_dim, self.head_dim):
            raise ValueError(f"{name} must have {n * self.head_dim} or {self.head_dim} elements, got {t.numel()}")
        return t

    def _qk_norm(self, x: torch.Tensor, w, n: int, eps: float) -> torch.Tensor:
        """x [seq, n * d] -> [seq, n, d], the same type (bf16, or fp32 from a quantized projection)."""
        seq, d = x.shape[0], self.head_dim
        if w is None:
            return x.reshape(seq, n, d)
        if w.numel() == n * d:
            return rms_norm(x.contiguous(), w, eps).reshape(seq, n, d)
        return rms_norm(x.reshape(seq, n, d).contiguous(), w, eps)

    def forward(self, h: torch.Tensor, spans: list, layer: int, rope: "_Rope", pooled=None) -> torch.Tensor:
        """h [N, H] fp32 (the residual stream of every span's tokens, one after the other) ->
        [N, H] fp32.  Each ``_Span`` writes its sequence's cache at ``start .. start + n - 1`` of
        ``layer`` and attends over it; the projections, norms, RoPE and the FFN run once over
        all N tokens.  ``pooled`` = ``(pool, slots, starts)`` when every span is one token of a
        cache in the same ``KvPool``: attention is then one launch for all of them."""
        N = h.shape[0]
        H, Hkv, d = self.heads, self.kv_heads, self.head_dim
        x = rms_norm(h, self.ln1, rope.eps).to(torch.bfloat16)
        qkv = _project(self.wqkv, x)
        q = self._qk_norm(qkv[:, : H * d], self.q_norm, H, rope.eps)
        k = self._qk_norm(qkv[:, H * d: (H + Hkv) * d], self.k_norm, Hkv, rope.eps)
        vt = qkv[:, (H + Hkv) * d:].reshape(N, Hkv, d).transpose(0, 1)
        if len(spans) == 1:
            s = spans[0]
            pos = torch.arange(s.start, s.start + s.n, dtype=torch.int32, device=h.device)
        else:
            pos = torch.cat([torch.arange(s.start, s.start + s.n, dtype=torch.int32) for s in spans]).to(h.device)
        qr, kr = apply_rope(q.transpose(0, 1).unsqueeze(0), k.transpose(0, 1).unsqueeze(0), rope.inv_freq,
                            pos.reshape(1, N), rope.attn_factor, rope.scaling_type)
        qr = qr.to(torch.bfloat16)
        for s in spans:
            s.cache.k[layer, :, s.start: s.start + s.n] = kr[0, :, s.off: s.off + s.n]
            s.cache.v[layer, :, s.start: s.start + s.n] = vt[:, s.off: s.off + s.n]
        if pooled is not None:  # N sequences of one token each: q [N, heads, 1, d]
            pool, slots, starts = pooled
            o = _attend_pool(qr[0].transpose(0, 1).unsqueeze(2).contiguous(), pool, layer, slots, starts,
                             rope.softcap)
            o2 = o[:, :, 0, :].reshape(N, H * d)
        else:
            outs = [_attend(qr[:, :, s.off: s.off + s.n].contiguous(), s.cache.k[layer], s.cache.v[layer], s.start,
                            rope.softcap) for s in spans]
            o = outs[0] if len(outs) == 1 else torch.cat(outs, dim=2)
            o2 = o[0].transpose(0, 1).reshape(N, H * d)
        h = h + _project(self.wo, o2).float()
        x2 = rms_norm(h, self.ln2, rope.eps).to(torch.bfloat16)
        return h + self.ffn.forward(x2, out_dtype=torch.float32)


def _fuse_inputs(parts: list):
    """Projections of the same input run as one: bf16 weights concatenated (one cuBLAS GEMM),
    ``QuantLinear`` ones fused into one, else the list (``_project`` runs each)."""
    if all(isinstance(p, torch.Tensor) for p in parts):
        return torch.cat(parts, 0).contiguous()
    if all(isinstance(p, QuantLinear) for p in parts):
        return QuantLinear.cat(parts)
    return list(parts)


def _weight(m, shape: tuple, dev, name: str, projection_ok: bool = True):
    """A bf16 ``[out, in]`` weight of ``shape`` or a projection object mapping ``in`` to ``out``."""
    if _is_projection(m):
        if not projection_ok:
            raise ValueError(f"{name} must be a dense matrix")
        if (m.out_features, m.in_features) != shape:
            raise ValueError(f"{name} must map {shape[1]} to {shape[0]} features, got {m.in_features} -> "
                             f"{m.out_features}")
        return m
    t = _tensor(m, dev, torch.bfloat16)
    if tuple(t.shape) != shape:
        raise ValueError(f"{name} must be {shape}, got {tuple(t.shape)}")
    return t


class MlaDecoderLayer:
    """One multi-head latent attention decoder layer (DeepSeek-V2 / V3).

    Checkpoint ``[out, in]`` matrices (converted to bf16) or projection objects
    (``quant.QuantLinear``): ``wq`` = ``q_proj`` [heads * (d_nope + d_rope), H], or with
    ``q_a`` / ``q_a_norm`` (``q_a_proj`` [q_rank, H] and its RMSNorm) the ``q_b_proj``
    [heads * (d_nope + d_rope), q_rank]; ``wkv_a`` = ``kv_a_proj_with_mqa`` [rank + d_rope, H];
    ``wkv_b`` = ``kv_b_proj`` [heads * (d_nope + d_v), rank], per head ``d_nope`` rows of k then
    ``d_v`` rows of v (a dense matrix: its blocks are kept as fp32 ``k_up`` [heads, d_nope, rank]
    and ``v_up`` [heads, rank, d_v] for the batched GEMMs around the kernel); ``wo`` =
    ``o_proj`` [H, heads * d_v]; ``kv_norm`` = ``kv_a_layernorm`` [rank] or None.
    ``softmax_scale`` None is ``(d_nope + d_rope) ** -0.5``.  ``ccut_mla_attention`` takes
    ``kv_lora_rank`` 512 and ``qk_rope_head_dim`` 64; other sizes raise ``NotImplementedError``."""

    def __init__(self, ln1, wq, wkv_a, wkv_b, wo, ln2, ffn, kv_norm=None, *, heads: int, qk_nope_head_dim: int,
                 qk_rope_head_dim: int, v_head_dim: int, kv_lora_rank: int = 512, q_a=None, q_a_norm=None,
                 softmax_scale: float | None = None, device="cuda"):
        dev = torch.device(device)
        if (kv_lora_rank, qk_rope_head_dim) != (512, 64):
            raise NotImplementedError(f"MLA with kv_lora_rank {kv_lora_rank} / qk_rope_head_dim {qk_rope_head_dim} "
                                      "(have 512 / 64)")
        H_, dn, dr, dv, R = int(heads), int(qk_nope_head_dim), int(qk_rope_head_dim), int(v_head_dim), 512
        if H_ <= 0 or dn <= 0 or dv <= 0:
            raise ValueError("heads, qk_nope_head_dim and v_head_dim must be positive")
        self.heads, self.d_nope, self.d_rope, self.d_v, self.rank = H_, dn, dr, dv, R
        self.ln1, self.ln2 = _tensor(ln1, dev, torch.float32), _tensor(ln2, dev, torch.float32)
        H = self.ln1.numel()
        if self.ln2.numel() != H:
            raise ValueError("ln1 and ln2 must have the same size")
        self.hidden = H
        if (q_a is None) != (q_a_norm is None):
            raise ValueError("q_a and q_a_norm go together")
        self.q_rank = 0
        if q_a is not None:
            self.q_rank = int(q_a.out_features if _is_projection(q_a) else np.shape(q_a)[0])
            q_a = _weight(q_a, (self.q_rank, H), dev, "q_a")
            self.q_a_norm = _tensor(q_a_norm, dev, torch.float32)
            if self.q_a_norm.numel() != self.q_rank:
                raise ValueError(f"q_a_norm must have {self.q_rank} elements")
        wq = _weight(wq, (H_ * (dn + dr), self.q_rank or H), dev, "wq")
        wkv_a = _weight(wkv_a, (R + dr, H), dev, "wkv_a")
        self.w_in = _fuse_inputs([q_a if q_a is not None else wq, wkv_a])
        self.wq_b = wq if q_a is not None else None
        b = _tensor(wkv_b, dev, torch.float32) if not _is_projection(wkv_b) else None
        if b is None or tuple(b.shape) != (H_ * (dn + dv), R):
            raise ValueError(f"wkv_b must be a dense [{H_ * (dn + dv)}, {R}] matrix")
        b = b.view(H_, dn + dv, R)
        self.k_up = b[:, :dn].contiguous()  # [heads, d_nope, rank]
        self.v_up = b[:, dn:].transpose(1, 2).contiguous()  # [heads, rank, d_v]
        self.wo = _weight(wo, (H, H_ * dv), dev, "wo")
        self.kv_norm = None
        if kv_norm is not None:
            self.kv_norm = _tensor(kv_norm, dev, torch.float32)
            if self.kv_norm.numel() != R:
                raise ValueError(f"kv_norm must have {R} elements")
        self.scale = float(softmax_scale) if softmax_scale is not None else float((dn + dr) ** -0.5)
        if not self.scale > 0:
            raise ValueError("softmax_scale must be positive")
        self.ffn = ffn
        self.device = dev

    @property
    def cache_layout(self) -> tuple:
        return ("mla", 1, self.rank + self.d_rope)

    @property
    def rope_dim(self) -> int:
        return self.d_rope

    def forward(self, h: torch.Tensor, spans: list, layer: int, rope: "_Rope", pooled=None) -> torch.Tensor:
        """h [N, H] fp32 -> [N, H] fp32, as ``DecoderLayer.forward``; each span writes its
        latent rows at ``start .. start + n - 1`` of ``layer`` and attends over rows ``0 ..
        start + n - 1`` with ``causal_start = start``; with ``pooled`` (one token per span, all
        caches in one ``KvPool``) in one launch for all of them."""
        N = h.shape[0]
        H, dn, dr, dv, R = self.heads, self.d_nope, self.d_rope, self.d_v, self.rank
        x = rms_norm(h, self.ln1, rope.eps).to(torch.bfloat16)
        proj = _project(self.w_in, x)
        if self.wq_b is not None:
            qa = rms_norm(proj[:, : self.q_rank].contiguous(), self.q_a_norm, rope.eps)
            q = _project(self.wq_b, qa.to(torch.bfloat16))
        else:
            q = proj[:, : H * (dn + dr)]
        q = q.reshape(N, H, dn + dr)
        kv_a = proj[:, -(R + dr):]
        c = kv_a[:, :R].contiguous()
        if self.kv_norm is not None:
            c = rms_norm(c, self.kv_norm, rope.eps)
        if len(spans) == 1:
            s = spans[0]
            pos = torch.arange(s.start, s.start + s.n, dtype=torch.int32, device=h.device)
        else:
            pos = torch.cat([torch.arange(s.start, s.start + s.n, dtype=torch.int32) for s in spans]).to(h.device)
        q_pe, k_pe = apply_rope(q[:, :, dn:].transpose(0, 1).unsqueeze(0).contiguous(),
                                kv_a[:, R:].reshape(1, 1, N, dr).contiguous(), rope.inv_freq, pos.reshape(1, N),
                                rope.attn_factor, rope.scaling_type)
        for s in spans:
            rows = s.cache.k[layer, 0, s.start: s.start + s.n]
            rows[:, :R] = c[s.off: s.off + s.n]
            rows[:, R:] = k_pe[0, 0, s.off: s.off + s.n]
        q_lat = torch.bmm(q[:, :, :dn].float().transpose(0, 1), self.k_up)  # [heads, N, rank]
        qq = torch.cat([q_lat.transpose(0, 1), q_pe[0].transpose(0, 1).float()], dim=-1).contiguous()  # [N, H, 576]
        if pooled is not None:  # N sequences of one token each
            pool, slots, starts = pooled
            o_lat = _mla_attend_pool(qq, pool, layer, slots, starts, self.scale).view(N, H, R)
        else:
            o_lat = torch.cat([_mla_attend(qq[s.off: s.off + s.n], s.cache.k[layer, 0, : s.start + s.n], s.start,
                                           self.scale).view(s.n, H, R) for s in spans])
        o = torch.bmm(o_lat.transpose(0, 1), self.v_up)  # [heads, N, d_v]
        o2 = o.transpose(0, 1).reshape(N, H * dv).to(torch.bfloat16)
        h = h + _project(self.wo, o2).float()
        x2 = rms_norm(h, self.ln2, rope.eps).to(torch.bfloat16)
        return h + self.ffn.forward(x2, out_dtype=torch.float32)


class _Span:
    """One sequence's part of a batch: ``n`` tokens at rows ``off ..`` of the batch, positions
    ``start ..`` of ``cache``."""

    def __init__(self, cache: KvCache, start: int, off: int, n: int):
        self.cache, self.start, self.off, self.n = cache, start, off, n


class _Rope:
    """The per-model constants every layer's attention reads."""

    def __init__(self, inv_freq: torch.Tensor, attn_factor: float, scaling_type: str, eps: float, softcap):
        self.inv_freq, self.attn_factor, self.scaling_type = inv_freq, float(attn_factor), scaling_type
        self.eps, self.softcap = float(eps), softcap


class MoeDecoder:
    """Embedding, decoder layers, final norm and ``lm_head`` of one model.

    ``layers``: ``DecoderLayer`` or ``MlaDecoderLayer`` objects, all of one kind (the cache
    layout is the model's).  ``embed`` / ``lm_head`` [vocab, H]; ``inv_freq`` / ``attention_factor`` / ``scaling_type``
    as ``build_rope`` returns them (``rope_table`` for the plain cases); ``eps`` the epsilon of
    every RMSNorm (the reference's layer calls ``rms_norm`` with its default, 1e-6); ``softcap``
    the model's ``attn_logit_softcapping`` (or None)."""

    def __init__(self, embed, layers: list, final_norm, lm_head, *, inv_freq, attention_factor: float = 1.0,
                 scaling_type: str = "none", eps: float = 1e-6, softcap: float | None = None, device="cuda"):
        dev = torch.device(device)
        if not layers:
            raise ValueError("a decoder needs at least one layer")
        self.embed = _tensor(embed, dev, torch.bfloat16)
        self.final_norm = _tensor(final_norm, dev, torch.float32)
        self.lm_head = _tensor(lm_head, dev, torch.float32)
        V, H = self.embed.shape
        if tuple(self.lm_head.shape) != (V, H) or self.final_norm.numel() != H:
            raise ValueError(f"lm_head must be {(V, H)} and final_norm [{H}]")
        for i, lay in enumerate(layers):
            if lay.hidden != H or lay.cache_layout != layers[0].cache_layout or lay.rope_dim != layers[0].rope_dim:
                raise ValueError(f"layer {i} does not match the model's hidden size / kv layout")
        self.layers = list(layers)
        self.vocab, self.hidden = V, H
        self.layout = layers[0].cache_layout
        ft = _tensor(inv_freq, dev, torch.float32)
        if ft.numel() != layers[0].rope_dim // 2:
            raise ValueError(f"inv_freq has {ft.numel()} entries for rope dim {layers[0].rope_dim}")
        if self.layout[0] == "mla" and softcap:
            raise NotImplementedError("attention logit soft-capping in MLA layers")
        self.rope = _Rope(ft, attention_factor, scaling_type, eps, softcap)
        self.device = dev

    def new_cache(self, max_len: int) -> KvCache:
        kind, kvh, width = self.layout
        return KvCache(len(self.layers), kvh, max_len, width, self.device, values=kind == "gqa")

    def new_pool(self, slots: int, max_len: int) -> KvPool:
        kind, kvh, width = self.layout
        return KvPool(slots, len(self.layers), kvh, max_len, width, self.device, values=kind == "gqa")

    def _ids(self, tokens) -> torch.Tensor:
        if isinstance(tokens, torch.Tensor):
            return tokens.to(device=self.device, dtype=torch.int64).reshape(-1)
        return torch.as_tensor(np.asarray(tokens, dtype=np.int64).reshape(-1)).to(self.device)

    def forward(self, tokens, cache: KvCache, start_pos: int | None = None, all_logits: bool = False) -> torch.Tensor:
        """Run ``tokens`` at positions ``start_pos ..`` (default: after the cached ones) and return
        the fp32 logits of the last token ``[vocab]`` (``all_logits``: of every token
        ``[seq, vocab]``).  Positions from ``start_pos`` on are replaced in ``cache``."""
        return self.forward_batch([(tokens, cache, start_pos)], all_logits)[0]

    def forward_batch(self, items: list, all_logits: bool = False) -> list:
        """Several sequences in one pass: ``items`` = ``[(tokens, cache, start_pos or None), ...]``
        with a different cache each.  The projections and the FFN run once over all tokens (the
        MoE block sees every sequence's tokens together); attention runs per sequence over its
        own cache.  Returns per item the logits of its last token ``[vocab]`` (``all_logits``:
        ``[n, vocab]``)."""
        if not items:
            return []
        spans, ids_all, off = [], [], 0
        for tokens, cache, start_pos in items:
            ids = self._ids(tokens)
            n = ids.numel()
            p = cache.length if start_pos is None else int(start_pos)
            if n == 0:
                raise ValueError("no tokens to run")
            if not 0 <= p <= cache.length:
                raise ValueError(f"start position {p} is past the {cache.length} cached positions")
            if p + n > cache.max_len:
                raise ValueError(f"{p} + {n} positions do not fit the cache of {cache.max_len}")
            if any(s.cache is cache or (cache.pool is not None and s.cache.pool is cache.pool
                                        and s.cache.slot == cache.slot) for s in spans):
                raise ValueError("each sequence of a batch needs its own cache")
            spans.append(_Span(cache, p, off, n))
            ids_all.append(ids)
            off += n
        ids = ids_all[0] if len(ids_all) == 1 else torch.cat(ids_all)
        if int(ids.min()) < 0 or int(ids.max()) >= self.vocab:
            raise ValueError(f"token ids must be in [0, {self.vocab})")
        pool = spans[0].cache.pool
        pooled = None
        if len(spans) > 1 and pool is not None and all(s.n == 1 and s.cache.pool is pool for s in spans):
            slots = torch.tensor([s.cache.slot for s in spans], dtype=torch.int32).to(self.device)
            starts = torch.tensor([s.start for s in spans], dtype=torch.int32).to(self.device)
            pooled = (pool, slots, starts)
        h = self.embed.index_select(0, ids).float()
        for i, lay in enumerate(self.layers):
            h = lay.forward(h, spans, i, self.rope, pooled)
        for s in spans:
            s.cache.length = s.start + s.n
        if all_logits:
            logits = F.linear(rms_norm(h, self.final_norm, self.rope.eps), self.lm_head)
            return [logits[s.off: s.off + s.n] for s in spans]
        last = torch.tensor([s.off + s.n - 1 for s in spans], dtype=torch.int64).to(self.device)
        logits = F.linear(rms_norm(h.index_select(0, last), self.final_norm, self.rope.eps), self.lm_head)
        return [logits[j] for j in range(len(spans))]
