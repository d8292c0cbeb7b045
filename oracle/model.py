"""CPU restatement (numpy, fp32) of the reference's generic decoder path.

Test infrastructure only: the GPU tests check ``ccut_b200.model`` (the decoder stack that
the engine backend ``ccut_b200.backend.GenericBackend`` runs) against these functions, and
these functions are pinned to the reference's own layer forward
(``tests/golden/model_decode.npz``, made by ``tests/golden/make_golden_model.py``).

* ``decoder_layer`` follows ``model_forward_layer`` (``ccut/models/generic.py:403-447``) for a
  ``full_attn`` layer: ``h + attn(rms_norm(h, ln1))``, then ``h + ffn(rms_norm(h, ln2))``.
* ``attention`` follows ``full_attn_forward`` (``ccut/models/generic.py:304-345``): q / k / v
  projections ``x @ W^T``, the optional q / k RMSNorm, RoPE at absolute positions
  ``start_pos ..``, the new k (rotated) and v appended to the layer's cache, causal GQA
  attention over the whole cache (``gqa_attention_fast`` with ``build_causal_mask``), then
  ``o_proj``.  The reference's own call passes q as ``[1, seq, heads, d]`` to functions that
  take ``[batch, heads, seq, d]``; the two layouts agree for one token and one kv head
  (the case the golden vectors pin).  Here every block gets its documented layout, so
  prefill and grouped kv heads follow the block semantics pinned in ``oracle.attention``.
  The q / k norm weight covers the whole projection (``[heads * d]``, the reference's
  ``rms_norm(q.reshape(seq, -1), w)``) or one head (``[d]``, applied per head).
* ``mla_attention_block`` is a multi-head latent attention layer (DeepSeek-V2 / V3) built
  from the reference's MLA blocks (``ccut/blocks/attn_mla.py``), whose module docstring
  (``:1-13``) gives the data flow: ``kv_a = x @ kv_a_proj`` split into the latent ``c`` and
  ``k_pe``, ``q = x @ q_proj`` split into ``q_nope`` and ``q_pe``, RoPE on ``q_pe`` / ``k_pe``
  only, ``c`` and the rotated ``k_pe`` appended to the cache (``mla_update_state``), the
  attention of ``mla_prefill`` / ``mla_decode`` (``oracle.attention.mla_attention``) with
  ``k_up`` / ``v_up`` the per-head blocks of ``kv_b_proj``, then ``o_proj``.  The reference has
  no MLA layer of its own (its layer forward runs ``full_attn`` and ``linear_attn`` layers);
  the layer adds what DeepSeek-V2's published architecture adds around those blocks: the
  RMSNorm of ``c`` (``kv_a_layernorm``) and, with a q rank, ``q = rms_norm(x @ q_a^T) @ q_b^T``.
* ``moe_ffn`` is the MoE branch of the same layer (``ccut/models/generic.py:348-386``, the
  restatement in ``oracle.moe.moe_forward``).
* ``model_forward`` is the data flow of the module docstring (``ccut/models/generic.py:9-18``):
  embedding rows (``ccut/blocks/heads.py:45-46``), the layers, the final RMSNorm and
  ``lm_head`` (``hidden @ W^T``, ``ccut/blocks/heads.py:59-60``).

``bf16_acts=True`` rounds to bf16 where the GPU path stores bf16 (each GEMM input, the
q / k / v projections, the rotated q and k, the attention output, the o_proj output), so the
GPU comparison can use tight tolerances; ``False`` is the reference's fp32 path.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable

import numpy as np

from oracle import attention, formats, moe

__all__ = ["AttnWeights", "DecoderSpec", "KvCache", "MlaWeights", "attention_block", "decoder_layer",
           "mla_attention_block", "mla_up_blocks", "moe_ffn", "model_forward", "round_bf16"]


def round_bf16(x: np.ndarray) -> np.ndarray:
    return formats.bf16_bits_to_f32(formats.bf16_bits_from_f32(np.asarray(x, np.float32)))


@dataclass
class AttnWeights:
    """One full-attention decoder layer's dense weights (fp32, [out, in] like the checkpoint)."""

    ln1: np.ndarray  # [H] input_layernorm
    wq: np.ndarray  # [heads * d, H]
    wk: np.ndarray  # [kv_heads * d, H]
    wv: np.ndarray  # [kv_heads * d, H]
    wo: np.ndarray  # [H, heads * d]
    ln2: np.ndarray  # [H] post_attention_layernorm
    q_norm: np.ndarray | None = None  # [heads * d] or [d]
    k_norm: np.ndarray | None = None  # [kv_heads * d] or [d]


@dataclass
class MlaWeights:
    """One MLA decoder layer's dense weights (fp32, [out, in] like the checkpoint).  ``wq`` is
    ``q_proj`` [heads * (d_nope + d_rope), H], or with ``wq_a`` / ``q_a_norm`` the ``q_b_proj``
    [heads * (d_nope + d_rope), q_rank] after ``q_a_proj`` [q_rank, H]; ``wkv_b`` holds per head
    ``d_nope`` rows of k then ``d_v`` rows of v.  ``scale`` None is ``(d_nope + d_rope) ** -0.5``."""

    ln1: np.ndarray  # [H]
    wq: np.ndarray
    wkv_a: np.ndarray  # [rank + d_rope, H] kv_a_proj_with_mqa
    wkv_b: np.ndarray  # [heads * (d_nope + d_v), rank]
    wo: np.ndarray  # [H, heads * d_v]
    ln2: np.ndarray  # [H]
    heads: int
    d_nope: int
    d_rope: int
    d_v: int
    kv_norm: np.ndarray | None = None  # [rank] kv_a_layernorm
    wq_a: np.ndarray | None = None  # [q_rank, H]
    q_a_norm: np.ndarray | None = None  # [q_rank]
    scale: float | None = None

    @property
    def rank(self) -> int:
        return self.wkv_a.shape[0] - self.d_rope

    @property
    def softmax_scale(self) -> float:
        return float(self.scale) if self.scale is not None else float((self.d_nope + self.d_rope) ** -0.5)


def mla_up_blocks(wkv_b: np.ndarray, heads: int, d_nope: int, d_v: int) -> tuple[np.ndarray, np.ndarray]:
    """``kv_b_proj`` [heads * (d_nope + d_v), rank] -> the reference blocks' ``k_up_proj``
    [rank, heads * d_nope] and ``v_up_proj`` [rank, heads * d_v] (``c @ k_up`` = every head's
    k_nope side by side)."""
    w = np.asarray(wkv_b, np.float32)
    rank = w.shape[1]
    b = w.reshape(heads, d_nope + d_v, rank)
    k_up = b[:, :d_nope].transpose(2, 0, 1).reshape(rank, heads * d_nope)
    v_up = b[:, d_nope:].transpose(2, 0, 1).reshape(rank, heads * d_v)
    return np.ascontiguousarray(k_up), np.ascontiguousarray(v_up)


@dataclass
class DecoderSpec:
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    inv_freq: np.ndarray  # [head_dim / 2]
    attn_factor: float = 1.0
    scaling_type: str = "none"
    eps: float = 1e-6
    softcap: float | None = None


@dataclass
class KvCache:
    """Per layer: k (rotated) and v, ``[kv_heads, positions, d]`` fp32; for an MLA layer the
    latent ``c`` ``[1, positions, rank]`` and the rotated ``k_pe`` ``[1, positions, d_rope]``."""

    k: list = field(default_factory=list)
    v: list = field(default_factory=list)

    def length(self, layer: int) -> int:
        return 0 if layer >= len(self.k) else self.k[layer].shape[1]


def _rb(x: np.ndarray, on: bool) -> np.ndarray:
    return round_bf16(x) if on else np.asarray(x, np.float32)


def _qk_norm(x: np.ndarray, w: np.ndarray | None, heads: int, d: int, eps: float) -> np.ndarray:
    """x [seq, heads, d]; w over the whole row ([heads * d]) or one head ([d])."""
    if w is None:
        return x
    seq = x.shape[0]
    if w.size == heads * d:
        return attention.rms_norm(x.reshape(seq, heads * d), w, eps).reshape(seq, heads, d)
    if w.size == d:
        return attention.rms_norm(x, w, eps)
    raise ValueError(f"q / k norm weight of {w.size} elements for {heads} heads of {d}")


def attention_block(x: np.ndarray, w: AttnWeights, spec: DecoderSpec, cache: KvCache, layer: int, start_pos: int,
                    bf16_acts: bool = False) -> np.ndarray:
    """x [seq, H] (the normed hidden state) -> o_proj output [seq, H]; appends to ``cache``."""
    seq = x.shape[0]
    H, Hkv, d = spec.heads, spec.kv_heads, spec.head_dim
    if cache.length(layer) != start_pos:
        raise ValueError(f"layer {layer} caches {cache.length(layer)} positions, the batch starts at {start_pos}")
    x = _rb(x, bf16_acts)
    q = _rb(x @ w.wq.T, bf16_acts).reshape(seq, H, d)
    k = _rb(x @ w.wk.T, bf16_acts).reshape(seq, Hkv, d)
    v = _rb(x @ w.wv.T, bf16_acts).reshape(seq, Hkv, d)
    q = _rb(_qk_norm(q, w.q_norm, H, d, spec.eps), bf16_acts)
    k = _rb(_qk_norm(k, w.k_norm, Hkv, d, spec.eps), bf16_acts)
    pos = np.arange(start_pos, start_pos + seq, dtype=np.int64)[None, :]
    qr, kr = attention.apply_rope(q.transpose(1, 0, 2)[None], k.transpose(1, 0, 2)[None], spec.inv_freq, pos,
                                  spec.attn_factor, spec.scaling_type)
    qr, kr = _rb(qr, bf16_acts), _rb(kr, bf16_acts)
    _append(cache, layer, kr[0], v.transpose(1, 0, 2))
    mask = attention.causal_mask(seq, start_pos)
    o = attention.gqa_attention(qr, cache.k[layer][None], cache.v[layer][None], mask, None, spec.softcap)
    o = _rb(o[0].transpose(1, 0, 2).reshape(seq, H * d), bf16_acts)
    return _rb(o @ w.wo.T, bf16_acts)


def _append(cache: KvCache, layer: int, k: np.ndarray, v: np.ndarray) -> None:
    if layer == len(cache.k):
        cache.k.append(k)
        cache.v.append(v)
    else:
        cache.k[layer] = np.concatenate([cache.k[layer], k], axis=1)
        cache.v[layer] = np.concatenate([cache.v[layer], v], axis=1)


def mla_attention_block(x: np.ndarray, w: MlaWeights, spec: DecoderSpec, cache: KvCache, layer: int, start_pos: int,
                        bf16_acts: bool = False) -> np.ndarray:
    """x [seq, H] (the normed hidden state) -> o_proj output [seq, H]; appends ``c`` and the
    rotated ``k_pe`` to ``cache``.  ``spec.inv_freq`` is the table of the rope dimension;
    ``spec.attn_factor`` scales ``q_pe`` as ``apply_rope`` does for the yarn / linear scalings.
    With ``bf16_acts`` the rotated ``q_pe`` stays fp32 (the GPU path keeps it so)."""
    seq = x.shape[0]
    H, dn, dr, dv, R = w.heads, w.d_nope, w.d_rope, w.d_v, w.rank
    if cache.length(layer) != start_pos:
        raise ValueError(f"layer {layer} caches {cache.length(layer)} positions, the batch starts at {start_pos}")
    x = _rb(x, bf16_acts)
    if w.wq_a is not None:
        qa = _rb(x @ w.wq_a.T, bf16_acts)
        qa = _rb(attention.rms_norm(qa, w.q_a_norm, spec.eps), bf16_acts)
        q = _rb(qa @ w.wq.T, bf16_acts)
    else:
        q = _rb(x @ w.wq.T, bf16_acts)
    q = q.reshape(seq, H, dn + dr)
    kv_a = _rb(x @ w.wkv_a.T, bf16_acts)
    c, k_pe = kv_a[:, :R], kv_a[:, R:]
    if w.kv_norm is not None:
        c = _rb(attention.rms_norm(c, w.kv_norm, spec.eps), bf16_acts)
    pos = np.arange(start_pos, start_pos + seq, dtype=np.int64)[None, :]
    q_pe, k_rot = attention.apply_rope(q[:, :, dn:].transpose(1, 0, 2)[None], k_pe[None, None], spec.inv_freq, pos,
                                       spec.attn_factor, spec.scaling_type)
    _append(cache, layer, c[None], _rb(k_rot[0], bf16_acts))
    k_up, v_up = mla_up_blocks(w.wkv_b, H, dn, dv)
    o = attention.mla_attention(cache.k[layer][0], cache.v[layer][0], q[:, :, :dn], q_pe[0].transpose(1, 0, 2), k_up,
                                v_up, w.softmax_scale, start_pos)
    o = _rb(np.asarray(o, np.float32).reshape(seq, H * dv), bf16_acts)
    return _rb(o @ w.wo.T, bf16_acts)


def moe_ffn(router: np.ndarray, top_k: int, mode: str, w_lookup, shared=None, shared_gate: float = 1.0,
            route_kw: dict | None = None) -> Callable[[np.ndarray], np.ndarray]:
    """The MoE branch as a callable ``x [seq, H] -> [seq, H]`` (``oracle.moe.moe_forward``)."""

    def f(x: np.ndarray) -> np.ndarray:
        return moe.moe_forward(x, router, top_k, mode, w_lookup, shared, shared_gate, route_kw=route_kw)[0]

    return f


def decoder_layer(h: np.ndarray, w, ffn: Callable[[np.ndarray], np.ndarray], spec: DecoderSpec, cache: KvCache,
                  layer: int, start_pos: int, bf16_acts: bool = False) -> np.ndarray:
    """``w``: ``AttnWeights`` (a ``full_attn`` layer) or ``MlaWeights`` (an MLA layer)."""
    h = np.asarray(h, np.float32)
    block = mla_attention_block if isinstance(w, MlaWeights) else attention_block
    h = h + block(attention.rms_norm(h, w.ln1, spec.eps), w, spec, cache, layer, start_pos, bf16_acts)
    x2 = _rb(attention.rms_norm(h, w.ln2, spec.eps), bf16_acts)
    return (h + ffn(x2)).astype(np.float32)


def model_forward(tokens, embed: np.ndarray, layers: list, ffns: list, final_norm: np.ndarray, lm_head: np.ndarray,
                  spec: DecoderSpec, cache: KvCache, start_pos: int, bf16_acts: bool = False):
    """tokens [seq] -> (logits [seq, vocab] fp32, hidden state after each layer)."""
    h = np.asarray(embed, np.float32)[np.asarray(tokens, np.int64)]
    hs = []
    for i, (w, f) in enumerate(zip(layers, ffns)):
        h = decoder_layer(h, w, f, spec, cache, i, start_pos, bf16_acts)
        hs.append(h)
    hn = attention.rms_norm(h, final_norm, spec.eps)
    return (hn @ np.asarray(lm_head, np.float32).T).astype(np.float32), hs
