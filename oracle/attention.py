"""CPU restatement (numpy, fp32) of the reference's attention and RMSNorm blocks.

Test infrastructure only: the GPU tests check ``ccut_b200.blocks.attn_gqa`` and
``ccut_b200.blocks.norm`` against these functions, and these functions are pinned to the
reference's own outputs (``tests/golden/attn_norm.npz``, made by
``tests/golden/make_golden_attn.py``).

* ``gqa_attention`` follows ``gqa_attention_fast`` (``ccut/blocks/attn_gqa.py:127-153``), the
  function the reference's attention layer calls (``ccut/models/generic.py:343``): fp32
  scores ``q . k * scale`` (``scale = 1/sqrt(d)``), additive mask, row max subtracted,
  ``exp``, entries whose shifted score is below -1e29 set to 0, normalised by
  ``max(sum, 1e-30)``, then ``probs @ v``.  Query head ``h`` reads kv head ``h // (heads /
  kv_heads)``.  The optional ``softcap`` (``tanh(s / c) * c`` before the mask) is the
  parameter of the per-token variant ``gqa_attention`` (``:76-124``).
* ``causal_mask`` follows ``build_causal_mask`` (``:65-73``): query ``i`` of a batch that
  starts at absolute position ``start_pos`` sees kv positions ``<= start_pos + i``.
* ``rms_norm`` follows ``ccut/blocks/norm.py:14-26``: ``x * (mean(x^2) + eps) ** -0.5 * w``
  in fp32.
* ``apply_rope`` follows ``ccut/blocks/rope.py:130-175``: half rotation with
  ``freqs = positions * inv_freq`` (fp32), ``x1 * cos - x2 * sin`` and ``x2 * cos + x1 * sin``
  over the two halves of the head dim, q first scaled by the attention factor for the
  ``yarn`` / ``linear`` scalings; q ``[batch, heads, seq, d]``, k ``[batch, kv_heads, seq,
  d]``, positions ``[batch, seq]``.
* ``mla_attention`` follows ``mla_prefill`` / ``mla_decode`` (``ccut/blocks/attn_mla.py:85-167``):
  over a latent cache ``c [kv_len, rank]`` and ``k_pe [kv_len, d_rope]``, head h scores
  ``(c @ k_up)[:, h] . q_nope[h] + k_pe . q_pe[h]`` times ``scale``, query row s of a batch that
  starts at ``start_pos`` sees ``min(start_pos + s + 1, kv_len)`` positions, and the output is
  ``softmax @ (c @ v_up)[:, h]``.  ``mla_attention_absorbed`` computes the same through the
  latent space (``q_nope`` folded into ``k_up``, the output unfolded through ``v_up``), the
  form a GPU kernel streams.
"""

from __future__ import annotations

import numpy as np

__all__ = ["apply_rope", "causal_mask", "gqa_attention", "mla_attention", "mla_attention_absorbed", "rms_norm"]


def causal_mask(seq_len: int, start_pos: int) -> np.ndarray:
    """[seq_len, start_pos + seq_len] float32: 0 where visible, -1e30 where masked."""
    q_idx = np.arange(start_pos, start_pos + seq_len)[:, None]
    kv_idx = np.arange(start_pos + seq_len)[None, :]
    m = np.zeros((seq_len, start_pos + seq_len), dtype=np.float32)
    m[kv_idx > q_idx] = -1e30
    return m


def gqa_attention(q, k, v, mask=None, scale=None, softcap=None) -> np.ndarray:
    """q [b, heads, s, d], k / v [b, kv_heads, kv_len, d] -> [b, heads, s, d] float32."""
    q32 = np.asarray(q, dtype=np.float32)
    k32 = np.asarray(k, dtype=np.float32)
    v32 = np.asarray(v, dtype=np.float32)
    b, heads, s, d = q32.shape
    kvh = k32.shape[1]
    if heads % kvh:
        raise ValueError(f"heads ({heads}) must be a multiple of kv_heads ({kvh})")
    g = heads // kvh
    scale = scale or 1.0 / np.sqrt(d)
    if g > 1:
        k32 = np.repeat(k32, g, axis=1)
        v32 = np.repeat(v32, g, axis=1)
    scores = np.einsum("bhqd,bhkd->bhqk", q32, k32) * np.float32(scale)
    if softcap is not None:
        scores = (np.tanh(scores / np.float32(softcap)) * np.float32(softcap)).astype(np.float32)
    if mask is not None:
        scores = scores + np.asarray(mask, dtype=np.float32)
    scores = scores - scores.max(axis=-1, keepdims=True)
    ex = np.exp(scores)
    ex[scores < -1e29] = 0.0
    probs = ex / np.maximum(ex.sum(axis=-1, keepdims=True), 1e-30)
    return np.einsum("bhqk,bhkd->bhqd", probs, v32).astype(np.float32)


def rms_norm(x, weight=None, eps: float = 1e-6) -> np.ndarray:
    x32 = np.asarray(x, dtype=np.float32)
    var = np.mean(x32 * x32, axis=-1, keepdims=True)
    y = x32 * (var + np.float32(eps)) ** np.float32(-0.5)
    if weight is not None:
        y = y * np.asarray(weight, dtype=np.float32)
    return y.astype(np.float32)


def apply_rope(q, k, inv_freq, positions, attention_factor: float = 1.0, scaling_type: str = "none"):
    q32 = np.asarray(q, dtype=np.float32)
    k32 = np.asarray(k, dtype=np.float32)
    freqs = np.asarray(positions).astype(np.float32)[..., None] * np.asarray(inv_freq, np.float32)[None, None, :]
    if scaling_type in ("yarn", "linear") and attention_factor != 1.0:
        q32 = q32 * np.float32(attention_factor)
    cos = np.cos(freqs)[:, None, :, :]
    sin = np.sin(freqs)[:, None, :, :]

    def rot(x):
        half = x.shape[-1] // 2
        x1, x2 = x[..., :half], x[..., half:]
        out = np.empty_like(x)
        out[..., :half] = x1 * cos - x2 * sin
        out[..., half:] = x2 * cos + x1 * sin
        return out

    return rot(q32), rot(k32)


def _mla_probs(scores: np.ndarray, seq: int, kv_len: int, start_pos: int) -> np.ndarray:
    """scores [seq, heads, kv_len] (already scaled) -> causal softmax probabilities."""
    vis = np.minimum(start_pos + np.arange(seq) + 1, kv_len)
    masked = np.arange(kv_len)[None, :] >= vis[:, None]  # [seq, kv_len]
    scores = np.where(masked[:, None, :], np.float32(-1e30), scores).astype(np.float32)
    scores = scores - scores.max(axis=-1, keepdims=True)
    ex = np.exp(scores)
    ex[scores < -1e29] = 0.0
    return (ex / np.maximum(ex.sum(axis=-1, keepdims=True), 1e-30)).astype(np.float32)


def mla_attention(c, k_pe, q_nope, q_pe, k_up, v_up, scale: float, start_pos: int) -> np.ndarray:
    """c [kv_len, rank], k_pe [kv_len, d_rope], q_nope [seq, heads, d_nope], q_pe [seq, heads,
    d_rope], k_up [rank, heads * d_nope], v_up [rank, heads * d_v] -> [seq, heads, d_v]."""
    c, k_pe = np.asarray(c, np.float32), np.asarray(k_pe, np.float32)
    q_nope, q_pe = np.asarray(q_nope, np.float32), np.asarray(q_pe, np.float32)
    seq, heads, d_nope = q_nope.shape
    kv_len = c.shape[0]
    k = (c @ np.asarray(k_up, np.float32)).reshape(kv_len, heads, d_nope)
    v = (c @ np.asarray(v_up, np.float32)).reshape(kv_len, heads, -1)
    scores = (np.einsum("shd,khd->shk", q_nope, k) + np.einsum("shd,kd->shk", q_pe, k_pe)) * np.float32(scale)
    probs = _mla_probs(scores, seq, kv_len, start_pos)
    return np.einsum("shk,khd->shd", probs, v).astype(np.float32)


def mla_attention_absorbed(c, k_pe, q_nope, q_pe, k_up, v_up, scale: float, start_pos: int) -> np.ndarray:
    """``mla_attention`` through the latent space: q_lat[s, h] = k_up_h @ q_nope[s, h] (rank),
    scores = q_lat . c + q_pe . k_pe, o_lat = probs @ c, out = o_lat @ v_up_h."""
    c, k_pe = np.asarray(c, np.float32), np.asarray(k_pe, np.float32)
    q_nope, q_pe = np.asarray(q_nope, np.float32), np.asarray(q_pe, np.float32)
    seq, heads, d_nope = q_nope.shape
    rank, kv_len = c.shape[1], c.shape[0]
    ku = np.asarray(k_up, np.float32).reshape(rank, heads, d_nope)
    vu = np.asarray(v_up, np.float32).reshape(rank, heads, -1)
    q_lat = np.einsum("shd,rhd->shr", q_nope, ku)
    scores = (np.einsum("shr,kr->shk", q_lat, c) + np.einsum("shd,kd->shk", q_pe, k_pe)) * np.float32(scale)
    probs = _mla_probs(scores, seq, kv_len, start_pos)
    o_lat = np.einsum("shk,kr->shr", probs, c)
    return np.einsum("shr,rhd->shd", o_lat, vu).astype(np.float32)
