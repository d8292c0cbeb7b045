"""Weight formats of the MoE expert path (CPU restatement, test infrastructure only).

AWQ int4, group 128 along K
    Checkpoint layout (AutoAWQ "GEMM" format, [in, out] = [K, N]):
      ``qweight`` int32 [K, N/8]      8 unsigned nibbles per word, packed along N
      ``qzeros``  int32 [K/128, N/8]  zero-points, packed the same way
      ``scales``  fp16  [K/128, N]
    ``w[k, n] = (q[k, n] - z[k // 128, n]) * s[k // 128, n]`` evaluated in fp32.  The
    product of a 5-bit integer and an fp16 scale fits fp32's mantissa, so the dequantized
    value is exact (order independent) and a GPU export can match it bit for bit.
    The nibble extraction follows the reference's low-nibble-first int4 unpack
    (``ccut/quant/kernels.py:276-295``); unlike the reference's signed per-column int4
    (``int4_w4a16_sym``, ``ccut/quant/spec.py:145``) the nibbles are unsigned with an
    explicit zero-point, as AWQ checkpoints store them.  Within a word, nibble slot ``i``
    (bits ``4i..4i+3``) holds column ``AWQ_ORDER[i]`` of its 8-column group (AutoAWQ's
    interleave); ``order="sequential"`` selects slot ``i`` = column ``i``.

FP8 e4m3, 128x128 blocks
    Checkpoint layout (DeepSeek-V3 "fp8" format, [out, in] = [N, K]):
      ``weight``  uint8 (e4m3fn) [N, K]
      ``scale``   fp32 [ceil(N/128), ceil(K/128)]   (``weight_scale_inv``)
    ``w[n, k] = e4m3(b[n, k]) * scale[n // 128, k // 128]`` in fp32.  The e4m3 decode is
    the reference's bit-level decode (``ccut/quant/kernels.py:52-74``): bias 7, subnormal
    ``m/8 * 2^-6``, 0x7F / 0xFF = NaN, no infinities.  The reference only implements the
    per-row scaled variant (``ccut/quant/kernels.py:150-171``); the block variant is a
    restatement (the reference's ``Fp8Config`` raises, ``ccut/quant/fp8.py:37-51``).

FP8 e4m3, one scale per output channel (the reference's own FP8)
    ``weight`` uint8 [N, K], ``scale`` fp32 [N]:
    ``w[n, k] = e4m3(b[n, k]) * scale[n]``, ``fp8_dequant_mat`` (``ccut/quant/kernels.py:
    150-171``; ``fp8_static_channel_sym``, ``ccut/quant/spec.py:139``).

Signed int4 weight-only (the reference's ``int4_w4a16_sym``)
    ``weight`` uint8 [N, K/2] (two signed nibbles per byte, low nibble = even column),
    ``scale`` fp32 [K] (one per input column): ``w[n, k] = v[n, k] * scale[k]``,
    ``int4_dequant_row`` (``ccut/quant/kernels.py:277-295``) as ``WeightOnlyMethod.apply``
    calls it (``ccut/quant/weight_only.py:37-54``).
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "GROUP",
    "BLOCK",
    "AWQ_ORDER",
    "FP8_E4M3_TABLE",
    "awq_pack",
    "awq_unpack",
    "awq_dequant",
    "fp8_e4m3_decode",
    "fp8_e4m3_encode",
    "fp8_block_dequant",
    "fp8_channel_dequant",
    "int4_sym_unpack",
    "int4_sym_dequant",
    "bf16_bits_from_f32",
    "bf16_bits_to_f32",
]

GROUP = 128
BLOCK = 128
#: nibble slot i of an AWQ word holds column AWQ_ORDER[i] of its 8-column group
AWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)
SEQ_ORDER = tuple(range(8))


def _order(order: str | tuple) -> tuple:
    if isinstance(order, tuple):
        return order
    if order == "awq":
        return AWQ_ORDER
    if order == "sequential":
        return SEQ_ORDER
    raise ValueError(f"unknown nibble order {order!r}")


def awq_pack(vals: np.ndarray, order: str | tuple = "awq") -> np.ndarray:
    """Pack unsigned nibbles ``vals`` uint8 [R, C] (C % 8 == 0) into int32 [R, C/8]."""
    vals = np.asarray(vals)
    if vals.ndim != 2 or vals.shape[1] % 8:
        raise ValueError("awq_pack expects [R, C] with C a multiple of 8")
    if vals.size and (vals.min() < 0 or vals.max() > 15):
        raise ValueError("nibbles must lie in [0, 15]")
    o = _order(order)
    v = vals.astype(np.uint32).reshape(vals.shape[0], -1, 8)
    word = np.zeros(v.shape[:2], dtype=np.uint32)
    for slot in range(8):
        word |= v[:, :, o[slot]] << np.uint32(4 * slot)
    return word.view(np.int32)


def awq_unpack(packed: np.ndarray, order: str | tuple = "awq") -> np.ndarray:
    """Inverse of :func:`awq_pack`: int32 [R, C/8] -> uint8 [R, C].

    Low nibble first, as ``ccut/quant/kernels.py:287-289`` extracts nibbles."""
    o = _order(order)
    w = np.ascontiguousarray(packed).view(np.uint32)
    out = np.empty((w.shape[0], w.shape[1], 8), dtype=np.uint8)
    for slot in range(8):
        out[:, :, o[slot]] = (w >> np.uint32(4 * slot)) & np.uint32(0xF)
    return out.reshape(w.shape[0], w.shape[1] * 8)


def awq_dequant(
    qweight: np.ndarray,
    qzeros: np.ndarray,
    scales: np.ndarray,
    group: int = GROUP,
    order: str | tuple = "awq",
) -> np.ndarray:
    """AWQ int4 -> fp32 [K, N] (``[in, out]``, the ``[hidden, inter]`` layout that
    ``expert_ffn`` consumes, ``ccut/blocks/moe.py:128-132``)."""
    q = awq_unpack(qweight, order).astype(np.float32)  # [K, N]
    z = awq_unpack(qzeros, order).astype(np.float32)  # [K/g, N]
    s = np.asarray(scales, dtype=np.float16).astype(np.float32)  # [K/g, N]
    K, N = q.shape
    if K % group or z.shape != (K // group, N) or s.shape != (K // group, N):
        raise ValueError(f"inconsistent AWQ shapes q{q.shape} z{z.shape} s{s.shape}")
    zz = np.repeat(z, group, axis=0)
    ss = np.repeat(s, group, axis=0)
    return ((q - zz) * ss).astype(np.float32)


def _build_e4m3_table() -> np.ndarray:
    """Decode table of all 256 e4m3fn codes, following ``ccut/quant/kernels.py:52-74``."""
    out = np.empty(256, dtype=np.float32)
    for b in range(256):
        sign = -1.0 if (b & 0x80) else 1.0
        exp = (b >> 3) & 0x0F
        mant = b & 0x07
        if exp == 0:
            val = (mant * 0.125) * (2.0 ** -6)
        elif exp == 15 and mant == 7:
            val = np.nan
        else:
            val = (1.0 + mant * 0.125) * (2.0 ** (exp - 7))
        out[b] = sign * val
    return out


FP8_E4M3_TABLE = _build_e4m3_table()


def fp8_e4m3_decode(codes: np.ndarray) -> np.ndarray:
    """uint8 e4m3fn codes -> fp32 (table lookup, bit-identical to the reference decode)."""
    return FP8_E4M3_TABLE[np.asarray(codes, dtype=np.uint8)]


# positive finite codes 0x00..0x7E are strictly increasing in value
_POS_VALS = FP8_E4M3_TABLE[:0x7F].astype(np.float64)


def fp8_e4m3_encode(x: np.ndarray) -> np.ndarray:
    """fp32 -> e4m3fn codes, round-to-nearest-even, saturating at +-448, NaN -> 0x7F.

    Used only to synthesise weights (the reference's own encoder rounds half up,
    ``ccut/quant/kernels.py:77-123``; generation needs no particular tie rule)."""
    x = np.asarray(x, dtype=np.float32)
    a = np.minimum(np.abs(x).astype(np.float64), 448.0)
    hi = np.searchsorted(_POS_VALS, a, side="left")  # first value >= a
    hi = np.minimum(hi, 0x7E)
    lo = np.maximum(hi - 1, 0)
    dlo = a - _POS_VALS[lo]
    dhi = _POS_VALS[hi] - a
    pick_hi = (dhi < dlo) | ((dhi == dlo) & ((hi & 1) == 0))
    code = np.where(pick_hi, hi, lo).astype(np.uint8)
    code = np.where(np.signbit(x), code | np.uint8(0x80), code)
    code = np.where(np.isnan(x), np.uint8(0x7F), code)
    return code.astype(np.uint8)


def fp8_block_dequant(w: np.ndarray, scale: np.ndarray, block: int = BLOCK) -> np.ndarray:
    """FP8 e4m3 block-scaled -> fp32 [N, K] (``[out, in]``): one fp32 multiply per element."""
    w = np.asarray(w, dtype=np.uint8)
    N, K = w.shape
    nb, kb = (N + block - 1) // block, (K + block - 1) // block
    scale = np.asarray(scale, dtype=np.float32)
    if scale.shape != (nb, kb):
        raise ValueError(f"scale shape {scale.shape} != {(nb, kb)}")
    sfull = np.repeat(np.repeat(scale, block, axis=0), block, axis=1)[:N, :K]
    return (fp8_e4m3_decode(w) * sfull).astype(np.float32)


def fp8_channel_dequant(w: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """Per-output-channel FP8 -> fp32 [N, K] (``[out, in]``), following ``fp8_dequant_mat``
    (``ccut/quant/kernels.py:150-171``): ``out[n, k] = e4m3(w[n, k]) * scale[n]``.  The exact
    product of an e4m3 value and an fp32 scale has at most 28 significant bits, so the
    reference's float64 product rounded once to fp32 equals this fp32 multiply."""
    w = np.asarray(w, dtype=np.uint8)
    scale = np.asarray(scale, dtype=np.float32).reshape(-1)
    if scale.shape != (w.shape[0],):
        raise ValueError(f"scale shape {scale.shape} != ({w.shape[0]},)")
    return (fp8_e4m3_decode(w) * scale[:, None]).astype(np.float32)


def int4_sym_unpack(packed: np.ndarray) -> np.ndarray:
    """uint8 [N, K/2] of two signed nibbles (low nibble = even column) -> int8 [N, K] in
    [-8, 7], as ``int4_dequant_row`` reads them (``ccut/quant/kernels.py:283-293``)."""
    p = np.asarray(packed, dtype=np.uint8)
    v = np.empty((p.shape[0], p.shape[1] * 2), dtype=np.int8)
    lo, hi = (p & 0x0F).astype(np.int8), (p >> 4).astype(np.int8)
    v[:, 0::2] = np.where(lo >= 8, lo - 16, lo)
    v[:, 1::2] = np.where(hi >= 8, hi - 16, hi)
    return v


def int4_sym_dequant(packed: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """Signed int4 weight-only -> fp32 [N, K] (``[out, in]``), following ``int4_dequant_row``
    (``ccut/quant/kernels.py:277-295``): ``out[n, k] = v[n, k] * scale[k]``."""
    v = int4_sym_unpack(packed)
    scale = np.asarray(scale, dtype=np.float32).reshape(-1)
    if scale.shape != (v.shape[1],):
        raise ValueError(f"scale shape {scale.shape} != ({v.shape[1]},)")
    return (v.astype(np.float32) * scale[None, :]).astype(np.float32)


def bf16_bits_from_f32(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round-to-nearest-even (NaN kept quiet)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rnd = ((u >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    out = ((u + rnd) >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    return np.where(nan, np.uint16(0x7FC0), out).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    """bf16 bit patterns -> fp32 by the 16-bit shift of ``ccut/io_/safetensors_io.py:53-57``."""
    u = np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)
    return u.view(np.float32)
