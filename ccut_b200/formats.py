"""Checkpoint tensors of one quantized matrix -> the inputs of ``ccut_pack_matrix``.

Four formats (``_lib.FORMATS``), each accepted per matrix as a mapping or an object with
attributes, numpy arrays or torch tensors:

``awq_int4_g128``  ``qweight`` int32 [K, N/8], ``qzeros`` int32 [K/128, N/8], ``scales`` fp16
                   [K/128, N] (AutoAWQ, ``[in, out]``).
``fp8_b128``       ``weight`` e4m3 [N, K], ``scale`` / ``weight_scale_inv`` fp32
                   [N/128, K/128] (DeepSeek block FP8, ``[out, in]``).
``fp8_channel``    ``weight`` e4m3 [N, K] with ``scale`` / ``weight_scale`` fp32 per output
                   channel: [N], [N, 1] (compressed-tensors ``channel``) or one value
                   (``tensor``) -- the reference's own FP8 (``fp8_dequant_mat``,
                   ``ccut/quant/kernels.py:150-171``); or ``scales`` fp32 [K/128, N] (one
                   scale per output channel per 128-k group).
``int4_sym_g128``  the reference's signed int4 W4A16 (``ccut/quant/weight_only.py:37-54``):
                   ``weight`` uint8 [N, K/2] (low nibble = even input column) with ``scale`` /
                   ``weight_scale`` fp32 [K] (one per input column, constant within each
                   128-column group); or ``qweight`` int32 [K, N/8] holding ``v + 8`` in AWQ's
                   nibble order with ``scales`` fp32 [K/128, N].

``canonical`` brings a matrix to one form per format (the second form of each of the last
two), the ``slice_*`` helpers cut the intermediate channels of shared-expert slices, and
``pack_args`` uploads the tensors ``ccut_pack_matrix`` reads.  Conversions move bytes and
repeat scales only: every format dequantizes to the same fp32 values before and after.
"""

from __future__ import annotations

import warnings

import numpy as np
import torch

__all__ = ["FORMATS", "canonical", "repacked", "slice_out", "slice_in", "pack_args", "int4_sym_from_reference",
           "awq_words", "awq_columns"]

FORMATS = ("awq_int4_g128", "fp8_b128", "fp8_channel", "int4_sym_g128")

# nibble slot i (bits 4i .. 4i + 3) of an AWQ qweight / qzeros word holds column _AWQ_COL_OF_SLOT[i]
# of its group of 8 output channels (the AutoAWQ checkpoint layout)
_AWQ_COL_OF_SLOT = (0, 2, 4, 6, 1, 3, 5, 7)


def _get(m, *names, default=KeyError):
    for n in names:
        if isinstance(m, dict) and n in m:
            return m[n]
        if not isinstance(m, dict) and hasattr(m, n):
            return getattr(m, n)
    if default is KeyError:
        raise KeyError(f"checkpoint matrix lacks any of {names}")
    return default


def _has(m, name) -> bool:
    return (name in m) if isinstance(m, dict) else hasattr(m, name)


def _np(a) -> np.ndarray:
    return a.detach().cpu().numpy() if isinstance(a, torch.Tensor) else np.asarray(a)


def awq_columns(words) -> np.ndarray:
    """int32 ``[rows, N / 8]`` AWQ words -> uint8 ``[rows, N]`` nibbles in column order."""
    w = np.ascontiguousarray(_np(words)).view(np.uint32)
    out = np.empty(w.shape + (8,), np.uint8)
    for slot, col in enumerate(_AWQ_COL_OF_SLOT):
        out[..., col] = (w >> np.uint32(4 * slot)) & np.uint32(15)
    return out.reshape(w.shape[0], -1)


def awq_words(cols: np.ndarray) -> np.ndarray:
    """The inverse of ``awq_columns``."""
    c = np.asarray(cols).reshape(cols.shape[0], -1, 8).astype(np.uint32)
    w = np.zeros(c.shape[:2], np.uint32)
    for slot, col in enumerate(_AWQ_COL_OF_SLOT):
        w |= c[..., col] << np.uint32(4 * slot)
    return w.view(np.int32)


def int4_sym_from_reference(weight, scale) -> dict:
    """The reference's signed int4 matrix (``weight`` uint8 [N, K/2], two signed nibbles per
    byte, low nibble = even input column; ``scale`` fp32 [K], one per input column) as
    ``{"qweight": int32 [K, N/8] of v + 8 in AWQ's nibble order, "scales": fp32 [K/128, N]}``.
    ``ValueError`` when a scale varies inside a 128-column group: the kernels multiply the
    exact integer codes and apply one fp32 scale per channel per 128-k group."""
    p = np.ascontiguousarray(_np(weight), dtype=np.uint8)
    s = np.ascontiguousarray(_np(scale), dtype=np.float32).reshape(-1)
    N, K = p.shape[0], p.shape[1] * 2
    if s.shape != (K,) or K % 128:
        raise ValueError(f"int4 weight [{N}, {K // 2}] needs a per-column scale of {K} values (K % 128 == 0), "
                         f"got {s.shape}")
    sg = s.reshape(K // 128, 128)
    if not np.array_equal(sg, np.repeat(sg[:, :1], 128, axis=1)):
        raise ValueError("int4 per-column scales must be constant within each 128-column group")
    q = np.empty((K, N), np.uint8)  # v + 8, [in, out]
    q[0::2] = ((p & 0x0F) ^ 0x08).T  # v + 8 for a signed nibble is the nibble with bit 3 flipped
    q[1::2] = ((p >> 4) ^ 0x08).T
    return {"qweight": awq_words(q), "scales": np.ascontiguousarray(np.repeat(sg[:, :1], N, axis=1))}


def _expand_channel_scale(s, K: int, N: int):
    """fp32 per-output-channel scale ([N], [N, 1] or one value) -> [K/128, N]."""
    if isinstance(s, torch.Tensor):
        t = s.to(torch.float32).reshape(-1)
        if t.numel() == 1:
            t = t.expand(N)
        if t.numel() != N:
            raise ValueError(f"per-channel scale must have {N} values, got {tuple(s.shape)}")
        return t.reshape(1, N).expand(K // 128, N).contiguous()
    a = np.asarray(s, dtype=np.float32).reshape(-1)
    if a.size == 1:
        a = np.full(N, a[0], np.float32)
    if a.shape != (N,):
        raise ValueError(f"per-channel scale must have {N} values, got {np.shape(s)}")
    return np.ascontiguousarray(np.broadcast_to(a[None, :], (K // 128, N)))


def canonical(fmt: str, mat) -> dict:
    """One matrix's checkpoint tensors in the canonical form of ``fmt`` (module docstring)."""
    if fmt == "awq_int4_g128":
        return {"qweight": _get(mat, "qweight"), "qzeros": _get(mat, "qzeros", "zeros"), "scales": _get(mat, "scales")}
    if fmt == "fp8_b128":
        return {"weight": _get(mat, "weight"), "scale": _get(mat, "scale", "weight_scale_inv")}
    if fmt == "fp8_channel":
        w = _get(mat, "weight")
        N, K = int(w.shape[0]), int(w.shape[1])
        if _has(mat, "scales"):
            return {"weight": w, "scales": _get(mat, "scales")}
        return {"weight": w, "scales": _expand_channel_scale(_get(mat, "scale", "weight_scale"), K, N)}
    if fmt == "int4_sym_g128":
        if _has(mat, "qweight"):
            return {"qweight": _get(mat, "qweight"), "scales": _get(mat, "scales")}
        return int4_sym_from_reference(_get(mat, "weight"), _get(mat, "scale", "weight_scale"))
    raise NotImplementedError(f"weight format {fmt!r} is not supported (have {sorted(FORMATS)})")


def repacked(fmt: str, mat) -> bool:
    """True when ``canonical`` builds new int4 words for ``mat`` (they are in AWQ's nibble
    order whatever order the caller's own ``qweight`` tensors use)."""
    return fmt == "int4_sym_g128" and not _has(mat, "qweight")


def slice_out(fmt: str, t: dict, lo: int, width: int) -> dict:
    """Output channels [lo, lo + width) of a canonical matrix (``width`` % 128 == 0)."""
    if fmt in ("awq_int4_g128", "int4_sym_g128"):
        out = {"qweight": t["qweight"][:, lo // 8:(lo + width) // 8], "scales": t["scales"][:, lo:lo + width]}
        if "qzeros" in t:
            out["qzeros"] = t["qzeros"][:, lo // 8:(lo + width) // 8]
        return out
    if fmt == "fp8_b128":
        return {"weight": t["weight"][lo:lo + width], "scale": t["scale"][lo // 128:(lo + width) // 128]}
    return {"weight": t["weight"][lo:lo + width], "scales": t["scales"][:, lo:lo + width]}


def slice_in(fmt: str, t: dict, lo: int, width: int) -> dict:
    """Input channels [lo, lo + width) of a canonical matrix (``lo``, ``width`` % 128 == 0)."""
    g0, g1 = lo // 128, (lo + width) // 128
    if fmt in ("awq_int4_g128", "int4_sym_g128"):
        out = {"qweight": t["qweight"][lo:lo + width], "scales": t["scales"][g0:g1]}
        if "qzeros" in t:
            out["qzeros"] = t["qzeros"][g0:g1]
        return out
    if fmt == "fp8_b128":
        return {"weight": t["weight"][:, lo:lo + width], "scale": t["scale"][:, g0:g1]}
    return {"weight": t["weight"][:, lo:lo + width], "scales": t["scales"][g0:g1]}


def _dev(a, device, dtype) -> torch.Tensor:
    if isinstance(a, torch.Tensor):
        t = a
    else:
        a = np.ascontiguousarray(a)
        with warnings.catch_warnings():  # read-only views (mmap'd checkpoints) are only read
            warnings.simplefilter("ignore", UserWarning)
            t = torch.from_numpy(a)
    if t.dtype != dtype:
        t = t.view(dtype) if t.element_size() == torch.empty((), dtype=dtype).element_size() else t.to(dtype)
    return t.to(device, non_blocking=False).contiguous()


def pack_args(fmt: str, t: dict, K: int, N: int, device, what: str = "matrix"):
    """Device tensors (q, z, s) of a canonical matrix for ``ccut_pack_matrix`` (z is None when
    the format has no zero points), with their shapes checked against K inputs x N outputs."""
    if fmt in ("awq_int4_g128", "int4_sym_g128"):
        f16 = fmt == "awq_int4_g128"
        q = _dev(t["qweight"], device, torch.int32)
        z = _dev(t["qzeros"], device, torch.int32) if f16 else None
        s = _dev(t["scales"], device, torch.float16 if f16 else torch.float32)
        if tuple(q.shape) != (K, N // 8) or tuple(s.shape) != (K // 128, N) or (
                z is not None and tuple(z.shape) != (K // 128, N // 8)):
            raise ValueError(f"{what}: {fmt} tensors have shapes q{tuple(q.shape)} s{tuple(s.shape)} for K={K} N={N}")
        return q, z, s
    q = _dev(t["weight"], device, torch.uint8)
    if fmt == "fp8_b128":
        s = _dev(t["scale"], device, torch.float32)
        want = (N // 128, K // 128)
    else:
        s = _dev(t["scales"], device, torch.float32)
        want = (K // 128, N)
    if tuple(q.shape) != (N, K) or tuple(s.shape) != want:
        raise ValueError(f"{what}: {fmt} tensors have shapes w{tuple(q.shape)} s{tuple(s.shape)} for K={K} N={N}")
    return q, None, s
