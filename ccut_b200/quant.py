"""``QuantizeMethodBase``-compatible linear methods for the two new weight formats.

Mirrors the reference's method interface (``ccut/quant/method.py:27-62``):
``create_weights(spec)`` checks the scale tensors once, ``apply(weight_bytes, scales, x)``
returns ``y = x @ dequant(W)`` as fp32 ``[batch, out]``, and
``process_weights_after_loading()`` is a hook.  ``apply`` packs the weight into the kernel
tile layout on its first call (cached per weight buffer) and then runs
``ccut_quant_linear`` on the GPU.  numpy in gives numpy out; torch in gives torch out.

Formats (no reference implementation; the nearest reference methods are
``ccut/quant/weight_only.py:37-54`` and ``ccut/quant/fp8.py:37-51``):
  AWQ int4 g128    weight = qweight int32 [in, out/8]; scales = {"scales": fp16 [in/128, out],
                   "qzeros": int32 [in/128, out/8]}
  FP8 e4m3 b128    weight = e4m3 bytes [out, in]; scales = {"weight_scale_inv" (or "scale"):
                   fp32 [out/128, in/128]}
Missing scales raise ``ValueError`` and unknown formats ``NotImplementedError``, as in the
reference.
"""

from __future__ import annotations

import numpy as np
import torch

from ccut_b200 import _lib
from ccut_b200.layer import _dev, _ptr, _stream

__all__ = ["QuantizeMethodBase", "AwqInt4G128Method", "Fp8Block128Method", "make_method", "dequantize",
           "QuantLinear", "cat_checkpoint_tensors", "permute_out_channels", "pad_out_channels", "ct_int4_to_awq"]


class QuantizeMethodBase:
    """Interface of the reference's quantize methods."""

    compute_path = "bf16"

    def create_weights(self, spec=None) -> None:
        return None

    def apply(self, weight_bytes, scales: dict, x):
        raise NotImplementedError

    def process_weights_after_loading(self) -> None:
        return None


class _PackedLinear(QuantizeMethodBase):
    fmt = ""
    scale_names: tuple[tuple[str, ...], ...] = ()

    def __init__(self, in_features: int, out_features: int, layout: str = "frags", device="cuda"):
        if in_features % 128 or out_features % 128:
            raise ValueError("in_features and out_features must be multiples of 128")
        if layout not in _lib.LAYOUTS:
            raise NotImplementedError(f"layout {layout!r} is not supported (have {sorted(_lib.LAYOUTS)})")
        self.K, self.N = int(in_features), int(out_features)
        self.layout = layout
        self.device = torch.device(device)
        self.lib = _lib.load()
        self.code = _lib.FORMATS[self.fmt]
        self._packed: dict = {}
        self._ws: torch.Tensor | None = None

    def create_weights(self, spec=None) -> None:
        names = getattr(spec, "scales", None)
        if spec is not None and not names:
            raise ValueError(f"{getattr(spec, 'layer_name', 'layer')}: quantized layer has no scale tensors")

    def _scale(self, scales: dict, names: tuple[str, ...]):
        for n in names:
            if n in scales:
                return scales[n]
        raise ValueError(f"missing scale tensor (one of {names})")

    def _pack(self, weight_bytes, scales: dict) -> torch.Tensor:
        key = (id(weight_bytes), tuple(id(scales.get(n)) for group in self.scale_names for n in group))
        hit = self._packed.get(key)
        if hit is not None:
            return hit[0]
        q, z, s = self._tensors(weight_bytes, scales)
        packed = torch.empty(self.lib.ccut_packed_matrix_bytes(self.code, self.K, self.N), dtype=torch.uint8,
                             device=self.device)
        with torch.cuda.device(self.device):
            _lib.call("ccut_pack_matrix", self.code, _lib.LAYOUTS[self.layout], _ptr(q), _ptr(z), _ptr(s), self.K,
                      self.N, _lib.NIBBLES_AWQ, _ptr(packed), 1, 0, _stream())
        self._packed[key] = (packed, weight_bytes)  # keep the source alive: its id is the key
        return packed

    def apply(self, weight_bytes, scales: dict, x):
        packed = self._pack(weight_bytes, scales)
        was_np = not isinstance(x, torch.Tensor)
        xt = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)) if was_np else x
        if xt.dim() != 2 or xt.shape[1] != self.K:
            raise ValueError(f"x must be [batch, {self.K}], got {tuple(xt.shape)}")
        xb = xt.to(self.device, torch.bfloat16).contiguous()
        M = xb.shape[0]
        y = torch.empty((M, self.N), dtype=torch.float32, device=self.device)
        if M:
            nbytes = self.lib.ccut_quant_linear_workspace_bytes(self.code, M, self.K)
            if self._ws is None or self._ws.numel() < nbytes:
                self._ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
            with torch.cuda.device(self.device):
                _lib.call("ccut_quant_linear", self.code, _lib.LAYOUTS[self.layout], _ptr(packed), self.K, self.N,
                          _ptr(xb), M, _ptr(y), _ptr(self._ws), self._ws.numel(), _stream())
        return y.cpu().numpy() if was_np else y


class AwqInt4G128Method(_PackedLinear):
    """W4A16: unsigned int4 weights, group-128 zero-points and fp16 scales along the input."""

    compute_path = "w4a16"
    fmt = "awq_int4_g128"
    scale_names = (("scales",), ("qzeros", "zeros"))

    def _tensors(self, weight_bytes, scales):
        q = _as_array(weight_bytes, np.int32).reshape(self.K, self.N // 8)
        s = np.asarray(self._scale(scales, ("scales",)), dtype=np.float16).reshape(self.K // 128, self.N)
        z = np.asarray(self._scale(scales, ("qzeros", "zeros")), dtype=np.int32).reshape(self.K // 128, self.N // 8)
        return (_dev(q, self.device, torch.int32), _dev(z, self.device, torch.int32),
                _dev(s, self.device, torch.float16))


class Fp8Block128Method(_PackedLinear):
    """W8A16: e4m3 weights with one fp32 scale per 128 x 128 block."""

    compute_path = "w8a16"
    fmt = "fp8_b128"
    scale_names = (("weight_scale_inv", "scale"),)

    def _tensors(self, weight_bytes, scales):
        w = _as_array(weight_bytes, np.uint8).reshape(self.N, self.K)
        s = np.asarray(self._scale(scales, ("weight_scale_inv", "scale")), dtype=np.float32).reshape(
            self.N // 128, self.K // 128)
        return _dev(w, self.device, torch.uint8), None, _dev(s, self.device, torch.float32)


def _as_array(b, dtype) -> np.ndarray:
    if isinstance(b, torch.Tensor):
        return b.detach().cpu().numpy().view(dtype)
    if isinstance(b, (bytes, bytearray, memoryview)):
        return np.frombuffer(b, dtype=dtype).copy()
    return np.asarray(b).view(dtype)


def make_method(fmt: str, in_features: int, out_features: int, **kw) -> QuantizeMethodBase:
    """Format name -> method (``"awq_int4_g128"`` | ``"fp8_b128"``)."""
    if fmt == "awq_int4_g128":
        return AwqInt4G128Method(in_features, out_features, **kw)
    if fmt == "fp8_b128":
        return Fp8Block128Method(in_features, out_features, **kw)
    raise NotImplementedError(f"weight format {fmt!r} is not supported")


def dequantize(fmt: str, weight_bytes, scales: dict, in_features: int, out_features: int,
               device="cuda") -> torch.Tensor:
    """fp32 ``[out, in]`` of one checkpoint matrix (the tensors ``apply`` takes), on the device:
    packed with ``ccut_pack_matrix``, exported with ``ccut_dequant_matrix`` (``(q - z) * s`` /
    ``e4m3 * scale``, bit-identical to the checkpoint dequant)."""
    m = make_method(fmt, in_features, out_features, layout="rows", device=device)
    packed = m._pack(weight_bytes, scales)
    out = torch.empty((m.K, m.N), dtype=torch.float32, device=m.device)
    with torch.cuda.device(m.device):
        _lib.call("ccut_dequant_matrix", m.code, _lib.LAYOUTS["rows"], _ptr(packed), m.K, m.N, 1, 0, _ptr(out),
                  _stream())
    return out.t()


# checkpoint tensor names of one matrix per format: the weight, then its scale tensors, with the
# axis along which the output channels run in each
_TENSORS = {"awq_int4_g128": (("qweight", 1), ("qzeros", 1), ("scales", 1)),
            "fp8_b128": (("weight", 0), ("weight_scale_inv", 0))}


class QuantLinear:
    """A linear projection ``y = x @ W^T`` kept in its checkpoint format (``W`` [out, in]) and
    run by ``ccut_quant_linear`` (fp32 out) -- a quarter (AWQ) or half (FP8) of the bytes of
    a bf16 copy.  ``tensors``: the checkpoint tensors of the matrix (AWQ ``qweight`` /
    ``qzeros`` / ``scales``; FP8 ``weight`` / ``weight_scale_inv`` or ``scale``).  The
    weight is packed into the kernel layout once, at construction."""

    def __init__(self, fmt: str, tensors: dict, in_features: int, out_features: int, device="cuda",
                 layout: str = "frags"):
        if fmt not in _TENSORS:
            raise NotImplementedError(f"weight format {fmt!r} is not supported")
        t = dict(tensors)
        if fmt == "fp8_b128" and "weight_scale_inv" not in t and "scale" in t:
            t["weight_scale_inv"] = t.pop("scale")
        missing = [n for n, _ in _TENSORS[fmt] if n not in t]
        if missing:
            raise ValueError(f"missing checkpoint tensors {missing}")
        self.fmt, self.in_features, self.out_features = fmt, int(in_features), int(out_features)
        self.tensors = {n: t[n] for n, _ in _TENSORS[fmt]}
        self.method = make_method(fmt, self.in_features, self.out_features, layout=layout, device=device)
        main = _TENSORS[fmt][0][0]
        self._weight = self.tensors[main]
        self._scales = {n: v for n, v in self.tensors.items() if n != main}
        self.method._pack(self._weight, self._scales)
        self.device = self.method.device

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        """x [M, in] (bf16, or converted to bf16) -> fp32 [M, out]."""
        return self.method.apply(self._weight, self._scales, x)

    @classmethod
    def cat(cls, parts: list) -> "QuantLinear":
        """One projection whose outputs are those of ``parts`` side by side (same format and
        input size): the checkpoint tensors concatenated along the output channels."""
        p0 = parts[0]
        if any(p.fmt != p0.fmt or p.in_features != p0.in_features for p in parts):
            raise ValueError("projections to concatenate need the same format and input size")
        return cls(p0.fmt, cat_checkpoint_tensors(p0.fmt, [p.tensors for p in parts]), p0.in_features,
                   sum(p.out_features for p in parts), p0.device, p0.method.layout)


def cat_checkpoint_tensors(fmt: str, parts: list) -> dict:
    """The checkpoint tensors of one matrix whose output channels are those of ``parts`` (each
    a dict of one matrix's tensors) in order: AWQ ``qweight`` / ``qzeros`` / ``scales`` side by
    side along their last axis, FP8 ``weight`` / ``weight_scale_inv`` stacked along the first.
    Each part's output channels must be a multiple of 128 (one FP8 scale block)."""
    if fmt not in _TENSORS:
        raise NotImplementedError(f"weight format {fmt!r} is not supported")
    return {n: np.concatenate([np.asarray(p[n]) for p in parts], axis=ax) for n, ax in _TENSORS[fmt]}


# nibble slot i (bits 4i .. 4i + 3) of an AWQ qweight / qzeros word holds column _AWQ_COL_OF_SLOT[i]
# of its group of 8 output channels (the AutoAWQ checkpoint layout)
_AWQ_COL_OF_SLOT = (0, 2, 4, 6, 1, 3, 5, 7)


def _awq_columns(words: np.ndarray) -> np.ndarray:
    """int32 ``[rows, N / 8]`` AWQ words -> uint8 ``[rows, N]`` nibbles in column order."""
    w = np.ascontiguousarray(words).view(np.uint32)
    out = np.empty(w.shape + (8,), np.uint8)
    for slot, col in enumerate(_AWQ_COL_OF_SLOT):
        out[..., col] = (w >> np.uint32(4 * slot)) & np.uint32(15)
    return out.reshape(w.shape[0], -1)


def _awq_words(cols: np.ndarray) -> np.ndarray:
    """The inverse of ``_awq_columns``."""
    c = cols.reshape(cols.shape[0], -1, 8).astype(np.uint32)
    w = np.zeros(c.shape[:2], np.uint32)
    for slot, col in enumerate(_AWQ_COL_OF_SLOT):
        w |= c[..., col] << np.uint32(4 * slot)
    return w.view(np.int32)


def permute_out_channels(fmt: str, tensors: dict, perm) -> dict:
    """The checkpoint tensors of ``W[perm]`` (output channel ``j`` of the result is channel
    ``perm[j]`` of ``W``), in the same format: AWQ nibbles and scales moved along the output
    axis; FP8 weight rows moved, which needs every row to stay in its 128-row scale block
    (``ValueError`` otherwise).  Byte moves only: the values dequantize to the permuted rows
    exactly."""
    perm = np.asarray(perm, np.int64)
    if fmt == "awq_int4_g128":
        n = tensors["scales"].shape[1]
        if perm.shape != (n,):
            raise ValueError(f"perm must have {n} entries")
        return {"qweight": _awq_words(_awq_columns(tensors["qweight"])[:, perm]),
                "qzeros": _awq_words(_awq_columns(tensors["qzeros"])[:, perm]),
                "scales": np.ascontiguousarray(np.asarray(tensors["scales"])[:, perm])}
    if fmt == "fp8_b128":
        w = np.asarray(tensors["weight"])
        if perm.shape != (w.shape[0],):
            raise ValueError(f"perm must have {w.shape[0]} entries")
        if np.any(perm // 128 != np.arange(perm.size) // 128):
            raise ValueError("an FP8 row permutation must keep every row in its 128-row scale block")
        out = dict(tensors)
        out["weight"] = np.ascontiguousarray(w[perm])
        return out
    raise NotImplementedError(f"weight format {fmt!r} is not supported")


def pad_out_channels(fmt: str, tensors: dict, out_features: int) -> dict:
    """The checkpoint tensors with zero output channels appended up to ``out_features`` (so
    that a matrix whose output size is not a multiple of 128 can be packed and dequantized;
    the padded channels dequantize to 0)."""
    if fmt == "awq_int4_g128":
        s = np.asarray(tensors["scales"])
        extra = out_features - s.shape[1]
        if extra < 0 or extra % 8 or s.shape[1] % 8:
            raise ValueError(f"cannot pad {s.shape[1]} AWQ output channels to {out_features}")

        def pad(a, n):
            a = np.asarray(a)
            return np.concatenate([a, np.zeros((a.shape[0], n), a.dtype)], axis=1)

        return {"qweight": pad(tensors["qweight"], extra // 8), "qzeros": pad(tensors["qzeros"], extra // 8),
                "scales": pad(s, extra)}
    if fmt == "fp8_b128":
        w = np.asarray(tensors["weight"])
        extra = out_features - w.shape[0]
        if extra < 0:
            raise ValueError(f"cannot pad {w.shape[0]} FP8 output channels to {out_features}")
        sc = np.asarray(tensors.get("weight_scale_inv", tensors.get("scale")))
        blocks = -(-out_features // 128)
        sc = np.concatenate([sc, np.ones((blocks - sc.shape[0], sc.shape[1]), sc.dtype)]) if blocks > sc.shape[0] else sc
        return {"weight": np.concatenate([w, np.zeros((extra, w.shape[1]), w.dtype)]), "weight_scale_inv": sc}
    raise NotImplementedError(f"weight format {fmt!r} is not supported")


def _nibbles_sequential(words: np.ndarray) -> np.ndarray:
    """int32 ``[rows, C]`` words holding 8 nibbles each, nibble i in bits 4i .. 4i + 3 ->
    uint8 ``[rows, 8 C]`` in that order."""
    w = np.ascontiguousarray(words).view(np.uint32)
    return np.stack([(w >> np.uint32(4 * i)) & np.uint32(15) for i in range(8)], axis=-1).astype(
        np.uint8).reshape(w.shape[0], -1)


def ct_int4_to_awq(weight_packed, weight_scale, weight_zero_point=None, weight_shape=None,
                   group_size: int = 128) -> dict:
    """A compressed-tensors ``pack-quantized`` int4 matrix (W4A16, group strategy) as the AWQ
    tensors this path runs, with the same values: ``weight_packed`` int32 [N, K/8] holds
    ``v + 8`` for the signed int4 ``v`` of element (n, k) in nibble ``k % 8`` of word
    ``k / 8``; ``weight_scale`` [N, K/group] (float); ``weight_zero_point`` int32
    [N/8, K/group] holds ``zp + 8`` packed the same way along N, or None (symmetric: zero point
    0).  ``(v - zp) * s`` equals AWQ's ``(q - z) * s`` with ``q = v + 8`` and ``z = zp + 8``, so
    the repack moves nibbles only: ``qweight`` [K, N/8] and ``qzeros`` [K/group, N/8] in AWQ's
    nibble order, ``scales`` fp16 [K/group, N] (``ValueError`` when a scale is not exactly an
    fp16 value, or the sizes do not fit group-128 AWQ)."""
    wp = np.asarray(weight_packed)
    if wp.dtype != np.int32 or wp.ndim != 2:
        raise ValueError("weight_packed must be a 2-D int32 array")
    N, K = (int(v) for v in weight_shape) if weight_shape is not None else (wp.shape[0], wp.shape[1] * 8)
    if group_size != 128 or K % 128 or N % 8 or wp.shape != (N, -(-K // 8)):
        raise ValueError(f"a [{N}, {K}] int4 matrix packed as {wp.shape} does not fit AWQ int4 group 128")
    s = np.asarray(weight_scale, np.float32)
    if s.shape != (N, K // 128):
        raise ValueError(f"weight_scale must be [{N}, {K // 128}], got {s.shape}")
    s16 = s.astype(np.float16)
    if not np.array_equal(s16.astype(np.float32), s):
        raise ValueError("weight_scale holds values that fp16 does not represent exactly")
    q = _nibbles_sequential(wp)[:, :K]  # [N, K] = v + 8
    if weight_zero_point is None:
        z = np.full((K // 128, N), 8, np.uint8)
    else:
        zp = np.asarray(weight_zero_point)
        if zp.dtype != np.int32 or zp.shape != (N // 8, K // 128):
            raise ValueError(f"weight_zero_point must be int32 [{N // 8}, {K // 128}], got {zp.dtype} {zp.shape}")
        z = _nibbles_sequential(np.ascontiguousarray(zp.T))[:, :N]  # [K / 128, N] = zp + 8
    return {"qweight": _awq_words(np.ascontiguousarray(q.T)), "qzeros": _awq_words(z),
            "scales": np.ascontiguousarray(s16.T)}
