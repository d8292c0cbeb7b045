"""``QuantizeMethodBase``-compatible linear methods for the path's weight formats.

Mirrors the reference's method interface (``ccut/quant/method.py:27-62``):
``create_weights(spec)`` checks the scale tensors once, ``apply(weight_bytes, scales, x)``
returns ``y = x @ dequant(W)^T`` as fp32 ``[batch, out]``, and
``process_weights_after_loading()`` is a hook.  ``apply`` packs the weight into the kernel
tile layout on its first call (cached per weight buffer) and then runs
``ccut_quant_linear`` on the GPU.  numpy in gives numpy out; torch in gives torch out.
``make_method_for_spec`` is the reference's ``make_method_for_spec``
(``ccut/quant/method.py:157-183``): a ``LayerQuantSpec`` (``ccut_b200.quant_spec``, or the
reference's own, read by field names) selects the method by its ``QuantKey``.

Formats and the tensors ``apply`` takes (``weight_bytes`` + the ``scales`` dict):
  AWQ int4 g128       qweight int32 [in, out/8]; {"scales": fp16 [in/128, out], "qzeros": int32
                      [in/128, out/8]}                               (key ``awq_int4_g128``)
  FP8 e4m3 b128       e4m3 bytes [out, in]; {"weight_scale_inv" (or "scale"): fp32
                      [out/128, in/128]}                              (key ``fp8_block128``)
  FP8 e4m3 channel    e4m3 bytes [out, in]; {spec scale name, "weight_scale" or "scale": fp32
                      [out] or one value} -- the reference's FP8 (``ccut/quant/method.py:
                      100-127``; keys ``fp8_static_channel_sym``, ``fp8_dynamic_token_sym``,
                      ``fp8_static_tensor_sym``)
  signed int4         uint8 [out, in/2], low nibble first; {spec scale name, "weight_scale" or
                      "scale": fp32 [in]} -- the reference's W4A16 (``ccut/quant/weight_only.py:
                      37-54``; key ``int4_w4a16_sym``)
The reference computes its w8a8 path as the w8a16 one (``ccut/quant/method.py:131-139``:
dequantize, then ``x @ w.T``), so the FP8 methods run both labels the same way.  Missing
scales raise ``ValueError`` and unknown formats ``NotImplementedError``, as in the reference.
"""

from __future__ import annotations

import numpy as np
import torch

from ccut_b200 import _lib, formats
from ccut_b200.formats import awq_columns as _awq_columns, awq_words as _awq_words
from ccut_b200.layer import _dev, _ptr, _stream
from ccut_b200.quant_spec import QuantDType

__all__ = ["QuantizeMethodBase", "UnquantizedMethod", "AwqInt4G128Method", "Fp8Block128Method", "Fp8ChannelMethod",
           "Int4SymMethod", "make_method", "make_method_for_spec", "dequantize", "QuantLinear",
           "cat_checkpoint_tensors", "permute_out_channels", "pad_out_channels", "ct_int4_to_awq", "ct_int4_to_sym"]


class QuantizeMethodBase:
    """Interface of the reference's quantize methods."""

    compute_path = "bf16"

    def create_weights(self, spec=None) -> None:
        return None

    def apply(self, weight_bytes, scales: dict, x):
        raise NotImplementedError

    def process_weights_after_loading(self) -> None:
        return None


def _x_tensor(x, K):
    was_np = not isinstance(x, torch.Tensor)
    xt = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)) if was_np else x
    if xt.dim() != 2 or (K is not None and xt.shape[1] != K):
        raise ValueError(f"x must be [batch, {K}], got {tuple(xt.shape)}")
    return xt, was_np


def _nbytes(b) -> int:
    if isinstance(b, torch.Tensor):
        return b.numel() * b.element_size()
    if isinstance(b, (bytes, bytearray, memoryview)):
        return len(b)
    return np.asarray(b).nbytes


class _PackedLinear(QuantizeMethodBase):
    fmt = ""
    scale_names: tuple[tuple[str, ...], ...] = ()
    bits = 8  # weight bits per element (infers the output size from the weight bytes)

    def __init__(self, in_features: int | None = None, out_features: int | None = None, layout: str = "frags",
                 device="cuda", spec=None):
        if layout not in _lib.LAYOUTS:
            raise NotImplementedError(f"layout {layout!r} is not supported (have {sorted(_lib.LAYOUTS)})")
        self.K = int(in_features) if in_features is not None else None
        self.N = int(out_features) if out_features is not None else None
        self._check_sizes()
        self.layout = layout
        self.device = torch.device(device)
        self.lib = _lib.load()
        self.code = _lib.FORMATS[self.fmt]
        self.spec = spec
        self.scale_name = spec.scales[0].name if spec is not None and getattr(spec, "scales", None) else None
        self._packed: dict = {}
        self._ws: torch.Tensor | None = None

    def _check_sizes(self):
        for v in (self.K, self.N):
            if v is not None and v % 128:
                raise ValueError("in_features and out_features must be multiples of 128")

    def create_weights(self, spec=None) -> None:
        names = getattr(spec, "scales", None)
        if spec is not None and not getattr(spec, "skipped", False) and not names:
            raise ValueError(f"{getattr(spec, 'layer_name', 'layer')}: quantized layer has no scale tensors")
        if spec is not None and names:
            self.spec = spec
            self.scale_name = names[0].name

    def _scale(self, scales: dict, names: tuple[str, ...]):
        for n in ((self.scale_name,) if self.scale_name else ()) + tuple(names):
            if n in scales:
                return scales[n]
        raise ValueError(f"missing scale tensor (one of {names})")

    def _pack(self, weight_bytes, scales: dict) -> torch.Tensor:
        if self.N is None:  # the output size follows from the weight bytes
            self.N = _nbytes(weight_bytes) * 8 // (self.bits * self.K)
            self._check_sizes()
        key = (id(weight_bytes), tuple(id(v) for v in scales.values()))
        hit = self._packed.get(key)
        if hit is not None:
            return hit[0]
        t = formats.canonical(self.fmt, self._matrix(weight_bytes, scales))
        q, z, s = formats.pack_args(self.fmt, t, self.K, self.N, self.device)
        packed = torch.empty(self.lib.ccut_packed_matrix_bytes(self.code, self.K, self.N), dtype=torch.uint8,
                             device=self.device)
        with torch.cuda.device(self.device):
            _lib.call("ccut_pack_matrix", self.code, _lib.LAYOUTS[self.layout], _ptr(q), _ptr(z), _ptr(s), self.K,
                      self.N, _lib.NIBBLES_AWQ, _ptr(packed), 1, 0, _stream())
        self._packed[key] = (packed, weight_bytes, scales)  # keep the sources alive: their ids are the key
        return packed

    def apply(self, weight_bytes, scales: dict, x):
        xt, was_np = _x_tensor(x, self.K)
        if self.K is None:
            self.K = int(xt.shape[1])
            self._check_sizes()
        packed = self._pack(weight_bytes, scales)
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
    bits = 4

    def _matrix(self, weight_bytes, scales):
        return {"qweight": _as_array(weight_bytes, np.int32).reshape(self.K, self.N // 8),
                "scales": np.asarray(self._scale(scales, ("scales",)), dtype=np.float16).reshape(self.K // 128, self.N),
                "qzeros": np.asarray(self._scale(scales, ("qzeros", "zeros")), dtype=np.int32).reshape(
                    self.K // 128, self.N // 8)}


class Fp8Block128Method(_PackedLinear):
    """W8A16: e4m3 weights with one fp32 scale per 128 x 128 block."""

    compute_path = "w8a16"
    fmt = "fp8_b128"
    scale_names = (("weight_scale_inv", "scale"),)

    def _matrix(self, weight_bytes, scales):
        return {"weight": _as_array(weight_bytes, np.uint8).reshape(self.N, self.K),
                "scale": np.asarray(self._scale(scales, ("weight_scale_inv", "scale")), dtype=np.float32).reshape(
                    self.N // 128, self.K // 128)}


class Fp8ChannelMethod(_PackedLinear):
    """W8A16: e4m3 weights with one fp32 scale per output channel (or one for the tensor) --
    the reference's FP8 linear (``ccut/quant/method.py:100-127``, ``ccut/quant/fp8.py:19-35``)."""

    compute_path = "w8a16"
    fmt = "fp8_channel"
    scale_names = (("weight_scale", "scale"),)

    def _matrix(self, weight_bytes, scales):
        w = _as_array(weight_bytes, np.uint8).reshape(self.N, self.K)
        if "scales" in scales and self.scale_name not in scales:  # one scale per channel per 128-k group
            return {"weight": w, "scales": np.asarray(scales["scales"], np.float32).reshape(self.K // 128, self.N)}
        return {"weight": w,
                "scale": np.asarray(self._scale(scales, ("weight_scale", "scale")), dtype=np.float32).reshape(-1)}


class Int4SymMethod(_PackedLinear):
    """W4A16: signed int4 weights with one fp32 scale per input column, constant within each
    128-column group -- the reference's weight-only int4 (``ccut/quant/weight_only.py:37-54``)."""

    compute_path = "w4a16"
    fmt = "int4_sym_g128"
    scale_names = (("weight_scale", "scale"),)
    bits = 4

    def _matrix(self, weight_bytes, scales):
        if "scales" in scales and self.scale_name not in scales:  # qweight int32 [K, N/8] of v + 8
            return {"qweight": _as_array(weight_bytes, np.int32).reshape(self.K, self.N // 8),
                    "scales": np.asarray(scales["scales"], np.float32).reshape(self.K // 128, self.N)}
        return {"weight": _as_array(weight_bytes, np.uint8).reshape(self.N, self.K // 2),
                "scale": np.asarray(self._scale(scales, ("weight_scale", "scale")), dtype=np.float32).reshape(-1)}


class UnquantizedMethod(QuantizeMethodBase):
    """bf16 / fp16 / fp32 weights ``[out, in]`` (layers a checkpoint leaves unquantized,
    ``ccut/quant/method.py:65-76``): ``x @ w.T`` in fp32 on the GPU (cuBLAS), with the
    weight uploaded once per buffer."""

    compute_path = "bf16"
    _DT = {QuantDType.BF16: torch.bfloat16, QuantDType.FP16: torch.float16, QuantDType.FP32: torch.float32}

    def __init__(self, weight_dtype: str = QuantDType.BF16, device="cuda"):
        if weight_dtype not in self._DT:
            raise NotImplementedError(f"unquantized weight dtype {weight_dtype!r} is not supported")
        self.weight_dtype = weight_dtype
        self.device = torch.device(device)
        self._w: dict = {}

    def apply(self, weight_bytes, scales, x):
        xt, was_np = _x_tensor(x, None)
        K = int(xt.shape[1])
        hit = self._w.get(id(weight_bytes))
        if hit is None:
            dt = self._DT[self.weight_dtype]
            raw = weight_bytes if isinstance(weight_bytes, torch.Tensor) else torch.from_numpy(
                np.frombuffer(weight_bytes, np.uint8).copy() if isinstance(weight_bytes, (bytes, bytearray, memoryview))
                else np.ascontiguousarray(weight_bytes).view(np.uint8))
            w = raw.reshape(-1).view(torch.uint8).view(dt).reshape(-1, K).to(self.device).float()
            hit = self._w[id(weight_bytes)] = (w, weight_bytes)
        y = xt.to(self.device, torch.float32) @ hit[0].t()
        return y.cpu().numpy() if was_np else y


def _as_array(b, dtype) -> np.ndarray:
    if isinstance(b, torch.Tensor):
        return b.detach().cpu().numpy().view(dtype)
    if isinstance(b, (bytes, bytearray, memoryview)):
        return np.frombuffer(b, dtype=dtype).copy()
    return np.asarray(b).view(dtype)


_METHODS = {"awq_int4_g128": AwqInt4G128Method, "fp8_b128": Fp8Block128Method, "fp8_channel": Fp8ChannelMethod,
            "int4_sym_g128": Int4SymMethod}


def make_method(fmt: str, in_features: int | None = None, out_features: int | None = None, **kw) -> QuantizeMethodBase:
    """Format name -> method (``"awq_int4_g128"`` | ``"fp8_b128"`` | ``"fp8_channel"`` |
    ``"int4_sym_g128"``)."""
    cls = _METHODS.get(fmt)
    if cls is None:
        raise NotImplementedError(f"weight format {fmt!r} is not supported (have {sorted(_METHODS)})")
    return cls(in_features, out_features, **kw)


def format_for_key(key) -> str:
    """This path's weight format for a ``QuantKey`` (read by field names), as
    ``make_method_for_spec`` picks it; ``NotImplementedError`` for keys whose weights this
    path does not run (int8, nf4, e5m2, the MX formats)."""
    wd = key.weight_dtype
    gs = getattr(key, "group_shape", None)
    rows, cols = (getattr(gs, "rows", None), getattr(gs, "cols", None)) if gs is not None else (None, None)
    if wd == QuantDType.FP8_E4M3:
        if rows == 128 and cols == 128:
            return "fp8_b128"
        if key.weight_scale in ("channel", "tensor", "token"):
            return "fp8_channel"
    elif wd == QuantDType.INT4:
        if not key.symmetric and rows == 128:
            return "awq_int4_g128"
        if key.symmetric and key.weight_scale == "channel":
            return "int4_sym_g128"
    raise NotImplementedError(f"QuantKey {getattr(key, 'name', '') or key!r}: weight dtype {wd!r} with "
                              f"{key.weight_scale!r} scales is not run by this path")


def make_method_for_spec(spec, in_features: int | None = None, out_features: int | None = None,
                         layout: str = "frags", device="cuda") -> QuantizeMethodBase:
    """``LayerQuantSpec`` -> method, as the reference's ``make_method_for_spec``
    (``ccut/quant/method.py:157-183``): skipped layers get ``UnquantizedMethod``; otherwise
    the effective key's weight format selects the method (``format_for_key``).  Sizes are
    taken from the first ``apply`` when not given."""
    key = spec.effective_key()
    if getattr(spec, "skipped", False) or key.weight_scale == "none":
        return UnquantizedMethod(weight_dtype=key.weight_dtype, device=device)
    return make_method(format_for_key(key), in_features, out_features, layout=layout, device=device, spec=spec)


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
# axis along which the output channels run in each (None: shared by all output channels)
_TENSORS = {"awq_int4_g128": (("qweight", 1), ("qzeros", 1), ("scales", 1)),
            "fp8_b128": (("weight", 0), ("weight_scale_inv", 0)),
            "fp8_channel": (("weight", 0), ("weight_scale", 0)),
            "int4_sym_g128": (("weight", 0), ("weight_scale", None))}
_ALIASES = {"fp8_b128": {"scale": "weight_scale_inv"}, "fp8_channel": {"scale": "weight_scale"},
            "int4_sym_g128": {"scale": "weight_scale"}}
# the grouped forms of the per-channel formats (``ccut_b200.formats``): fp32 scales [in/128, out]
_GROUPED = {"fp8_channel": (("weight", 0), ("scales", 1)), "int4_sym_g128": (("qweight", 1), ("scales", 1))}


def _names(fmt: str, t: dict) -> tuple:
    """Tensor names (and output-channel axes) of one matrix's checkpoint tensors ``t``."""
    if fmt in _GROUPED and "scales" in t:
        return _GROUPED[fmt]
    return _TENSORS[fmt]


class QuantLinear:
    """A linear projection ``y = x @ W^T`` kept in its checkpoint format (``W`` [out, in]) and
    run by ``ccut_quant_linear`` (fp32 out) -- a quarter (int4) or half (FP8) of the bytes of
    a bf16 copy.  ``tensors``: the checkpoint tensors of the matrix (AWQ ``qweight`` /
    ``qzeros`` / ``scales``; FP8 ``weight`` / ``weight_scale_inv`` (blocks) or
    ``weight_scale`` (channels), or ``scale`` for either; signed int4 ``weight`` /
    ``weight_scale``).  The weight is packed into the kernel layout once, at construction."""

    def __init__(self, fmt: str, tensors: dict, in_features: int, out_features: int, device="cuda",
                 layout: str = "frags"):
        if fmt not in _TENSORS:
            raise NotImplementedError(f"weight format {fmt!r} is not supported")
        t = dict(tensors)
        for alias, name in _ALIASES.get(fmt, {}).items():
            if name not in t and alias in t:
                t[name] = t.pop(alias)
        names = _names(fmt, t)
        missing = [n for n, _ in names if n not in t]
        if missing:
            raise ValueError(f"missing checkpoint tensors {missing}")
        self.fmt, self.in_features, self.out_features = fmt, int(in_features), int(out_features)
        self.tensors = {n: t[n] for n, _ in names}
        self.method = make_method(fmt, self.in_features, self.out_features, layout=layout, device=device)
        main = names[0][0]
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
    side along their last axis, FP8 ``weight`` / scales stacked along the first, signed int4
    ``weight`` stacked with the one per-input-column scale the parts must share.  For block
    FP8 each part's output channels must be a multiple of 128 (one scale block)."""
    if fmt not in _TENSORS:
        raise NotImplementedError(f"weight format {fmt!r} is not supported")
    out = {}
    for n, ax in _names(fmt, parts[0]):
        arrs = [np.asarray(p[n]) for p in parts]
        if ax is None:
            if any(not np.array_equal(a, arrs[0]) for a in arrs[1:]):
                raise ValueError(f"{fmt}: the parts' {n} tensors differ, so they cannot share one matrix")
            out[n] = arrs[0]
        else:
            out[n] = np.concatenate(arrs, axis=ax)
    return out


def permute_out_channels(fmt: str, tensors: dict, perm) -> dict:
    """The checkpoint tensors of ``W[perm]`` (output channel ``j`` of the result is channel
    ``perm[j]`` of ``W``), in the same format: AWQ nibbles and scales moved along the output
    axis; FP8 weight rows (and per-channel scales) moved -- block FP8 needs every row to stay
    in its 128-row scale block (``ValueError`` otherwise); signed int4 weight rows moved.  Byte
    moves only: the values dequantize to the permuted rows exactly."""
    perm = np.asarray(perm, np.int64)
    if fmt == "awq_int4_g128" or (fmt == "int4_sym_g128" and "qweight" in tensors):
        n = tensors["scales"].shape[1]
        if perm.shape != (n,):
            raise ValueError(f"perm must have {n} entries")
        out = {"qweight": _awq_words(_awq_columns(tensors["qweight"])[:, perm]),
               "scales": np.ascontiguousarray(np.asarray(tensors["scales"])[:, perm])}
        if "qzeros" in tensors:
            out["qzeros"] = _awq_words(_awq_columns(tensors["qzeros"])[:, perm])
        return out
    if fmt == "fp8_channel" and "scales" in tensors:
        w = np.asarray(tensors["weight"])
        if perm.shape != (w.shape[0],):
            raise ValueError(f"perm must have {w.shape[0]} entries")
        return {"weight": np.ascontiguousarray(w[perm]),
                "scales": np.ascontiguousarray(np.asarray(tensors["scales"])[:, perm])}
    if fmt in ("fp8_b128", "fp8_channel", "int4_sym_g128"):
        w = np.asarray(tensors["weight"])
        if perm.shape != (w.shape[0],):
            raise ValueError(f"perm must have {w.shape[0]} entries")
        out = dict(tensors)
        out["weight"] = np.ascontiguousarray(w[perm])
        if fmt == "fp8_b128" and np.any(perm // 128 != np.arange(perm.size) // 128):
            raise ValueError("an FP8 row permutation must keep every row in its 128-row scale block")
        if fmt == "fp8_channel":
            key = "weight_scale" if "weight_scale" in tensors else "scale"
            sc = np.asarray(tensors[key], np.float32).reshape(-1)
            out[key] = sc if sc.size == 1 else np.ascontiguousarray(sc[perm])
        return out
    raise NotImplementedError(f"weight format {fmt!r} is not supported")


def pad_out_channels(fmt: str, tensors: dict, out_features: int) -> dict:
    """The checkpoint tensors with zero output channels appended up to ``out_features`` (so
    that a matrix whose output size is not a multiple of 128 can be packed and dequantized;
    the padded channels dequantize to 0)."""
    if fmt in ("int4_sym_g128", "fp8_channel") and "scales" in tensors:  # grouped forms: zero scales
        s = np.asarray(tensors["scales"])
        extra = out_features - s.shape[1]
        if extra < 0 or (fmt == "int4_sym_g128" and (extra % 8 or s.shape[1] % 8)):
            raise ValueError(f"cannot pad {s.shape[1]} output channels to {out_features}")
        out = {"scales": np.concatenate([s, np.zeros((s.shape[0], extra), s.dtype)], axis=1)}
        if fmt == "int4_sym_g128":
            q = np.asarray(tensors["qweight"])
            out["qweight"] = np.concatenate([q, np.full((q.shape[0], extra // 8), -0x77777778, np.int32)], axis=1)
        else:
            w = np.asarray(tensors["weight"])
            out["weight"] = np.concatenate([w, np.zeros((extra, w.shape[1]), w.dtype)])
        return out
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
    if fmt in ("fp8_b128", "fp8_channel", "int4_sym_g128"):
        w = np.asarray(tensors["weight"])
        extra = out_features - w.shape[0]
        if extra < 0:
            raise ValueError(f"cannot pad {w.shape[0]} output channels to {out_features}")
        out = {k: v for k, v in tensors.items() if k != "weight"}
        out["weight"] = np.concatenate([w, np.zeros((extra, w.shape[1]), w.dtype)])
        if fmt == "fp8_b128":
            sc = np.asarray(tensors.get("weight_scale_inv", tensors.get("scale")))
            blocks = -(-out_features // 128)
            if blocks > sc.shape[0]:
                sc = np.concatenate([sc, np.ones((blocks - sc.shape[0], sc.shape[1]), sc.dtype)])
            out.pop("scale", None)
            out["weight_scale_inv"] = sc
        elif fmt == "fp8_channel":
            key = "weight_scale" if "weight_scale" in tensors else "scale"
            sc = np.asarray(tensors[key], np.float32).reshape(-1)
            if sc.size > 1:
                out[key] = np.concatenate([sc, np.ones(out_features - sc.size, np.float32)])
        return out
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


def ct_int4_to_sym(weight_packed, weight_scale, weight_shape=None, group_size: int = 128) -> dict:
    """A symmetric compressed-tensors ``pack-quantized`` int4 matrix (group strategy, no zero
    point) as ``int4_sym_g128`` tensors with the same values and any fp32 scale:
    ``weight_packed`` int32 [N, K/8] holds ``v + 8`` in nibble ``k % 8`` of word ``k / 8``,
    ``weight_scale`` [N, K/group]; the result is ``qweight`` int32 [K, N/8] (``v + 8`` in AWQ's
    nibble order) and ``scales`` fp32 [K/group, N] (``ValueError`` when the sizes do not fit
    group 128)."""
    wp = np.asarray(weight_packed)
    if wp.dtype != np.int32 or wp.ndim != 2:
        raise ValueError("weight_packed must be a 2-D int32 array")
    N, K = (int(v) for v in weight_shape) if weight_shape is not None else (wp.shape[0], wp.shape[1] * 8)
    if group_size != 128 or K % 128 or N % 8 or wp.shape != (N, -(-K // 8)):
        raise ValueError(f"a [{N}, {K}] int4 matrix packed as {wp.shape} does not fit int4 group 128")
    s = np.asarray(weight_scale, np.float32)
    if s.shape != (N, K // 128):
        raise ValueError(f"weight_scale must be [{N}, {K // 128}], got {s.shape}")
    q = _nibbles_sequential(wp)[:, :K]  # [N, K] = v + 8
    return {"qweight": _awq_words(np.ascontiguousarray(q.T)), "scales": np.ascontiguousarray(s.T)}
