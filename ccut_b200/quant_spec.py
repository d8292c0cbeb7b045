"""Declarative quantization keys of the drop-in: the reference's ``QuantKey`` /
``LayerQuantSpec`` interface (``ccut/quant/spec.py:29-193``) with the same field names, key
names and predicates, so that a ``LayerQuantSpec`` built by the reference's config code (or by
this module) selects a method through ``ccut_b200.quant.make_method_for_spec``.

Two keys are new to this path: ``awq_int4_g128`` (unsigned int4 with group-128 fp16 scales
and packed zero points) and ``fp8_block128`` (e4m3 with one fp32 scale per 128 x 128 block).
The reference's keys keep their meaning; the ones whose weights this path runs are
``fp8_static_channel_sym`` / ``fp8_dynamic_token_sym`` / ``fp8_static_tensor_sym``
(``fp8_channel`` weights) and ``int4_w4a16_sym`` (``int4_sym_g128`` weights).
"""

from __future__ import annotations

from dataclasses import dataclass, field

__all__ = ["QuantDType", "ScaleStrategy", "GroupShape", "QuantKey", "ScaleDesc", "LayerQuantSpec",
           "get_quant_key", "registered_keys", "K_AWQ_INT4_G128", "K_FP8_BLOCK128"]


class QuantDType:
    """Stored element types (the reference's string values)."""

    BF16 = "bf16"
    FP16 = "fp16"
    FP32 = "fp32"
    INT8 = "int8"
    FP8_E4M3 = "fp8_e4m3"
    FP8_E5M2 = "fp8_e5m2"
    INT4 = "int4"
    NF4 = "nf4"
    MXFP8 = "mxfp8"
    MXFP4 = "mxfp4"
    NVFP4 = "nvfp4"
    ALL = (BF16, FP16, FP32, INT8, FP8_E4M3, FP8_E5M2, INT4, NF4, MXFP8, MXFP4, NVFP4)


class ScaleStrategy:
    """Scale granularity (compressed-tensors strategy names)."""

    PER_TENSOR = "tensor"
    PER_CHANNEL = "channel"
    PER_TOKEN = "token"
    PER_GROUP = "group"
    NO_SCALE = "none"


@dataclass(frozen=True)
class GroupShape:
    """Group sizes: ``rows`` along the input dimension, ``cols`` along the output one."""

    rows: int | None = None
    cols: int | None = None

    def is_grouped(self) -> bool:
        return self.rows is not None and self.rows > 0

    @property
    def group_size(self) -> int:
        return self.rows if self.rows else 0


@dataclass(frozen=True)
class QuantKey:
    """One layer's weight / activation quantization (``ccut/quant/spec.py:101-137``)."""

    weight_dtype: str = QuantDType.BF16
    weight_scale: str = ScaleStrategy.NO_SCALE
    act_dtype: str = QuantDType.BF16
    act_scale: str = ScaleStrategy.NO_SCALE
    symmetric: bool = True
    group_shape: GroupShape = field(default_factory=GroupShape)
    name: str = ""

    def is_quantized(self) -> bool:
        return self.weight_scale != ScaleStrategy.NO_SCALE

    def is_weight_only(self) -> bool:
        return self.is_quantized() and self.act_scale == ScaleStrategy.NO_SCALE

    def is_w8a8(self) -> bool:
        return self.is_quantized() and self.act_scale != ScaleStrategy.NO_SCALE

    def compute_path(self) -> str:
        """``bf16`` / ``w8a16`` / ``w8a8`` / ``w4a16``, as the reference labels them."""
        if not self.is_quantized():
            return "bf16"
        if self.is_weight_only():
            return "w4a16" if self.weight_dtype in (QuantDType.INT4, QuantDType.NF4) else "w8a16"
        return "w8a8"


@dataclass(frozen=True)
class ScaleDesc:
    """One scale tensor of a layer (checkpoint name, dtype, shape)."""

    name: str
    dtype: str
    shape: tuple = ()
    offset: int = 0
    length: int = 0

    def is_e8m0(self) -> bool:
        return self.dtype.upper() in ("U8", "F8_E8M0")


@dataclass(frozen=True)
class LayerQuantSpec:
    """A layer's quantization (``ccut/quant/spec.py:162-193``)."""

    layer_name: str
    weight_key: QuantKey
    activation_key: QuantKey | None = None
    scales: tuple = ()
    skipped: bool = False
    quant_method: str = ""

    def effective_key(self) -> QuantKey:
        """The weight key with the activation side taken from ``activation_key``."""
        if self.skipped or self.activation_key is None:
            return self.weight_key
        w, a = self.weight_key, self.activation_key
        return QuantKey(weight_dtype=w.weight_dtype, weight_scale=w.weight_scale, act_dtype=a.weight_dtype,
                        act_scale=a.weight_scale, symmetric=w.symmetric, group_shape=w.group_shape, name=w.name)


K_FP8_DYNAMIC_TOKEN_SYM = "fp8_dynamic_token_sym"
K_FP8_STATIC_CHANNEL_SYM = "fp8_static_channel_sym"
K_FP8_STATIC_TENSOR_SYM = "fp8_static_tensor_sym"
K_INT8_STATIC_CHANNEL_SYM = "int8_static_channel_sym"
K_INT8_DYNAMIC_TOKEN_SYM = "int8_dynamic_token_sym"
K_INT8_W4A16_SYM = "int4_w4a16_sym"
K_NF4_W4A16 = "nf4_w4a16"
K_MXFP8_DYNAMIC = "mxfp8_dynamic"
K_MXFP4_DYNAMIC = "mxfp4_dynamic"
K_NVFP4_DYNAMIC = "nvfp4_dynamic"
K_BF16 = "bf16"
K_AWQ_INT4_G128 = "awq_int4_g128"
K_FP8_BLOCK128 = "fp8_block128"

_D, _S = QuantDType, ScaleStrategy
_KEYS: dict[str, QuantKey] = {
    K_BF16: QuantKey(_D.BF16, _S.NO_SCALE, _D.BF16, _S.NO_SCALE, True),
    K_FP8_DYNAMIC_TOKEN_SYM: QuantKey(_D.FP8_E4M3, _S.PER_CHANNEL, _D.FP32, _S.PER_TOKEN, True),
    K_FP8_STATIC_CHANNEL_SYM: QuantKey(_D.FP8_E4M3, _S.PER_CHANNEL, _D.FP32, _S.PER_TOKEN, True),
    K_FP8_STATIC_TENSOR_SYM: QuantKey(_D.FP8_E4M3, _S.PER_TENSOR, _D.FP32, _S.PER_TOKEN, True),
    K_INT8_STATIC_CHANNEL_SYM: QuantKey(_D.INT8, _S.PER_CHANNEL, _D.FP32, _S.PER_TOKEN, True),
    K_INT8_DYNAMIC_TOKEN_SYM: QuantKey(_D.INT8, _S.PER_CHANNEL, _D.FP32, _S.PER_TOKEN, True),
    K_INT8_W4A16_SYM: QuantKey(_D.INT4, _S.PER_CHANNEL, _D.FP32, _S.NO_SCALE, True),
    K_NF4_W4A16: QuantKey(_D.NF4, _S.PER_CHANNEL, _D.FP16, _S.NO_SCALE, True),
    K_MXFP8_DYNAMIC: QuantKey(_D.MXFP8, _S.PER_GROUP, _D.BF16, _S.PER_TOKEN, False, GroupShape(rows=32)),
    K_MXFP4_DYNAMIC: QuantKey(_D.MXFP4, _S.PER_GROUP, _D.BF16, _S.PER_TOKEN, False, GroupShape(rows=32)),
    K_NVFP4_DYNAMIC: QuantKey(_D.NVFP4, _S.PER_GROUP, _D.BF16, _S.PER_TOKEN, False, GroupShape(rows=16)),
    # new to this path
    K_AWQ_INT4_G128: QuantKey(_D.INT4, _S.PER_GROUP, _D.BF16, _S.NO_SCALE, False, GroupShape(rows=128),
                              K_AWQ_INT4_G128),
    K_FP8_BLOCK128: QuantKey(_D.FP8_E4M3, _S.PER_GROUP, _D.BF16, _S.NO_SCALE, True, GroupShape(rows=128, cols=128),
                             K_FP8_BLOCK128),
}


def get_quant_key(name: str) -> QuantKey:
    """A registered key by name (case-insensitive); ``KeyError`` for unknown names."""
    key = _KEYS.get(name.casefold())
    if key is None:
        raise KeyError(f"unknown QuantKey {name!r}, registered: {sorted(_KEYS)}")
    return key


def registered_keys() -> tuple:
    return tuple(sorted(_KEYS))
