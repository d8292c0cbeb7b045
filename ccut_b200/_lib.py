"""ctypes binding of ``libccut_moe.so`` (the C ABI in ``include/ccut_moe.h``).

There is no fallback: if the library is missing or cannot be loaded, importing a compute
entry point raises.  Status codes are mapped onto the exception classes the reference
raises for the same conditions (``ValueError`` for bad shapes / missing scales,
``NotImplementedError`` for unsupported formats, ``TimeoutError`` for an expired bounded
wait, ``RuntimeError`` for CUDA failures).
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("CCUT_B200_LIB", _PKG / "_build" / "libccut_moe.so"))

OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_WORKSPACE, ERR_TIMEOUT, ERR_NCCL = range(7)
FMT_AWQ_INT4_G128, FMT_FP8_E4M3_B128, FMT_FP8_E4M3_CH, FMT_INT4_SYM_G128 = 1, 2, 3, 4
NIBBLES_AWQ, NIBBLES_SEQUENTIAL = 0, 1
LAYOUT_ROWS, LAYOUT_FRAGS = 0, 1
ROUTE_SOFTMAX_TOPK, ROUTE_TOPK_SOFTMAX, ROUTE_SIGMOID_GROUP = 0, 1, 2
OUT_BF16, OUT_F32 = 0, 1

FORMATS = {"awq_int4_g128": FMT_AWQ_INT4_G128, "fp8_b128": FMT_FP8_E4M3_B128, "fp8_channel": FMT_FP8_E4M3_CH,
           "int4_sym_g128": FMT_INT4_SYM_G128}
LAYOUTS = {"rows": LAYOUT_ROWS, "frags": LAYOUT_FRAGS}
KERNEL_AUTO, KERNEL_TC, KERNEL_MMA = 0, 1, 2
KERNELS = {"auto": KERNEL_AUTO, "tc": KERNEL_TC, "mma": KERNEL_MMA}
ROUTING = {"softmax_topk": ROUTE_SOFTMAX_TOPK, "topk_softmax": ROUTE_TOPK_SOFTMAX, "sigmoid_group": ROUTE_SIGMOID_GROUP}

_vp, _sz, _i, _f = C.c_void_p, C.c_size_t, C.c_int, C.c_float


class RouteParams(C.Structure):
    _fields_ = [
        ("mode", _i), ("top_k", _i), ("n_group", _i), ("topk_group", _i),
        ("routed_scaling", _f), ("bias", _vp),
    ]


class MoeLayerDesc(C.Structure):
    _fields_ = [
        ("format", _i), ("kernel", _i), ("hidden", _i), ("inter", _i), ("num_experts", _i),
        ("num_shared_slices", _i), ("shared_gate", _f),
        ("w13", _vp), ("w2", _vp), ("w13_frags", _vp), ("w2_frags", _vp), ("router", _vp),
    ]


# name -> (restype, argtypes); mirrors include/ccut_moe.h
SIGNATURES: dict[str, tuple] = {
    "ccut_strerror": (C.c_char_p, [_i]),
    "ccut_abi_version": (_i, []),
    "ccut_packed_matrix_bytes": (_sz, [_i, _i, _i]),
    "ccut_w13_bytes": (_sz, [_i, _i, _i]),
    "ccut_w2_bytes": (_sz, [_i, _i, _i]),
    "ccut_pack_matrix": (_i, [_i, _i, _vp, _vp, _vp, _i, _i, _i, _vp, _i, _i, _vp]),
    "ccut_dequant_matrix": (_i, [_i, _i, _vp, _i, _i, _i, _i, _vp, _vp]),
    "ccut_route_workspace_bytes": (_sz, [_i, _i, _i]),
    "ccut_moe_route": (_i, [_vp, _vp, _i, _i, _i, C.POINTER(RouteParams), _vp, _vp, _vp, _vp, _sz, _vp]),
    "ccut_moe_topk": (_i, [_vp, _i, _i, C.POINTER(RouteParams), _vp, _vp, _vp]),
    "ccut_permute_workspace_bytes": (_sz, [_i]),
    "ccut_moe_permute": (_i, [_vp, _vp, _i, _i, _i, _i, _f, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "ccut_moe_permute_static": (_i, [_vp, _vp, _i, _i, _i, _i, _f, _vp, _vp, _vp, _vp, _vp]),
    "ccut_expert_ffn_workspace_bytes": (_sz, [C.POINTER(MoeLayerDesc), _i, _i]),
    "ccut_moe_expert_ffn": (_i, [C.POINTER(MoeLayerDesc), _vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "ccut_moe_expert_ffn_w4a16": (_i, [C.POINTER(MoeLayerDesc), _vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "ccut_moe_expert_ffn_fp8b128": (_i, [C.POINTER(MoeLayerDesc), _vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "ccut_moe_expert_ffn_w8a16": (_i, [C.POINTER(MoeLayerDesc), _vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "ccut_gate_up_workspace_bytes": (_sz, [C.POINTER(MoeLayerDesc), _i]),
    "ccut_down_workspace_bytes": (_sz, [C.POINTER(MoeLayerDesc)]),
    "ccut_moe_gate_up": (_i, [C.POINTER(MoeLayerDesc), _vp, _i, _i, _vp, _vp, _vp, _vp, _sz, _vp]),
    "ccut_moe_down": (_i, [C.POINTER(MoeLayerDesc), _vp, _i, _i, _vp, _vp, _vp, _vp, _sz, _vp]),
    "ccut_moe_combine": (_i, [_vp, _vp, _i, _i, _i, _i, _vp, _i, _vp]),
    "ccut_moe_forward_workspace_bytes": (_sz, [C.POINTER(MoeLayerDesc), _i, _i]),
    "ccut_moe_forward": (_i, [C.POINTER(MoeLayerDesc), C.POINTER(RouteParams), _vp, _i, _vp, _i, _vp, _vp, _vp, _sz,
                              _vp]),
    "ccut_quant_linear_workspace_bytes": (_sz, [_i, _i, _i]),
    "ccut_quant_linear": (_i, [_i, _i, _vp, _i, _i, _vp, _i, _vp, _vp, _sz, _vp]),
    "ccut_ep_unique_id_bytes": (_sz, []),
    "ccut_ep_unique_id": (_i, [_vp]),
    "ccut_ep_init": (_i, [_vp, _i, _i, C.c_double, C.POINTER(_vp)]),
    "ccut_ep_destroy": (_i, [_vp]),
    "ccut_moe_ep_exchange_workspace_bytes": (_sz, [_i, _i, _i, _i]),
    "ccut_moe_ep_dispatch": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp, _vp, _i, C.POINTER(_i), _vp, _sz,
                                  _vp]),
    "ccut_moe_ep_combine": (_i, [_vp, _vp, _i, _i, _i, _i, _vp, _vp, _sz, _vp]),
    "ccut_moe_ep_forward_workspace_bytes": (_sz, [C.POINTER(MoeLayerDesc), _i, _i, _i, _i]),
    "ccut_gqa_attention_workspace_bytes": (_sz, [_i, _i, _i, _i, _i, _i]),
    "ccut_gqa_attention": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _f, _f, _vp, _i, _vp, _sz, _vp]),
    "ccut_rms_norm": (_i, [_vp, _i, _vp, _i, _i, _f, _vp, _i, _vp]),
    "ccut_apply_rope": (_i, [_vp, _i, _i, _i, _i, _i, _vp, _vp, _f, _vp, _i, _vp]),
    "ccut_gqa_attention_pool": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, C.c_longlong, _i, _f, _f, _vp,
                                     _i, _vp, _sz, _vp]),
    "ccut_mla_attention_workspace_bytes": (_sz, [_i, _i, _i, _i]),
    "ccut_mla_attention": (_i, [_vp, _vp, _i, _i, _i, _i, _i, _i, _i, _f, _vp, _i, _vp, _sz, _vp]),
    "ccut_mla_attention_pool": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, C.c_longlong, _i, _f, _vp, _i, _vp,
                                     _sz, _vp]),
    "ccut_moe_ep_forward": (_i, [_vp, C.POINTER(MoeLayerDesc), _i, _i, C.POINTER(RouteParams), _vp, _i, _i, _vp,
                                 _i, _vp, _sz, _vp]),
    "ccut_workspace_status": (_i, [_vp, _vp]),
    "ccut_debug_wait_expiry": (_i, [_vp, C.c_longlong, _vp]),
}

_lib = None


def load(path: str | os.PathLike | None = None):
    """Load (once) and return the bound library.  Raises if it is absent."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(
            f"{p} is missing: build it with `python -m ccut_b200.build` (the CUDA path has no CPU fallback)"
        )
    lib = C.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


class CcutError(RuntimeError):
    pass


def check(code: int, what: str = "") -> None:
    """Raise the exception class the reference uses for this condition."""
    if code == OK:
        return
    msg = load().ccut_strerror(code).decode()
    msg = f"{what}: {msg}" if what else msg
    if code in (ERR_INVALID, ERR_WORKSPACE):
        raise ValueError(msg)
    if code == ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    if code == ERR_TIMEOUT:
        raise TimeoutError(msg)
    raise CcutError(msg)


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)
