"""HBM-resident quantized MoE layer driving the sm_100a kernels through the C ABI.

Replaces the reference's streamed expert tier (``ccut/experts/reader.py:86-334`` ring
buffer + ``ccut/models/generic.py:389-400`` per-call segment dequant): every expert's
checkpoint tensors are uploaded once, packed on the device into the kernel tile layout
and stay resident.  ``forward`` is the whole MoE layer of ``ccut/models/generic.py:348-386``.

Checkpoint tensors are accepted per matrix as a mapping (or object with attributes), in
the forms ``ccut_b200.formats`` lists: AWQ ``{"qweight": int32 [K, N/8], "qzeros": int32
[K/128, N/8], "scales": fp16 [K/128, N]}`` (``[in, out]``); block FP8 ``{"weight": e4m3/uint8
[N, K], "scale": fp32 [N/128, K/128]}`` (``[out, in]``, the ``weight_scale_inv`` tensor of
DeepSeek checkpoints); per-channel FP8 ``{"weight": [N, K], "scale": fp32 [N]}``; signed int4
``{"weight": uint8 [N, K/2], "scale": fp32 [K]}``.
"""

from __future__ import annotations

import ctypes as C
import warnings
from dataclasses import dataclass

import numpy as np
import torch

from ccut_b200 import _lib, formats

__all__ = ["MoeLayer", "Routing", "Permutation"]


def _get(m, *names):
    for n in names:
        if isinstance(m, dict) and n in m:
            return m[n]
        if hasattr(m, n):
            return getattr(m, n)
    raise KeyError(f"checkpoint matrix lacks any of {names}")


def _dev(a, device, dtype=None) -> torch.Tensor:
    if isinstance(a, torch.Tensor):
        t = a
    else:
        a = np.ascontiguousarray(a)
        with warnings.catch_warnings():  # read-only views (mmap'd checkpoints) are only read
            warnings.simplefilter("ignore", UserWarning)
            t = torch.from_numpy(a)
    if dtype is not None and t.dtype != dtype:
        t = t.view(dtype) if t.element_size() == torch.empty((), dtype=dtype).element_size() else t.to(dtype)
    return t.to(device, non_blocking=False).contiguous()


def _stream() -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t: torch.Tensor | None) -> C.c_void_p:
    return C.c_void_p(t.data_ptr() if t is not None else 0)


@dataclass
class Routing:
    ids: torch.Tensor  # int32 [T, k]
    weights: torch.Tensor  # fp32 [T, k]
    logits: torch.Tensor | None = None  # fp32 [T, E]


@dataclass
class Permutation:
    offsets: torch.Tensor  # int32 [E + slices + 1]
    row_token: torch.Tensor  # int32 [R]
    row_weight: torch.Tensor  # fp32 [R]
    pair_row: torch.Tensor  # int32 [T * k]


class MoeLayer:
    """One MoE layer with experts resident in HBM.

    ``fmt``: ``"awq_int4_g128"``, ``"fp8_b128"``, ``"fp8_channel"`` or ``"int4_sym_g128"``;
    ``routing``: ``"softmax_topk"``
    (``norm_topk_prob=False``), ``"topk_softmax"`` (``norm_topk_prob=True``) or
    ``"sigmoid_group"``.  ``kernel``: ``"auto"`` keeps both packed layouts resident and runs
    the mma.sync kernel for decode-sized batches and the tcgen05 kernel otherwise; ``"tc"``
    keeps only the tcgen05 layout; ``"mma"`` forces the mma.sync kernel.  ``workspaces``: a
    dict shared by layers that never run concurrently (the layers of one decoder), so that
    they reuse one set of device workspaces instead of one set each."""

    def __init__(
        self,
        fmt: str,
        hidden: int,
        inter: int,
        num_experts: int,
        top_k: int,
        routing: str,
        router: np.ndarray | torch.Tensor,
        experts: list,
        shared: list | None = None,
        shared_inter: int | None = None,
        shared_gate: float = 1.0,
        n_group: int = 1,
        topk_group: int = 1,
        routed_scaling: float = 1.0,
        bias: np.ndarray | torch.Tensor | None = None,
        nibble_order: str = "awq",
        kernel: str = "auto",
        device: str | torch.device = "cuda",
        workspaces: dict | None = None,
    ):
        if fmt not in _lib.FORMATS:
            raise NotImplementedError(f"weight format {fmt!r} is not supported (have {sorted(_lib.FORMATS)})")
        if routing not in _lib.ROUTING:
            raise NotImplementedError(f"routing mode {routing!r} is not supported")
        if hidden % 128 or inter % 128:
            raise ValueError("hidden and inter must be multiples of 128")
        if len(experts) != num_experts:
            raise ValueError(f"expected {num_experts} experts, got {len(experts)}")
        if kernel not in _lib.KERNELS:
            raise NotImplementedError(f"kernel policy {kernel!r} is not supported (have {sorted(_lib.KERNELS)})")
        self.lib = _lib.load()
        self.fmt, self.fmt_code = fmt, _lib.FORMATS[fmt]
        self.kernel = kernel
        self.hidden, self.inter, self.num_experts, self.top_k = hidden, inter, num_experts, top_k
        self.routing = routing
        self.device = torch.device(device)
        shared = list(shared or [])
        s_inter = shared_inter if shared_inter is not None else inter
        if shared and s_inter % inter:
            raise NotImplementedError("shared-expert intermediate must be a multiple of the routed one")
        self.slices_per_shared = s_inter // inter if shared else 0
        self.num_slices = len(shared) * self.slices_per_shared
        self.shared_gate = float(shared_gate)
        self.router = _dev(router, self.device, torch.float32)
        if tuple(self.router.shape) != (num_experts, hidden):
            raise ValueError(f"router must be [E, H] = {(num_experts, hidden)}, got {tuple(self.router.shape)}")
        self.bias = _dev(bias, self.device, torch.float32) if bias is not None else None
        self.route_params = _lib.RouteParams(
            _lib.ROUTING[routing], top_k, n_group, topk_group, float(routed_scaling), _ptr(self.bias).value or None
        )
        self.nibbles = _lib.NIBBLES_AWQ if nibble_order == "awq" else _lib.NIBBLES_SEQUENTIAL
        L = self.lib
        self.w13_bytes = L.ccut_w13_bytes(self.fmt_code, hidden, inter)
        self.w2_bytes = L.ccut_w2_bytes(self.fmt_code, hidden, inter)
        ne = num_experts + self.num_slices
        self.packed = {}  # layout name -> (w13, w2)
        layouts = ["rows"] + ([] if kernel == "tc" else ["frags"])
        with torch.cuda.device(self.device):
            for lay in layouts:
                w13 = torch.empty(ne * self.w13_bytes, dtype=torch.uint8, device=self.device)
                w2 = torch.empty(ne * self.w2_bytes, dtype=torch.uint8, device=self.device)
                code = _lib.LAYOUTS[lay]
                for e, ew in enumerate(experts):
                    self._pack_expert(code, w13, w2, e, ew, 0, inter)
                for j, sw in enumerate(shared):
                    for s in range(self.slices_per_shared):
                        self._pack_expert(code, w13, w2, num_experts + j * self.slices_per_shared + s, sw,
                                          s * inter, inter)
                self.packed[lay] = (w13, w2)
            torch.cuda.current_stream().synchronize()
        self.w13, self.w2 = self.packed["rows"]
        w13f, w2f = self.packed.get("frags", (None, None))
        self.desc = _lib.MoeLayerDesc(
            self.fmt_code, _lib.KERNELS[kernel], hidden, inter, num_experts, self.num_slices, self.shared_gate,
            _ptr(self.w13), _ptr(self.w2), _ptr(w13f), _ptr(w2f), _ptr(self.router),
        )
        # workspaces by entry point; layers that run one after another on one stream (the
        # layers of a decoder) may share one dict, so that a long prefill sizes one set
        self._ws: dict[str, torch.Tensor] = workspaces if workspaces is not None else {}

    # ---- packing ------------------------------------------------------------------
    def _slice(self, mat, role: str, lo: int, width: int):
        """Canonical checkpoint tensors of intermediate channels [lo, lo+width) of one matrix:
        the output channels of gate / up, the input channels of down."""
        t = formats.canonical(self.fmt, mat)
        return formats.slice_out(self.fmt, t, lo, width) if role in ("gate", "up") else formats.slice_in(
            self.fmt, t, lo, width)

    def _pack_one(self, layout_code, mat, role, lo, width, K, N, dst: torch.Tensor, nmat: int, slot: int):
        qd, zd, sd = formats.pack_args(self.fmt, self._slice(mat, role, lo, width), K, N, self.device, role)
        nibbles = _lib.NIBBLES_AWQ if formats.repacked(self.fmt, mat) else self.nibbles
        _lib.call("ccut_pack_matrix", self.fmt_code, layout_code, _ptr(qd), _ptr(zd), _ptr(sd), K, N, nibbles,
                  _ptr(dst), nmat, slot, _stream())

    def _pack_expert(self, code, w13_all, w2_all, e: int, ew, lo: int, width: int):
        H, I = self.hidden, self.inter
        w13 = w13_all[e * self.w13_bytes:(e + 1) * self.w13_bytes]
        w2 = w2_all[e * self.w2_bytes:(e + 1) * self.w2_bytes]
        self._pack_one(code, _get(ew, "gate"), "gate", lo, width, H, I, w13, 2, 0)
        self._pack_one(code, _get(ew, "up"), "up", lo, width, H, I, w13, 2, 1)
        self._pack_one(code, _get(ew, "down"), "down", lo, width, I, H, w2, 1, 0)

    # ---- workspace ------------------------------------------------------------------
    def _workspace(self, key: str, nbytes: int) -> torch.Tensor:
        ws = self._ws.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=self.device)
            self._ws[key] = ws
        return ws

    def _check_x(self, x: torch.Tensor) -> torch.Tensor:
        if x.device != self.device and not (x.is_cuda and self.device.type == "cuda" and self.device.index is None):
            raise ValueError("activations must be on the layer's device")
        if x.dtype != torch.bfloat16:
            raise ValueError("activations must be bf16")
        if x.dim() != 2 or x.shape[1] != self.hidden:
            raise ValueError(f"activations must be [T, {self.hidden}]")
        return x.contiguous()

    # ---- whole layer ----------------------------------------------------------------
    def forward(self, x: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16,
                return_routing: bool = False):
        x = self._check_x(x)
        T = x.shape[0]
        out = torch.empty((T, self.hidden), dtype=out_dtype, device=self.device)
        ids = torch.empty((T, self.top_k), dtype=torch.int32, device=self.device) if return_routing else None
        wts = torch.empty((T, self.top_k), dtype=torch.float32, device=self.device) if return_routing else None
        nbytes = self.lib.ccut_moe_forward_workspace_bytes(C.byref(self.desc), T, self.top_k)
        ws = self._workspace("fwd", nbytes)
        od = _lib.OUT_BF16 if out_dtype == torch.bfloat16 else _lib.OUT_F32
        if out_dtype not in (torch.bfloat16, torch.float32):
            raise ValueError("out_dtype must be bf16 or fp32")
        _lib.call("ccut_moe_forward", C.byref(self.desc), C.byref(self.route_params), _ptr(x), T, _ptr(out), od,
                  _ptr(ids), _ptr(wts), _ptr(ws), ws.numel(), _stream())
        if return_routing:
            return out, Routing(ids, wts)
        return out

    __call__ = forward

    def workspace_status(self) -> int:
        """Device status word of the forward workspace (0 = ok); clears it."""
        ws = self._ws.get("fwd")
        if ws is None:
            return 0
        return self.lib.ccut_workspace_status(_ptr(ws), _stream())

    # ---- stages ---------------------------------------------------------------------
    def route(self, x: torch.Tensor, want_logits: bool = False) -> Routing:
        x = self._check_x(x)
        T, E, k = x.shape[0], self.num_experts, self.top_k
        ids = torch.empty((T, k), dtype=torch.int32, device=self.device)
        wts = torch.empty((T, k), dtype=torch.float32, device=self.device)
        lg = torch.empty((T, E), dtype=torch.float32, device=self.device) if want_logits else None
        ws = self._workspace("route", self.lib.ccut_route_workspace_bytes(T, E, self.hidden))
        _lib.call("ccut_moe_route", _ptr(x), _ptr(self.router), T, self.hidden, E, C.byref(self.route_params),
                  _ptr(ids), _ptr(wts), _ptr(lg), _ptr(ws), ws.numel(), _stream())
        return Routing(ids, wts, lg)

    def topk(self, logits: torch.Tensor) -> Routing:
        logits = logits.to(self.device, torch.float32).contiguous()
        T, E = logits.shape
        ids = torch.empty((T, self.top_k), dtype=torch.int32, device=self.device)
        wts = torch.empty((T, self.top_k), dtype=torch.float32, device=self.device)
        _lib.call("ccut_moe_topk", _ptr(logits), T, E, C.byref(self.route_params), _ptr(ids), _ptr(wts), _stream())
        return Routing(ids, wts, logits)

    def permute(self, routing: Routing) -> Permutation:
        ids = routing.ids.to(self.device, torch.int32).contiguous()
        wts = routing.weights.to(self.device, torch.float32).contiguous()
        T, k = ids.shape
        R = T * k + self.num_slices * T
        ne = self.num_experts + self.num_slices
        perm = Permutation(
            torch.empty(ne + 1, dtype=torch.int32, device=self.device),
            torch.empty(max(R, 1), dtype=torch.int32, device=self.device),
            torch.empty(max(R, 1), dtype=torch.float32, device=self.device),
            torch.empty(max(T * k, 1), dtype=torch.int32, device=self.device),
        )
        ws = self._workspace("perm", self.lib.ccut_permute_workspace_bytes(self.num_experts))
        _lib.call("ccut_moe_permute", _ptr(ids), _ptr(wts), T, k, self.num_experts, self.num_slices,
                  C.c_float(self.shared_gate), _ptr(perm.offsets), _ptr(perm.row_token), _ptr(perm.row_weight),
                  _ptr(perm.pair_row), _ptr(ws), ws.numel(), _stream())
        return perm

    def expert_ffn(self, x: torch.Tensor, perm: Permutation, k: int | None = None) -> torch.Tensor:
        x = self._check_x(x)
        T = x.shape[0]
        k = k or self.top_k
        R = T * k + self.num_slices * T
        y = torch.empty((max(R, 1), self.hidden), dtype=torch.float32, device=self.device)
        ws = self._workspace("ffn", self.lib.ccut_expert_ffn_workspace_bytes(C.byref(self.desc), T, k))
        _lib.call("ccut_moe_expert_ffn", C.byref(self.desc), _ptr(x), T, k, _ptr(perm.offsets), _ptr(perm.row_token),
                  _ptr(perm.row_weight), _ptr(y), _ptr(ws), ws.numel(), _stream())
        return y[:R]

    def gate_up(self, x: torch.Tensor, perm: Permutation, k: int | None = None) -> torch.Tensor:
        """Intermediate rows h [R, I] as 16-bit bit patterns: bf16 when the call runs the tcgen05
        kernel, f16 when it runs the mma.sync kernel; ``down`` reads them back with the same kernel."""
        x = self._check_x(x)
        T = x.shape[0]
        k = k or self.top_k
        R = T * k + self.num_slices * T
        h = torch.empty((max(R, 1), self.inter), dtype=torch.int16, device=self.device)
        ws = self._workspace("gate_up", self.lib.ccut_gate_up_workspace_bytes(C.byref(self.desc), T))
        _lib.call("ccut_moe_gate_up", C.byref(self.desc), _ptr(x), T, k, _ptr(perm.offsets), _ptr(perm.row_token),
                  _ptr(h), _ptr(ws), ws.numel(), _stream())
        return h[:R]

    def down(self, h: torch.Tensor, perm: Permutation, T: int, k: int | None = None) -> torch.Tensor:
        k = k or self.top_k
        R = T * k + self.num_slices * T
        y = torch.empty((max(R, 1), self.hidden), dtype=torch.float32, device=self.device)
        ws = self._workspace("down", self.lib.ccut_down_workspace_bytes(C.byref(self.desc)))
        _lib.call("ccut_moe_down", C.byref(self.desc), _ptr(h), T, k, _ptr(perm.offsets), _ptr(perm.row_weight),
                  _ptr(y), _ptr(ws), ws.numel(), _stream())
        return y[:R]

    def combine(self, y_rows: torch.Tensor, perm: Permutation, T: int, k: int | None = None,
                out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        k = k or self.top_k
        out = torch.empty((T, self.hidden), dtype=out_dtype, device=self.device)
        od = _lib.OUT_BF16 if out_dtype == torch.bfloat16 else _lib.OUT_F32
        _lib.call("ccut_moe_combine", _ptr(y_rows), _ptr(perm.pair_row), T, k, self.hidden, self.num_slices,
                  _ptr(out), od, _stream())
        return out

    def dequant(self, expert: int, which: str, layout: str = "rows") -> torch.Tensor:
        """fp32 [K, N] ([in, out]) export of one packed matrix ("gate" | "up" | "down")."""
        H, I = self.hidden, self.inter
        w13_all, w2_all = self.packed[layout]
        if which in ("gate", "up"):
            src = w13_all[expert * self.w13_bytes:(expert + 1) * self.w13_bytes]
            K, N, nmat, slot = H, I, 2, 0 if which == "gate" else 1
        else:
            src = w2_all[expert * self.w2_bytes:(expert + 1) * self.w2_bytes]
            K, N, nmat, slot = I, H, 1, 0
        out = torch.empty((K, N), dtype=torch.float32, device=self.device)
        _lib.call("ccut_dequant_matrix", self.fmt_code, _lib.LAYOUTS[layout], _ptr(src), K, N, nmat, slot,
                  _ptr(out), _stream())
        return out
