"""Dense quantized SwiGLU FFN on every token: ``down(silu(x Wg) * (x Wu))``.

The reference runs this as three quant-linear projections and ``silu_mul_fused`` (the
shared-expert block of ``ccut/models/generic.py:380-385``; a dense layer's ``ffn`` at
``:446``, e.g. layer 0 of DeepSeek-V2-Lite with intermediate 10944).  Here it is the
grouped expert GEMMs with one expert that every token is routed to once, with weight 1:
the same dequant-fused kernels (mma.sync below 64 tokens, tcgen05 above), the SiLU fused
into the gate/up epilogue, and the bf16 (or fp32) output written by the combine kernel.

An intermediate size that is not a multiple of 128 (10944) is padded with zero channels
on the host before packing: the padded gate/up channels have zero weights (FP8 code 0,
AWQ scale 0, signed int4 value 0), so ``silu(0) * 0 = 0`` and the padded down-projection inputs contribute
nothing.  AWQ group-128 matrices need their input size to be a multiple of 128, so an AWQ
down projection must come with ``in_features`` already a multiple of 128.
"""

from __future__ import annotations

import numpy as np
import torch

from ccut_b200 import formats
from ccut_b200.layer import MoeLayer, Permutation, _get, _ptr, _stream

__all__ = ["DenseFfn"]


def _pad_to(a: np.ndarray, axis: int, size: int, value=0) -> np.ndarray:
    a = a.detach().cpu().numpy() if isinstance(a, torch.Tensor) else np.asarray(a)
    if a.shape[axis] == size:
        return a
    if a.shape[axis] > size:
        raise ValueError(f"cannot pad axis {axis} of {a.shape} down to {size}")
    pad = [(0, 0)] * a.ndim
    pad[axis] = (0, size - a.shape[axis])
    return np.pad(a, pad, constant_values=value)


_V0 = np.int32(-0x77777778)  # 0x88888888: eight nibbles v + 8 = 8, i.e. signed int4 zeros


class DenseFfn:
    """``fmt``: ``"awq_int4_g128"`` (matrices ``qweight``/``qzeros``/``scales``, ``[in, out]``),
    ``"fp8_b128"`` (``weight`` ``[out, in]`` + ``weight_scale_inv``/``scale``), or the
    ``"fp8_channel"`` / ``"int4_sym_g128"`` forms of ``ccut_b200.formats``.
    ``inter`` is the model's intermediate size; it is padded to a multiple of 128."""

    def __init__(self, fmt: str, hidden: int, inter: int, gate, up, down, kernel: str = "auto", device="cuda",
                 workspaces: dict | None = None):
        if hidden % 128:
            raise ValueError("hidden must be a multiple of 128")
        self.hidden, self.inter = int(hidden), int(inter)
        ip = (self.inter + 127) // 128 * 128
        self.inter_padded = ip
        if fmt == "awq_int4_g128":
            mats = {}
            for role, m in (("gate", gate), ("up", up)):  # [H, I]: pad the output channels
                q, z, s = _get(m, "qweight"), _get(m, "qzeros"), _get(m, "scales")
                if q.shape[1] * 8 != self.inter and q.shape[1] * 8 != ip:
                    raise ValueError(f"{role}: qweight {q.shape} does not hold {self.inter} channels")
                mats[role] = {"qweight": _pad_to(q, 1, ip // 8), "qzeros": _pad_to(z, 1, ip // 8),
                              "scales": _pad_to(s, 1, ip)}
            q, z, s = _get(down, "qweight"), _get(down, "qzeros"), _get(down, "scales")
            if q.shape[0] % 128:
                raise ValueError(f"down: AWQ group-128 input size {q.shape[0]} is not a multiple of 128")
            mats["down"] = {"qweight": _pad_to(q, 0, ip), "qzeros": _pad_to(z, 0, ip // 128),
                            "scales": _pad_to(s, 0, ip // 128)}
        elif fmt == "fp8_b128":
            mats = {}
            for role, m in (("gate", gate), ("up", up)):  # [I, H]: pad rows
                w, s = _get(m, "weight"), _get(m, "weight_scale_inv", "scale")
                mats[role] = {"weight": _pad_to(w, 0, ip), "scale": _pad_to(s, 0, ip // 128)}
            w, s = _get(down, "weight"), _get(down, "weight_scale_inv", "scale")  # [H, I]: pad columns
            mats["down"] = {"weight": _pad_to(w, 1, ip), "scale": _pad_to(s, 1, ip // 128)}
        elif fmt == "fp8_channel":
            mats = {}
            for role, m in (("gate", gate), ("up", up)):  # [I, H]: pad rows (zero codes)
                t = formats.canonical(fmt, m)
                mats[role] = {"weight": _pad_to(t["weight"], 0, ip), "scales": _pad_to(t["scales"], 1, ip)}
            t = formats.canonical(fmt, down)  # [H, I]: pad columns
            if t["weight"].shape[1] % 128:
                raise ValueError("down: per-channel FP8 input size must be a multiple of 128")
            mats["down"] = {"weight": _pad_to(t["weight"], 1, ip), "scales": _pad_to(t["scales"], 0, ip // 128)}
        elif fmt == "int4_sym_g128":
            mats = {}
            for role, m in (("gate", gate), ("up", up)):  # [H, I]: pad the output channels with v = 0
                t = formats.canonical(fmt, m)
                mats[role] = {"qweight": _pad_to(t["qweight"], 1, ip // 8, _V0), "scales": _pad_to(t["scales"], 1, ip)}
            t = formats.canonical(fmt, down)
            mats["down"] = {"qweight": _pad_to(t["qweight"], 0, ip, _V0), "scales": _pad_to(t["scales"], 0, ip // 128)}
        else:
            raise NotImplementedError(f"weight format {fmt!r} is not supported")
        self.layer = MoeLayer(fmt, self.hidden, ip, 1, 1, "softmax_topk", np.zeros((1, self.hidden), np.float32),
                              [mats], kernel=kernel, device=device, workspaces=workspaces)
        self.device = self.layer.device
        self._perm: dict[int, Permutation] = {}

    def _identity(self, T: int) -> Permutation:
        """Identity permutation of T tokens (cached for the last few batch sizes)."""
        p = self._perm.get(T)
        if p is None:
            if len(self._perm) >= 8:
                self._perm.pop(next(iter(self._perm)))
            dev = self.device
            ar = torch.arange(max(T, 1), dtype=torch.int32, device=dev)
            p = Permutation(torch.tensor([0, T], dtype=torch.int32, device=dev), ar,
                            torch.ones(max(T, 1), dtype=torch.float32, device=dev), ar)
            self._perm[T] = p
        return p

    def forward(self, x: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        """bf16 ``x [T, H]`` -> ``[T, H]`` (bf16 or fp32)."""
        x = self.layer._check_x(x)
        T = x.shape[0]
        if T == 0:
            return torch.empty((0, self.hidden), dtype=out_dtype, device=self.device)
        p = self._identity(T)
        y = self.layer.expert_ffn(x, p, k=1)
        return self.layer.combine(y, p, T, k=1, out_dtype=out_dtype)

    __call__ = forward

    def workspace_status(self) -> int:
        """Device status word of the FFN workspace (0 = ok); clears it."""
        ws = self.layer._ws.get("ffn")
        if ws is None:
            return 0
        return self.layer.lib.ccut_workspace_status(_ptr(ws), _stream())
