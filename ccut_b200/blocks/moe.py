"""Drop-ins for ``ccut.blocks.moe`` and ``ccut.models.generic.moe_forward`` on the GPU.

Same names, argument order and meaning as the reference; numpy arrays in give numpy arrays
out, torch tensors in give torch tensors out.  The differences are:

- experts are not fetched per call through a ``WeightReader``.  ``moe_forward``'s
  ``reader`` and ``moe_combine``'s ``w_lookup`` name the HBM-resident layer instead: a
  ``MoeLayer``, a mapping ``layer -> MoeLayer``, or an object with ``moe_layer(layer)``;
- activations enter the kernels as bf16 (the reference computes on fp32 activations);
- errors are the reference's exception classes: ``ValueError`` for shapes and
  inconsistent specs, ``NotImplementedError`` for unsupported modes or sizes.

Reference: ``ccut/blocks/moe.py:46-89`` (topk, topk_softmax), ``:144-174`` (moe_combine),
``:177-179`` (shared_expert_add), ``ccut/models/generic.py:348-386`` (moe_forward).
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from ccut_b200 import _lib
from ccut_b200.layer import MoeLayer, Routing, _ptr, _stream

__all__ = ["topk", "topk_softmax", "moe_combine", "moe_forward", "shared_expert_add"]

_MAX_COLS = 256  # routed experts the device top-k handles


def _to_device(a, dtype: torch.dtype, device="cuda") -> tuple[torch.Tensor, bool]:
    """(tensor on the GPU, whether the caller passed numpy)."""
    if isinstance(a, torch.Tensor):
        return a.to(device=device if not a.is_cuda else a.device, dtype=dtype).contiguous(), False
    return torch.from_numpy(np.ascontiguousarray(a)).to(device=device, dtype=dtype), True


def _device_topk(logits: torch.Tensor, k: int, mode: int) -> tuple[torch.Tensor, torch.Tensor]:
    if logits.dim() != 2:
        raise ValueError("logits must be [rows, cols]")
    T, E = logits.shape
    if not 1 <= k <= min(E, 16):
        raise ValueError(f"k = {k} outside [1, min(cols, 16)]")
    if E > _MAX_COLS:
        raise NotImplementedError(f"top-k over {E} > {_MAX_COLS} columns")
    ids = torch.empty((T, k), dtype=torch.int32, device=logits.device)
    w = torch.empty((T, k), dtype=torch.float32, device=logits.device)
    rp = _lib.RouteParams(mode, k, 1, 1, 1.0, None)
    if T:
        with torch.cuda.device(logits.device):
            _lib.call("ccut_moe_topk", _ptr(logits), T, E, C.byref(rp), _ptr(ids), _ptr(w), _stream())
    return ids, w


def topk(x, k: int):
    """Per-row top-k: (values [rows, k] in x's dtype, descending; indices int64 [rows, k]).
    Ties go to the lowest index (the reference's strict ``>`` scan)."""
    xt, was_np = _to_device(x, torch.float32)
    ids, _ = _device_topk(xt, k, _lib.ROUTE_TOPK_SOFTMAX)
    idx = ids.long()
    vals = torch.gather(xt, 1, idx)
    if was_np:
        return vals.cpu().numpy().astype(np.asarray(x).dtype), idx.cpu().numpy()
    return vals.to(x.dtype), idx


def topk_softmax(logits, k: int, norm_topk_prob: bool = True):
    """Routing weights: ``norm_topk_prob=True`` softmax over the top-k logits, ``False``
    top-k of the softmax over all columns.  Returns (weights fp32 [rows, k], ids int64)."""
    lt, was_np = _to_device(logits, torch.float32)
    mode = _lib.ROUTE_TOPK_SOFTMAX if norm_topk_prob else _lib.ROUTE_SOFTMAX_TOPK
    ids, w = _device_topk(lt, k, mode)
    if was_np:
        return w.cpu().numpy(), ids.long().cpu().numpy()
    return w, ids.long()


def _resolve_layer(src, layer=None) -> MoeLayer:
    if isinstance(src, MoeLayer):
        return src
    if isinstance(src, dict):
        if layer not in src:
            raise KeyError(f"no resident MoE layer {layer}")
        return src[layer]
    if hasattr(src, "moe_layer"):
        return src.moe_layer(layer)
    raise ValueError("expected a MoeLayer, a {layer: MoeLayer} mapping or an object with moe_layer(layer)")


def _x_bf16(x, hidden: int, device) -> tuple[torch.Tensor, bool]:
    xt, was_np = _to_device(x, torch.bfloat16, device)
    if xt.dim() != 2 or xt.shape[1] != hidden:
        raise ValueError(f"activations must be [seq, {hidden}], got {tuple(xt.shape)}")
    return xt, was_np


def moe_combine(x, expert_ids, weights, expert_outputs=None, expert_fn=None, w_lookup=None):
    """``y[t] = sum_j weights[t, j] * expert_{ids[t, j]}(x[t])`` in fp32 with the given
    routing; ``w_lookup`` is the resident layer.  Shared experts are not added (the
    reference adds them outside ``moe_combine``).

    ``expert_fn=None`` runs the layer's fused expert kernels.  A caller's ``expert_fn`` is
    called as in the reference, ``expert_fn(x_rows, w_gate, w_up, w_down)`` per expert on
    host arrays (fp32, ``[in, out]``), with the weights the layer's packed tiles export
    (bit-identical to the checkpoint dequant); its rows are weighted and summed per token by
    the combine kernel in slot order.  ``expert_outputs`` is accepted and not read: the
    reference's ``moe_combine`` does not read it either (``ccut/blocks/moe.py:144-174``)."""
    del expert_outputs
    L = _resolve_layer(w_lookup)
    if expert_fn is not None:
        return _combine_with_fn(L, x, expert_ids, weights, expert_fn)
    xt, was_np = _x_bf16(x, L.hidden, L.device)
    ids = expert_ids if isinstance(expert_ids, torch.Tensor) else torch.from_numpy(np.asarray(expert_ids))
    wts = weights if isinstance(weights, torch.Tensor) else torch.from_numpy(np.asarray(weights, dtype=np.float32))
    if ids.shape != wts.shape or ids.dim() != 2 or ids.shape[0] != xt.shape[0]:
        raise ValueError("expert_ids and weights must both be [seq, k] for the seq rows of x")
    ids = ids.to(L.device, torch.int32)
    if ids.numel() and (int(ids.min()) < 0 or int(ids.max()) >= L.num_experts):
        raise ValueError(f"expert ids must lie in [0, {L.num_experts})")
    T, k = ids.shape
    r = Routing(ids, wts.to(L.device, torch.float32))
    if L.num_slices:  # routed experts only: the shared rows are left out of the sum
        perm = L.permute(r)
        y = L.expert_ffn(xt, perm, k)
        y[T * k:] = 0
        out = L.combine(y, perm, T, k, out_dtype=torch.float32)
    else:
        perm = L.permute(r)
        out = L.combine(L.expert_ffn(xt, perm, k), perm, T, k, out_dtype=torch.float32)
    return out.cpu().numpy() if was_np else out


def _combine_with_fn(L: MoeLayer, x, expert_ids, weights, expert_fn):
    was_np = not isinstance(x, torch.Tensor)
    xf = np.asarray(x, dtype=np.float32) if was_np else x.detach().float().cpu().numpy()
    if xf.ndim != 2 or xf.shape[1] != L.hidden:
        raise ValueError(f"activations must be [seq, {L.hidden}], got {xf.shape}")
    ids = expert_ids if isinstance(expert_ids, torch.Tensor) else torch.from_numpy(np.asarray(expert_ids))
    wts = weights if isinstance(weights, torch.Tensor) else torch.from_numpy(np.asarray(weights, dtype=np.float32))
    if ids.shape != wts.shape or ids.dim() != 2 or ids.shape[0] != xf.shape[0]:
        raise ValueError("expert_ids and weights must both be [seq, k] for the seq rows of x")
    ids = ids.to(L.device, torch.int32)
    if ids.numel() and (int(ids.min()) < 0 or int(ids.max()) >= L.num_experts):
        raise ValueError(f"expert ids must lie in [0, {L.num_experts})")
    T, k = ids.shape
    perm = L.permute(Routing(ids, wts.to(L.device, torch.float32)))
    offs = perm.offsets.cpu().numpy()
    row_token = perm.row_token.cpu().numpy()
    y = torch.zeros((perm.row_token.numel(), L.hidden), dtype=torch.float32, device=L.device)
    for e in range(L.num_experts):
        lo, hi = int(offs[e]), int(offs[e + 1])
        if hi == lo:
            continue
        mats = [L.dequant(e, w).cpu().numpy() for w in ("gate", "up", "down")]
        ye = np.asarray(expert_fn(xf[row_token[lo:hi]], *mats), dtype=np.float32)
        if ye.shape != (hi - lo, L.hidden):
            raise ValueError(f"expert_fn returned {ye.shape} for {hi - lo} rows of expert {e}")
        y[lo:hi] = torch.from_numpy(ye).to(L.device) * perm.row_weight[lo:hi, None]
    out = L.combine(y, perm, T, k, out_dtype=torch.float32)
    return out.cpu().numpy() if was_np else out


def moe_forward(h, gate_w, reader, layer, moe_spec, shared_projs=None):
    """Whole MoE layer: router, top-k, experts, weighted combine, shared experts.

    ``gate_w`` must be the router the resident layer holds; ``moe_spec`` supplies
    ``top_k``, ``norm_topk_prob`` and ``has_shared_expert`` and must agree with the layer.
    Returns fp32 [seq, hidden]."""
    L = _resolve_layer(reader, layer)
    top_k = int(getattr(moe_spec, "top_k"))
    if top_k != L.top_k:
        raise ValueError(f"moe_spec.top_k = {top_k} but the resident layer routes top-{L.top_k}")
    norm = bool(getattr(moe_spec, "norm_topk_prob", True))
    if L.routing in ("softmax_topk", "topk_softmax") and norm != (L.routing == "topk_softmax"):
        raise ValueError(f"moe_spec.norm_topk_prob = {norm} but the resident layer uses {L.routing}")
    has_shared = bool(getattr(moe_spec, "has_shared_expert", False)) and shared_projs is not None
    if has_shared != (L.num_slices > 0):
        raise ValueError("shared-expert presence differs between moe_spec / shared_projs and the resident layer")
    gw = gate_w if isinstance(gate_w, torch.Tensor) else torch.from_numpy(np.asarray(gate_w, dtype=np.float32))
    if tuple(gw.shape) != tuple(L.router.shape):
        raise ValueError(f"gate_w must be {tuple(L.router.shape)}, got {tuple(gw.shape)}")
    xt, was_np = _x_bf16(h, L.hidden, L.device)
    out = L.forward(xt, out_dtype=torch.float32)
    return out.cpu().numpy() if was_np else out


def shared_expert_add(y, shared_out, gate_value: float) -> None:
    """In place: ``y += gate_value * shared_out``."""
    y += gate_value * shared_out
