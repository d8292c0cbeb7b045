"""Expert-parallel MoE layer: one process per GPU, routed experts sharded over the ranks.

Rank ``r`` of ``world`` keeps routed experts ``expert_range(E, world, r)`` and every shared
expert resident in its HBM.  ``forward`` takes this rank's tokens and runs
``ccut_moe_ep_forward``: route locally, exchange per-destination row counts, send each token
row once to every rank that owns one of its experts (NCCL send / receive of the routed rows
only), run the received rows through the local grouped FFN, send one partial row per
(token, rank) back to the token's owner, which sums them in rank order and adds the shared
experts (data-parallel on the local tokens).  The NCCL communicator belongs to the C library;
``torch.distributed`` (any backend) only carries its unique id from rank 0 to the others.

The reference has no expert parallelism (one process runs a layer's experts,
``ccut/models/generic.py:364-385``); the partitioning follows the layout of its experts
(index ``e`` of the layer's expert list).
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from ccut_b200 import _lib
from ccut_b200.layer import MoeLayer, _dev, _ptr, _stream

__all__ = ["ExpertParallelMoeLayer", "expert_range", "localize_ids"]


def expert_range(num_experts: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous block [lo, hi) of routed experts owned by ``rank`` (sizes differ by at most one)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if num_experts < world:
        raise ValueError(f"{num_experts} experts cannot be split over {world} ranks")
    base, extra = divmod(num_experts, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def localize_ids(ids, lo: int, hi: int):
    """Local expert index of each routed pair (``id - lo`` inside [lo, hi), else -1), the
    mapping the device applies before the local permutation."""
    if isinstance(ids, torch.Tensor):
        inside = (ids >= lo) & (ids < hi)
        return torch.where(inside, ids - lo, torch.full_like(ids, -1))
    ids = np.asarray(ids)
    return np.where((ids >= lo) & (ids < hi), ids - lo, -1).astype(ids.dtype)


def _broadcast_unique_id(lib, rank: int, world: int, group) -> bytes:
    n = lib.ccut_ep_unique_id_bytes()
    buf = (C.c_char * n)()
    if rank == 0:
        _lib.check(lib.ccut_ep_unique_id(C.cast(buf, C.c_void_p)), "ccut_ep_unique_id")
    if world == 1:
        return bytes(buf)
    import torch.distributed as dist

    obj = [bytes(buf) if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    return obj[0]


class ExpertParallelMoeLayer:
    """MoE layer whose routed experts are split over ``world`` GPUs (one process each).

    Arguments are those of ``MoeLayer`` for the whole layer (all ``num_experts`` routed
    experts); only this rank's block of experts is packed and kept.  ``rank`` / ``world``
    default to ``torch.distributed``'s.  Every rank calls ``forward`` (collective) with its own
    tokens; the counts may differ between ranks up to ``max_tokens``, which every rank must
    pass alike (default: each call's own count, for ranks that always carry equal batches)."""

    def __init__(self, fmt, hidden, inter, num_experts, top_k, routing, router, experts, shared=None,
                 shared_inter=None, shared_gate=1.0, n_group=1, topk_group=1, routed_scaling=1.0, bias=None,
                 nibble_order="awq", kernel="auto", device="cuda", rank=None, world=None, group=None,
                 timeout_s: float = 60.0, max_tokens: int | None = None):
        self.max_tokens = int(max_tokens) if max_tokens is not None else None
        if rank is None or world is None:
            import torch.distributed as dist

            rank = dist.get_rank(group) if rank is None else rank
            world = dist.get_world_size(group) if world is None else world
        self.rank, self.world = int(rank), int(world)
        self.num_experts = int(num_experts)
        self.lo, self.hi = expert_range(self.num_experts, self.world, self.rank)
        if len(experts) != num_experts:
            raise ValueError(f"expected {num_experts} experts, got {len(experts)}")
        router_all = router if isinstance(router, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(router))
        self.local = MoeLayer(fmt, hidden, inter, self.hi - self.lo, top_k, routing, router_all[self.lo:self.hi],
                              list(experts[self.lo:self.hi]), shared=shared, shared_inter=shared_inter,
                              shared_gate=shared_gate, n_group=n_group, topk_group=topk_group,
                              routed_scaling=routed_scaling, nibble_order=nibble_order, kernel=kernel, device=device)
        self.device = self.local.device
        self.hidden, self.top_k = hidden, top_k
        # routing runs against the global router / selection bias
        self.router = _dev(router_all, self.device, torch.float32)
        if tuple(self.router.shape) != (num_experts, hidden):
            raise ValueError(f"router must be [E, H] = {(num_experts, hidden)}, got {tuple(self.router.shape)}")
        self.bias = _dev(bias, self.device, torch.float32) if bias is not None else None
        self.route_params = _lib.RouteParams(_lib.ROUTING[routing], top_k, n_group, topk_group, float(routed_scaling),
                                             _ptr(self.bias).value or None)
        self.desc = _lib.MoeLayerDesc.from_buffer_copy(self.local.desc)
        self.desc.router = _ptr(self.router).value
        self.lib = self.local.lib
        uid = _broadcast_unique_id(self.lib, self.rank, self.world, group)
        self._uid = (C.c_char * len(uid)).from_buffer_copy(uid)
        handle = C.c_void_p()
        with torch.cuda.device(self.device):
            _lib.call("ccut_ep_init", C.cast(self._uid, C.c_void_p), self.rank, self.world, C.c_double(timeout_s),
                      C.byref(handle))
        self._ep = handle
        self._ws: torch.Tensor | None = None

    def forward(self, x: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        """This rank's tokens x bf16 [T_local, H] -> out [T_local, H] (bf16 or fp32)."""
        if self._ep is None or not self._ep.value:
            raise RuntimeError("expert-parallel layer is closed")
        x = self.local._check_x(x)
        T = x.shape[0]
        if out_dtype not in (torch.bfloat16, torch.float32):
            raise ValueError("out_dtype must be bf16 or fp32")
        out = torch.empty((T, self.hidden), dtype=out_dtype, device=self.device)
        T_cap = T if self.max_tokens is None else self.max_tokens
        if T > T_cap:
            raise ValueError(f"{T} tokens exceed max_tokens = {T_cap}")
        nbytes = self.lib.ccut_moe_ep_forward_workspace_bytes(C.byref(self.desc), self.num_experts, self.world,
                                                              T_cap, self.top_k)
        if nbytes == 0:
            raise ValueError("invalid expert-parallel layer or shape")
        if self._ws is None or self._ws.numel() < nbytes:
            self._ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        od = _lib.OUT_BF16 if out_dtype == torch.bfloat16 else _lib.OUT_F32
        _lib.call("ccut_moe_ep_forward", self._ep, C.byref(self.desc), self.lo, self.num_experts,
                  C.byref(self.route_params), _ptr(x), T, T_cap, _ptr(out), od, _ptr(self._ws), self._ws.numel(),
                  _stream())
        return out

    __call__ = forward

    def workspace_status(self) -> int:
        """Device status word of the forward workspace (0 = ok); clears it."""
        if self._ws is None:
            return 0
        return self.lib.ccut_workspace_status(_ptr(self._ws), _stream())

    def close(self) -> None:
        """Destroy the NCCL communicator (collective: every rank calls it)."""
        if self._ep is not None and self._ep.value:
            torch.cuda.current_stream().synchronize()
            rc = self.lib.ccut_ep_destroy(self._ep)
            self._ep = None
            _lib.check(rc, "ccut_ep_destroy")

    def __del__(self):
        try:
            if self._ep is not None and self._ep.value:
                self.lib.ccut_ep_destroy(self._ep)
                self._ep = None
        except Exception:
            pass
