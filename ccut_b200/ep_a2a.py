"""Expert parallelism with an all-to-all exchange: each token row travels only to the ranks
that own one of its experts, once per rank.

``ExpertParallelMoeLayer`` (``ccut_b200.ep``) all-gathers every rank's tokens and
reduce-scatters dense partial outputs, so each rank moves and combines all T tokens whatever
the routing.  ``AllToAllMoeLayer`` exchanges only what the routing needs:

1. route this rank's tokens against the global router (``ccut_moe_route``);
2. per destination rank, the tokens with at least one expert there, each sent once, with
   its k expert ids made local to that rank (-1 for experts elsewhere) and its k weights;
3. ``all_to_all`` of the row counts, then of the rows, ids and weights;
4. the received rows through the rank's own experts (``permute`` / ``expert_ffn`` /
   ``combine``: a -1 id takes no row), giving one weighted partial output per received row;
5. ``all_to_all`` of the partial outputs back, summed per token by its owner in destination
   order (deterministic), plus the shared experts on the owner's own tokens.

The collectives are ``torch.distributed`` ones (NCCL on GPUs; gloo on CPU for the tests of
the exchange).  Rank ``r`` owns routed experts ``expert_range(E, world, r)`` and every shared
expert.  The reference has no expert parallelism (one process runs a layer's experts,
``ccut/models/generic.py:364-385``).
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import torch
import torch.distributed as dist

from ccut_b200 import _lib
from ccut_b200.ep import expert_range
from ccut_b200.layer import MoeLayer, Routing, _dev, _ptr, _stream

__all__ = ["AllToAllMoeLayer", "exchange_plan", "compact_local_ids"]


def exchange_plan(ids: torch.Tensor, world: int, bounds: list[tuple[int, int]]):
    """For routing ``ids [T, k]`` (global expert ids): the token of every row to send, ordered
    by destination rank (``order``), the rows per destination (``counts``, host ints) and
    each sent row's ids made local to its destination (``local_ids [S, k]``, -1 elsewhere)."""
    T, k = ids.shape
    dev = ids.device
    ids64 = ids.long()
    his = torch.tensor([hi for _, hi in bounds], dtype=torch.int64, device=dev)
    los = torch.tensor([lo for lo, _ in bounds], dtype=torch.int64, device=dev)
    owner = torch.bucketize(ids64, his, right=True)  # rank of each (token, slot)
    owner = torch.where(ids64 < 0, torch.full_like(owner, world), owner)  # a missing expert goes nowhere
    hit = torch.zeros((T, world + 1), dtype=torch.bool, device=dev)
    hit.scatter_(1, owner, True)
    picks = [torch.nonzero(hit[:, d]).flatten() for d in range(world)]
    counts = [int(p.numel()) for p in picks]
    order = torch.cat(picks) if picks else torch.zeros(0, dtype=torch.int64, device=dev)
    dest = torch.repeat_interleave(torch.arange(world, device=dev), torch.tensor(counts, device=dev))
    sid = ids64[order]
    lo_d, hi_d = los[dest][:, None], his[dest][:, None]
    local_ids = torch.where((sid >= lo_d) & (sid < hi_d), sid - lo_d, torch.full_like(sid, -1))
    return order, counts, local_ids.to(torch.int32)


def compact_local_ids(local_ids: torch.Tensor, weights: torch.Tensor, num_local: int):
    """Narrow received rows ``local_ids [R, k]`` / ``weights [R, k]`` to ``min(k, num_local)``
    columns: a row's ids are distinct experts, so at most ``num_local`` of them are this rank's
    (>= 0); those move to the front in their original order (a stable sort), so the combine
    still sums them in slot order.  The expert FFN refuses a width above the rank's expert count
    (``ccut_moe_expert_ffn`` checks ``k <= num_experts``), which a split with fewer local
    experts than ``top_k`` (e.g. 64 experts, top-6, 16 ranks) would otherwise hit."""
    R, k = local_ids.shape
    kk = min(k, int(num_local))
    if kk >= k:
        return local_ids, weights
    foreign = (local_ids < 0).to(torch.int8)
    order = torch.argsort(foreign, dim=1, stable=True)[:, :kk]
    return torch.gather(local_ids, 1, order).contiguous(), torch.gather(weights, 1, order).contiguous()


class _GpuExperts:
    """The GPU side: global routing, the rank's routed experts and the shared experts."""

    def __init__(self, fmt, hidden, inter, num_experts, top_k, routing, router, experts, lo, hi, shared, shared_inter,
                 shared_gate, n_group, topk_group, routed_scaling, bias, kernel, device):
        router_all = router if isinstance(router, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(router))
        self.local = MoeLayer(fmt, hidden, inter, hi - lo, min(top_k, hi - lo), routing, router_all[lo:hi],
                              list(experts[lo:hi]), kernel=kernel, device=device)
        self.device = self.local.device
        self.hidden, self.num_experts, self.top_k = hidden, num_experts, top_k
        self.router = _dev(router_all, self.device, torch.float32)
        self.bias = _dev(bias, self.device, torch.float32) if bias is not None else None
        self.rp = _lib.RouteParams(_lib.ROUTING[routing], top_k, n_group, topk_group, float(routed_scaling),
                                   _ptr(self.bias).value or None)
        self.shared = None
        if shared:
            s_inter = shared_inter if shared_inter is not None else inter
            self.shared = MoeLayer(fmt, hidden, s_inter, len(shared), len(shared), "softmax_topk",
                                   np.zeros((len(shared), hidden), np.float32), list(shared), kernel=kernel,
                                   device=device)
        self.shared_gate = float(shared_gate)
        self._ws = None

    def route(self, x: torch.Tensor):
        T = x.shape[0]
        ids = torch.empty((T, self.top_k), dtype=torch.int32, device=self.device)
        wts = torch.empty((T, self.top_k), dtype=torch.float32, device=self.device)
        lib = self.local.lib
        n = lib.ccut_route_workspace_bytes(T, self.num_experts, self.hidden)
        if self._ws is None or self._ws.numel() < n:
            self._ws = torch.zeros(max(n, 256), dtype=torch.uint8, device=self.device)
        _lib.call("ccut_moe_route", _ptr(x), _ptr(self.router), T, self.hidden, self.num_experts, C.byref(self.rp),
                  _ptr(ids), _ptr(wts), None, _ptr(self._ws), self._ws.numel(), _stream())
        return ids, wts

    def routed(self, rows: torch.Tensor, local_ids: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        R = local_ids.shape[0]
        if R == 0:
            return torch.zeros((0, self.hidden), dtype=torch.float32, device=self.device)
        local_ids, weights = compact_local_ids(local_ids, weights, self.local.num_experts)
        k = local_ids.shape[1]
        perm = self.local.permute(Routing(local_ids, weights))
        y = self.local.expert_ffn(rows, perm, k)
        return self.local.combine(y, perm, R, k, out_dtype=torch.float32)

    def shared_out(self, x: torch.Tensor) -> torch.Tensor | None:
        if self.shared is None:
            return None
        T, n = x.shape[0], self.shared.num_experts
        ids = torch.arange(n, dtype=torch.int32, device=self.device).repeat(T, 1)
        w = torch.full((T, n), self.shared_gate, dtype=torch.float32, device=self.device)
        perm = self.shared.permute(Routing(ids, w))
        y = self.shared.expert_ffn(x, perm, n)
        return self.shared.combine(y, perm, T, n, out_dtype=torch.float32)


class AllToAllMoeLayer:
    """MoE layer with routed experts split over ``world`` ranks and the all-to-all exchange above.

    Arguments are those of ``MoeLayer`` for the whole layer; ``rank`` / ``world`` / ``group``
    default to ``torch.distributed``'s.  Every rank calls ``forward`` (collective) with its own
    tokens; the token counts may differ between ranks.  ``experts_impl`` replaces the GPU side
    (route / routed / shared_out), for tests of the exchange on CPU ranks."""

    def __init__(self, fmt, hidden, inter, num_experts, top_k, routing, router, experts, shared=None,
                 shared_inter=None, shared_gate=1.0, n_group=1, topk_group=1, routed_scaling=1.0, bias=None,
                 kernel="auto", device="cuda", rank=None, world=None, group=None, experts_impl=None):
        self.group = group
        self.rank = dist.get_rank(group) if rank is None else int(rank)
        self.world = dist.get_world_size(group) if world is None else int(world)
        if len(experts) != num_experts:
            raise ValueError(f"expected {num_experts} experts, got {len(experts)}")
        self.bounds = [expert_range(num_experts, self.world, r) for r in range(self.world)]
        self.lo, self.hi = self.bounds[self.rank]
        self.hidden = int(hidden)
        self.impl = experts_impl or _GpuExperts(fmt, hidden, inter, num_experts, top_k, routing, router, experts,
                                                self.lo, self.hi, shared, shared_inter, shared_gate, n_group,
                                                topk_group, routed_scaling, bias, kernel, device)
        self.rows_sent = 0  # token rows this rank sent (all destinations, itself included)

    def _a2a(self, x: torch.Tensor, send: list[int], recv: list[int]) -> torch.Tensor:
        out = torch.empty((sum(recv),) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_to_all_single(out, x.contiguous(), recv, send, group=self.group)
        return out

    def forward(self, x: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        """This rank's tokens x ``[T, H]`` -> ``[T, H]`` (``out_dtype``)."""
        if x.dim() != 2 or x.shape[1] != self.hidden:
            raise ValueError(f"x must be [T, {self.hidden}]")
        T = x.shape[0]
        ids, w = self.impl.route(x)
        order, send, local_ids = exchange_plan(ids, self.world, self.bounds)
        counts = torch.tensor(send, dtype=torch.int64, device=x.device)
        rc = torch.empty_like(counts)
        dist.all_to_all_single(rc, counts, group=self.group)
        recv = [int(c) for c in rc.tolist()]
        self.rows_sent += sum(send)
        rows = self._a2a(x[order], send, recv)
        lids = self._a2a(local_ids, send, recv)
        rw = self._a2a(w[order].float(), send, recv)
        part = self.impl.routed(rows, lids, rw)
        back = self._a2a(part.float(), recv, send)
        out = torch.zeros((T, self.hidden), dtype=torch.float32, device=x.device)
        off = 0
        for n in send:  # one destination at a time: its rows hit distinct tokens, so the sum order is fixed
            if n:
                out.index_add_(0, order[off: off + n], back[off: off + n])
            off += n
        s = self.impl.shared_out(x)
        if s is not None:
            out += s
        return out.to(out_dtype)

    __call__ = forward
