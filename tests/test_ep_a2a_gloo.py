"""The all-to-all expert-parallel exchange (``ccut_b200.ep_a2a``) on CPU ranks (gloo, world
size 2 and 3): the product's exchange code with the oracle standing in for the GPU experts
must give every rank the single-process oracle layer's output for its tokens, with ragged
token counts per rank, and send each token row at most once per destination."""

from __future__ import annotations

import datetime
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ccut_b200.ep import expert_range
from ccut_b200.ep_a2a import exchange_plan


def test_exchange_plan():
    bounds = [expert_range(8, 3, r) for r in range(3)]  # [0, 3), [3, 6), [6, 8)
    ids = torch.tensor([[0, 1], [2, 7], [4, 5], [6, -1]])
    order, counts, lids = exchange_plan(ids, 3, bounds)
    assert counts == [2, 1, 2]  # token 0 once to rank 0 although both its experts live there
    assert order.tolist() == [0, 1, 2, 1, 3]
    assert lids.tolist() == [[0, 1], [2, -1], [1, 2], [-1, 1], [0, -1]]


class _FakeLocal:
    """The rank's MoeLayer on the CPU, with the C ABI's argument rules: the permutation takes ids
    in [-1, E) only, and the expert FFN refuses a width k above the rank's expert count
    (``ccut_moe_expert_ffn`` returns CCUT_ERR_INVALID, raised as ValueError).  Expert e maps a
    row to (e + 1) * row."""

    def __init__(self, num_experts):
        self.num_experts = num_experts

    def permute(self, routing):
        ids = routing.ids
        assert int(ids.min()) >= -1 and int(ids.max()) < self.num_experts
        return routing

    def expert_ffn(self, rows, perm, k):
        if k > self.num_experts:
            raise ValueError("invalid argument or shape")
        ids, w = perm.ids.long(), perm.weights
        f = (ids + 1).clamp(min=0).float()[:, :, None] * rows[:, None, :]
        return torch.where(ids[:, :, None] >= 0, w[:, :, None] * f, torch.zeros_like(f))

    def combine(self, y, perm, R, k, out_dtype=torch.float32):
        out = torch.zeros((R, y.shape[2]), dtype=torch.float32)
        for j in range(k):  # slot order, as combine_kernel sums
            out += y[:, j]
        return out.to(out_dtype)


@pytest.mark.parametrize("num_local,k", [(1, 2), (2, 6), (3, 8), (6, 6)])
def test_routed_rows_narrowed_to_local_experts(num_local, k):
    """A rank that owns fewer experts than top_k (e.g. 64 experts, top-6 over 16 ranks gives 4)
    still runs its received rows: each row's local ids are narrowed to min(k, E_local) columns
    before the permutation, keeping their slot order, and the partial outputs are unchanged."""
    from types import SimpleNamespace

    from ccut_b200.ep_a2a import _GpuExperts, compact_local_ids

    g = torch.Generator().manual_seed(num_local * 31 + k)
    R, H = 9, 5
    lids = torch.full((R, k), -1, dtype=torch.int32)
    for r in range(R):  # distinct local experts at random slots, like a received row
        n = int(torch.randint(0, min(k, num_local) + 1, (1,), generator=g))
        slots = torch.randperm(k, generator=g)[:n]
        lids[r, slots] = torch.randperm(num_local, generator=g)[:n].int()
    w = torch.rand((R, k), generator=g)
    rows = torch.randn((R, H), generator=g)
    expect = torch.zeros((R, H))
    for r in range(R):
        for j in range(k):
            if lids[r, j] >= 0:
                expect[r] += w[r, j] * (int(lids[r, j]) + 1) * rows[r]
    nl, nw = compact_local_ids(lids, w, num_local)
    assert nl.shape == (R, min(k, num_local))
    for r in range(R):  # same valid ids in the same order
        assert [int(v) for v in lids[r] if v >= 0] == [int(v) for v in nl[r] if v >= 0]
    impl = SimpleNamespace(local=_FakeLocal(num_local), hidden=H, device="cpu")
    got = _GpuExperts.routed(impl, rows, lids, w)
    torch.testing.assert_close(got, expect, rtol=1e-6, atol=1e-6)
    if k > num_local:  # without the narrowing the FFN call is refused
        with pytest.raises(ValueError):
            _FakeLocal(num_local).expert_ffn(rows, SimpleNamespace(ids=lids, weights=w), k)


class _OracleExperts:
    """The oracle in place of the GPU side of one rank."""

    def __init__(self, ol, lo, hi, mode, k):
        self.ol, self.lo, self.hi, self.mode, self.k = ol, lo, hi, mode, k

    def route(self, x):
        from oracle import routing

        w, ids = routing.route(x.numpy() @ self.ol.router.T, self.k, self.mode)
        return torch.from_numpy(ids.astype(np.int32)), torch.from_numpy(w)

    def routed(self, rows, lids, w):
        from oracle import moe

        out = np.zeros((rows.shape[0], rows.shape[1]), np.float32)
        for r in range(rows.shape[0]):
            for j in range(lids.shape[1]):
                e = int(lids[r, j])
                if e >= 0:
                    out[r] += float(w[r, j]) * moe.expert_ffn(rows[r:r + 1].numpy(), *self.ol.w_lookup(self.lo + e))[0]
        return torch.from_numpy(out)

    def shared_out(self, x):
        from oracle import moe

        sc = self.ol.shared_cat()
        return None if sc is None else torch.from_numpy(moe.expert_ffn(x.numpy(), *sc))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, counts: list, out: dict):
    from ccut_b200.ep_a2a import AllToAllMoeLayer
    from oracle import formats, inputs, moe

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        cfg = inputs.MoeLayerConfig("a2a", hidden=128, inter=128, num_experts=6, top_k=2, num_shared=1,
                                    shared_inter=128, fmt="fp8_b128", routing="softmax_topk")
        ol = inputs.make_layer(cfg, seed=4)
        x_all = formats.bf16_bits_to_f32(ol.make_x(sum(counts)))
        start = sum(counts[:rank])
        x = torch.from_numpy(x_all[start: start + counts[rank]].copy())
        lo, hi = expert_range(6, world, rank)
        layer = AllToAllMoeLayer("fp8_b128", 128, 128, 6, 2, "softmax_topk", ol.router, ol.experts, shared=ol.shared,
                                 experts_impl=_OracleExperts(ol, lo, hi, "softmax_topk", 2))
        y = layer.forward(x, out_dtype=torch.float32)
        ref = moe.moe_forward(x.numpy(), ol.router, 2, "softmax_topk", ol.w_lookup, ol.shared_cat())[0]
        err = float(np.abs(y.numpy() - ref).max() / max(np.abs(ref).max(), 1e-30)) if len(ref) else 0.0
        out[rank] = (err, layer.rows_sent, counts[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("counts", [[5, 3], [4, 0, 7]])
def test_all_to_all_layer_matches_oracle(counts):
    world = len(counts)
    out = mp.Manager().dict()
    mp.spawn(_rank, args=(world, _free_port(), counts, out), nprocs=world, join=True)
    for r in range(world):
        err, sent, T = out[r]
        assert err < 1e-5, (r, err)
        assert sent <= T * min(2, world)  # each token at most once per destination, k = 2 destinations at most
