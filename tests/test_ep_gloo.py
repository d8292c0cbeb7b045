"""Expert-parallel decomposition on CPU ranks (gloo, world_size 2).

The partition (``ccut_b200.ep.expert_range``) and the pair localization
(``ccut_b200.ep.localize_ids``) are the host-side logic of the expert-parallel layer.
Here they drive an all-gather -> local experts -> reduce -> shared-expert pipeline whose
expert compute is the CPU oracle, and the result must equal the single-process oracle
layer on the same routing.  gloo has no reduce-scatter, so the combine is an all-reduce
followed by the rank's slice."""

from __future__ import annotations

import datetime
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ccut_b200.ep import expert_range, localize_ids


def test_expert_range_partitions_every_expert():
    for E in (2, 8, 64, 66, 128, 256):
        for world in (1, 2, 3, 4, 8):
            if E < world:
                continue
            ranges = [expert_range(E, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == E
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [hi - lo for lo, hi in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        expert_range(4, 8, 0)
    with pytest.raises(ValueError):
        expert_range(8, 2, 2)


def test_localize_ids_numpy_and_torch_agree():
    ids = np.array([[0, 5, 9], [3, 4, 11], [-1, 12, 6]], dtype=np.int32)
    want = np.array([[-1, 1, -1], [-1, 0, -1], [-1, -1, 2]], dtype=np.int32)
    assert np.array_equal(localize_ids(ids, 4, 8), want)
    assert torch.equal(localize_ids(torch.from_numpy(ids), 4, 8), torch.from_numpy(want))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, cfg_kw: dict, T: int, out: dict):
    from oracle import formats, inputs, moe, routing

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        cfg = inputs.MoeLayerConfig(**cfg_kw)
        lw = inputs.make_layer(cfg, seed=3)
        Tl = T // world
        x_all_b = lw.make_x(T)
        x_r = formats.bf16_bits_to_f32(x_all_b[rank * Tl:(rank + 1) * Tl])
        # 1. route the local tokens
        weights, ids = routing.route(x_r @ lw.router.T, cfg.top_k, cfg.routing, **cfg.route_kw)
        # 2. dispatch
        xs = [torch.empty(Tl, cfg.hidden) for _ in range(world)]
        dist.all_gather(xs, torch.from_numpy(x_r))
        ids_l = [torch.empty(Tl, cfg.top_k, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(ids_l, torch.from_numpy(ids.astype(np.int64)))
        w_l = [torch.empty(Tl, cfg.top_k) for _ in range(world)]
        dist.all_gather(w_l, torch.from_numpy(weights.astype(np.float32)))
        x_all = torch.cat(xs).numpy()
        ids_all = torch.cat(ids_l).numpy()
        w_all = torch.cat(w_l).numpy()
        # 3. local experts on the pairs routed to them
        lo, hi = expert_range(cfg.num_experts, world, rank)
        loc = localize_ids(ids_all, lo, hi)
        y_part = np.zeros((T, cfg.hidden), dtype=np.float32)
        for e in range(hi - lo):
            t_idx, j_idx = np.nonzero(loc == e)
            if t_idx.size:
                wg, wu, wd = lw.w_lookup(lo + e)
                y = moe.expert_ffn(x_all[t_idx], wg, wu, wd)
                np.add.at(y_part, t_idx, w_all[t_idx, j_idx][:, None] * y)
        # 4. combine: reduce, keep this rank's tokens
        yt = torch.from_numpy(y_part)
        dist.all_reduce(yt)
        y_loc = yt.numpy()[rank * Tl:(rank + 1) * Tl]
        # 5. shared experts on the local tokens
        if lw.shared:
            y_loc = y_loc + moe.expert_ffn(x_r, *lw.shared_cat())
        ref, _, _ = moe.moe_forward(formats.bf16_bits_to_f32(x_all_b), lw.router, cfg.top_k, cfg.routing, lw.w_lookup,
                                    shared=lw.shared_cat(), ids=ids_all, weights=w_all)
        ref = ref[rank * Tl:(rank + 1) * Tl]
        err = float(np.abs(y_loc - ref).max() / max(np.abs(ref).max(), 1e-30))
        out[rank] = (err, int((loc >= 0).sum()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("routing_mode,shared", [("softmax_topk", 2), ("topk_softmax", 0)])
def test_ep_decomposition_two_ranks(routing_mode, shared):
    world, T = 2, 24
    cfg_kw = dict(name="ep_t", hidden=256, inter=128, num_experts=8, top_k=3, num_shared=shared, shared_inter=128,
                  fmt="awq_int4_g128", routing=routing_mode)
    mgr = mp.Manager()
    out = mgr.dict()
    mp.start_processes(_rank_main, args=(world, _free_port(), cfg_kw, T, out), nprocs=world, join=True,
                       start_method="spawn")
    assert sorted(out.keys()) == [0, 1]
    assert sum(n for _, n in out.values()) == T * cfg_kw["top_k"]  # every pair ran on exactly one rank
    for rank, (err, _) in out.items():
        assert err <= 1e-5, f"rank {rank}: rel err {err}"
