"""Expert-parallel layer (``ccut_moe_ep_*`` over NCCL) against the CPU oracle.

World size 1 runs in-process on one GPU (the NCCL collectives degenerate to copies, every
other stage is the multi-GPU code path).  The two-GPU case spawns one process per GPU and
is skipped on a one-GPU box.  Each rank compares its own tokens with the oracle evaluated
on the routing the single-GPU layer chooses for the same tokens (identical logits)."""

from __future__ import annotations

import ctypes as C
import datetime
import socket

import pytest
import torch

from oracle import inputs
from tests.gpu_helpers import TOL, gpu_layer, oracle_forward, rel_err_rows, small_cfg, x_device

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from ccut_b200 import build
    build.build()


def _ep_layer(lw, rank, world, **kw):
    from ccut_b200.ep import ExpertParallelMoeLayer

    c = lw.cfg
    return ExpertParallelMoeLayer(
        c.fmt, c.hidden, c.inter, c.num_experts, c.top_k, c.routing, lw.router, lw.experts, shared=lw.shared,
        shared_inter=c.shared_inter, n_group=c.n_group, topk_group=c.topk_group, routed_scaling=c.routed_scaling,
        rank=rank, world=world, **kw)


def _check_rank(lw, xb, out, kernel):
    """Error of out (this rank's tokens) vs the oracle on the single-GPU layer's routing."""
    ref_layer = gpu_layer(lw, kernel=kernel)
    _, r = ref_layer.forward(x_device(xb), return_routing=True)
    ref, _, _ = oracle_forward(lw, xb, ids=r.ids.cpu().numpy(), weights=r.weights.cpu().numpy())
    y = out.float().cpu().numpy()
    return rel_err_rows(y, ref)


EP_CASES = [
    ("fp8_b128", "softmax_topk", 8, 2, 2, 3),
    ("awq_int4_g128", "topk_softmax", 16, 4, 0, 37),
    ("fp8_b128", "sigmoid_group", 16, 4, 1, 130),
]


@pytest.mark.parametrize("kernel", ["tc", "mma"])
@pytest.mark.parametrize("fmt,mode,E,k,shared,T", EP_CASES)
def test_ep_world1_matches_oracle(fmt, mode, E, k, shared, T, kernel):
    kw = dict(n_group=4, topk_group=2, routed_scaling=2.5) if mode == "sigmoid_group" else {}
    cfg = small_cfg(fmt, mode, hidden=256, inter=128, experts=E, top_k=k, shared=shared, **kw)
    lw = inputs.make_layer(cfg, seed=21)
    xb = lw.make_x(T)
    ep = _ep_layer(lw, 0, 1, kernel=kernel)
    out = ep.forward(x_device(xb))
    torch.cuda.synchronize()
    assert ep.workspace_status() == 0
    err = _check_rank(lw, xb, out, kernel)
    ep.close()
    assert err <= TOL, err


def test_ep_dispatch_and_combine_world1():
    """The routed-rows exchange on one rank: a token goes to the rank once if any of its ids is
    a global expert in [0, E) and never if none is; its ids arrive made local (-1 elsewhere);
    combine returns each token's partial row (0 for a token that went nowhere)."""
    from ccut_b200 import _lib
    from ccut_b200.ep import _broadcast_unique_id

    lib = _lib.load()
    uid = _broadcast_unique_id(lib, 0, 1, None)
    buf = (C.c_char * len(uid)).from_buffer_copy(uid)
    h = C.c_void_p()
    _lib.call("ccut_ep_init", C.cast(buf, C.c_void_p), 0, 1, C.c_double(30.0), C.byref(h))
    try:
        T, H, k, E = 9, 256, 3, 8
        x = torch.randn(T, H, device="cuda").to(torch.bfloat16)
        ids = torch.randint(0, E, (T, k), device="cuda", dtype=torch.int32)
        ids[2] = -1  # token 2 routed nowhere
        w = torch.rand(T, k, device="cuda")
        xr = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
        ir = torch.empty(T, k, dtype=torch.int32, device="cuda")
        wr = torch.empty(T, k, device="cuda")
        nb = lib.ccut_moe_ep_exchange_workspace_bytes(1, T, H, k)
        ws = torch.zeros(nb, dtype=torch.uint8, device="cuda")
        s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
        nrecv = C.c_int(-1)
        _lib.call("ccut_moe_ep_dispatch", h, p(x), p(ids), p(w), T, T, H, k, E, p(xr), p(ir), p(wr), T,
                  C.byref(nrecv), p(ws), nb, s)
        torch.cuda.synchronize()
        sent = [t for t in range(T) if t != 2]
        assert nrecv.value == T  # one segment of T_cap rows from the one rank
        assert torch.equal(xr[:len(sent)], x[sent]) and torch.equal(ir[:len(sent)], ids[sent])
        assert torch.equal(wr[:len(sent)], w[sent])
        assert (ir[len(sent):] == -1).all()  # the segment's unused row takes no expert
        y = torch.randn(T, H, device="cuda").to(torch.bfloat16)
        yl = torch.full((T, H), 7.0, device="cuda")
        _lib.call("ccut_moe_ep_combine", h, p(y), T, T, H, k, p(yl), p(ws), nb, s)
        torch.cuda.synchronize()
        assert torch.equal(yl[sent], y[:len(sent)].float()) and torch.equal(yl[2], torch.zeros(H, device="cuda"))
        with pytest.raises(ValueError):
            _lib.call("ccut_moe_ep_combine", h, p(y), -1, T, H, k, p(yl), p(ws), nb, s)
        with pytest.raises(ValueError):  # more tokens than the workspace was planned for
            _lib.call("ccut_moe_ep_dispatch", h, p(x), p(ids), p(w), T, T - 1, H, k, E, p(xr), p(ir), p(wr), T,
                      C.byref(nrecv), p(ws), nb, s)
    finally:
        _lib.call("ccut_ep_destroy", h)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, case, out):
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        fmt, mode, E, k, shared, T, kernel = case
        cfg = small_cfg(fmt, mode, hidden=256, inter=128, experts=E, top_k=k, shared=shared)
        lw = inputs.make_layer(cfg, seed=33)
        counts = T if isinstance(T, tuple) else (T // world,) * world  # tokens per rank (may differ)
        start = sum(counts[:rank])
        xb = lw.make_x(sum(counts))[start:start + counts[rank]]
        ep = _ep_layer(lw, rank, world, kernel=kernel, device=f"cuda:{rank}", timeout_s=60.0,
                       max_tokens=max(counts))
        y = ep.forward(x_device(xb, f"cuda:{rank}"))
        torch.cuda.synchronize()
        status = ep.workspace_status()
        err = _check_rank(lw, xb, y, kernel) if counts[rank] else 0.0
        ep.close()
        out[rank] = (err, status)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", [("fp8_b128", "softmax_topk", 8, 2, 2, 64, "tc"),
                                  ("awq_int4_g128", "topk_softmax", 16, 4, 0, 32, "mma"),
                                  # ragged token counts; top-6 over 4 experts per rank
                                  ("fp8_b128", "softmax_topk", 8, 6, 1, (40, 24), "tc"),
                                  # a rank with no tokens still takes part in the exchange
                                  ("awq_int4_g128", "topk_softmax", 16, 4, 1, (33, 0), "mma")])
def test_ep_two_gpus(case):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    mgr = mp.Manager()
    out = mgr.dict()
    mp.start_processes(_rank_main, args=(2, _free_port(), case, out), nprocs=2, join=True, start_method="spawn")
    assert sorted(out.keys()) == [0, 1]
    for rank, (err, status) in out.items():
        assert status == 0 and err <= TOL, f"rank {rank}: err {err} status {status}"
