"""The all-to-all expert-parallel layer (``ccut_b200.ep_a2a``) on GPUs against the oracle on
the single-GPU layer's routing: world 1 in-process (the exchange degenerates to copies over
NCCL; the GPU side -- global routing, the rank's experts with -1 ids for experts elsewhere,
the shared experts as a layer of their own -- is the one every world runs), and two GPUs,
one process each (skipped on a one-GPU box)."""

from __future__ import annotations

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


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer(lw, device):
    from ccut_b200.ep_a2a import AllToAllMoeLayer

    c = lw.cfg
    return AllToAllMoeLayer(c.fmt, c.hidden, c.inter, c.num_experts, c.top_k, c.routing, lw.router, lw.experts,
                            shared=lw.shared, shared_inter=c.shared_inter, n_group=c.n_group, topk_group=c.topk_group,
                            routed_scaling=c.routed_scaling, device=device)


def _err(lw, xb, y, device):
    ref_layer = gpu_layer(lw, device=device)
    _, r = ref_layer.forward(x_device(xb, device), return_routing=True)
    ref, _, _ = oracle_forward(lw, xb, ids=r.ids.cpu().numpy(), weights=r.weights.cpu().numpy())
    return rel_err_rows(y.float().cpu().numpy(), ref)


def _run(rank, world, port, case, out):
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
    try:
        fmt, mode, E, k, shared, counts = case
        lw = inputs.make_layer(small_cfg(fmt, mode, hidden=256, inter=128, experts=E, top_k=k, shared=shared), seed=41)
        xs = lw.make_x(sum(counts))
        start = sum(counts[:rank])
        xb = xs[start: start + counts[rank]]
        dev = f"cuda:{rank}"
        layer = _layer(lw, dev)
        y = layer.forward(x_device(xb, dev), out_dtype=torch.float32)
        torch.cuda.synchronize()
        out[rank] = _err(lw, xb, y, dev) if counts[rank] else 0.0
        dist.barrier()
    finally:
        dist.destroy_process_group()


CASES = [("fp8_b128", "softmax_topk", 8, 2, 2, (11,)), ("awq_int4_g128", "topk_softmax", 16, 4, 0, (37,))]


@pytest.mark.parametrize("case", CASES)
def test_all_to_all_world1(case):
    import torch.multiprocessing as mp

    out = mp.Manager().dict()
    mp.start_processes(_run, args=(1, _free_port(), case, out), nprocs=1, join=True, start_method="spawn")
    assert out[0] <= TOL, out[0]


def test_all_to_all_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    out = mp.Manager().dict()
    case = ("fp8_b128", "softmax_topk", 8, 2, 1, (20, 9))  # ragged token counts
    mp.start_processes(_run, args=(2, _free_port(), case, out), nprocs=2, join=True, start_method="spawn")
    assert max(out.values()) <= TOL, dict(out)
