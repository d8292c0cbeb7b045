"""ccut_moe_permute_static (scratch in a fixed device array, no workspace) against
ccut_moe_permute (caller workspace), both through the C ABI.

The permutation is integer work, so the bar is bit-exact.  Two calls in a row with
different routings check that the fixed counters start from zero on every call.  This
file is collected last and also runs alone in a fresh process."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_EXPERTS = 256  # CCUT_PERMUTE_STATIC_MAX_EXPERTS in include/ccut_moe.h


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from ccut_b200 import build
    build.build()


def _p(t):
    return C.c_void_p(t.data_ptr() if t is not None else 0)


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _routing(T, k, E, seed):
    rng = np.random.default_rng(seed)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    ids[: T // 8] = np.arange(k, dtype=np.int32)  # pile some pairs onto the first experts
    w = rng.random((T, k)).astype(np.float32)
    return torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda()


def _outputs(T, k, E, slices):
    R = T * k + slices * T
    return (torch.full((E + slices + 1,), -7, dtype=torch.int32, device="cuda"),
            torch.full((max(R, 1),), -7, dtype=torch.int32, device="cuda"),
            torch.full((max(R, 1),), -7.0, dtype=torch.float32, device="cuda"),
            torch.full((max(T * k, 1),), -7, dtype=torch.int32, device="cuda"))


def _permute_workspace(ids, w, T, k, E, slices, gate):
    from ccut_b200 import _lib

    out = _outputs(T, k, E, slices)
    nbytes = _lib.load().ccut_permute_workspace_bytes(E)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    _lib.call("ccut_moe_permute", _p(ids), _p(w), T, k, E, slices, C.c_float(gate), *map(_p, out), _p(ws),
              nbytes, _stream())
    return out


def _permute_static(ids, w, T, k, E, slices, gate):
    from ccut_b200 import _lib

    out = _outputs(T, k, E, slices)
    _lib.call("ccut_moe_permute_static", _p(ids), _p(w), T, k, E, slices, C.c_float(gate), *map(_p, out),
              _stream())
    return out


@pytest.mark.parametrize("T,k,E,slices", [(333, 4, 16, 1), (1000, 8, MAX_EXPERTS, 0), (64, 6, 64, 2)])
def test_static_scratch_matches_workspace_entry_point(T, k, E, slices):
    for seed in (11, 12):  # two calls in a row: the fixed counters must restart from zero
        ids, w = _routing(T, k, E, seed)
        ref = _permute_workspace(ids, w, T, k, E, slices, 0.5)
        got = _permute_static(ids, w, T, k, E, slices, 0.5)
        torch.cuda.synchronize()
        for name, a, b in zip(("offsets", "row_token", "row_weight", "pair_row"), got, ref):
            assert torch.equal(a, b), f"{name} differs (seed {seed})"


@pytest.mark.parametrize("case", ["unrouted", "empty"])
def test_static_scratch_unrouted_pairs_and_empty_batch(case):
    """Pairs without an expert (-1, or an id of E or more) get pair_row -1 from the kernel
    itself (the outputs start at -7, so a missing write would show), and T = 0 writes the
    offsets only; bit-exact against the workspace entry point, two calls in a row."""
    T, k, E, slices = (50, 4, 16, 1) if case == "unrouted" else (0, 4, 16, 2)
    for seed in (21, 22):
        if T:
            ids, w = _routing(T, k, E, seed)
            rng = np.random.default_rng(seed)
            bad = torch.from_numpy(rng.choice(np.array([-1, E, E + 3], np.int32), size=(T, k))).cuda()
            drop = torch.from_numpy(rng.random((T, k)) < 0.3).cuda()
            ids = torch.where(drop, bad, ids).contiguous()
        else:
            ids = torch.zeros((0, k), dtype=torch.int32, device="cuda")
            w = torch.zeros((0, k), dtype=torch.float32, device="cuda")
        ref = _permute_workspace(ids, w, T, k, E, slices, 0.5)
        got = _permute_static(ids, w, T, k, E, slices, 0.5)
        torch.cuda.synchronize()
        for name, a, b in zip(("offsets", "row_token", "row_weight", "pair_row"), got, ref):
            assert torch.equal(a, b), f"{name} differs (seed {seed})"
        if T:
            assert torch.equal(got[3].view(T, k) == -1, drop), "pair_row -1 exactly where unrouted"
        else:
            assert got[0].tolist() == [0] * (E + 1) + [0] * slices


def test_static_scratch_rejects_too_many_experts():
    ids, w = _routing(8, 2, 8, 0)
    with pytest.raises(NotImplementedError):
        _permute_static(ids, w, 8, 2, MAX_EXPERTS + 1, 0, 1.0)
