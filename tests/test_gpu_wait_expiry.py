"""The kernels' bounded device waits run out instead of hanging (no GPU fault is involved).

``ccut_debug_wait_expiry`` launches one small kernel that waits, with the same wait routines
(``mbar_wait``, ``mbar_spin``) and a budget of 100k SM cycles, on an mbarrier that completes and
on one that nothing ever arrives on.  The second wait expires: the kernel records
CCUT_ERR_TIMEOUT in the workspace status word and returns; the host reads it (the Python
layer raises ``TimeoutError``, the reference's class for a stalled wait,
ccut/experts/reader.py:327); the status is cleared by the read; and the next ordinary call
on the same context runs and matches the oracle."""

from __future__ import annotations

import ctypes as C

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


def test_bounded_wait_expires_and_the_context_stays_usable():
    from ccut_b200 import _lib

    lib = _lib.load()
    ws = torch.zeros(256, dtype=torch.uint8, device="cuda")
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = C.c_void_p(ws.data_ptr())
    _lib.call("ccut_debug_wait_expiry", p, 100_000, s)
    torch.cuda.synchronize()
    assert int(ws.view(torch.int32)[1]) == 1  # the completed wait passed, both idle waits ran out
    rc = lib.ccut_workspace_status(p, s)
    assert rc == _lib.ERR_TIMEOUT
    with pytest.raises(TimeoutError):
        _lib.check(rc, "ccut_debug_wait_expiry")
    assert lib.ccut_workspace_status(p, s) == 0  # the read cleared it
    # the context still runs ordinary work
    lw = inputs.make_layer(small_cfg("fp8_b128", hidden=256, inter=128, experts=8, top_k=2), seed=3)
    L = gpu_layer(lw, kernel="tc")
    xb = lw.make_x(40)
    y, r = L.forward(x_device(xb), return_routing=True)
    ref, _, _ = oracle_forward(lw, xb, ids=r.ids.cpu().numpy(), weights=r.weights.cpu().numpy())
    assert rel_err_rows(y.float().cpu().numpy(), ref) <= TOL
    assert L.workspace_status() == 0
