"""The ``ExpertPipeline`` drop-in on the GPU (``ccut_b200.experts``, one ``ccut_moe_forward`` per
step over resident experts) against the oracle's MoE layer on the same routing: with and
without shared experts, a per-call shared gate, the routing history and the step counters."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import formats, inputs, moe
from tests.gpu_helpers import TOL, gpu_layer, oracle_forward, rel_err_rows, small_cfg, x_device

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from ccut_b200 import build
    build.build()


@pytest.mark.parametrize("fmt, mode, shared", [("fp8_b128", "softmax_topk", 1), ("awq_int4_g128", "topk_softmax", 0)])
def test_pipeline_step_matches_oracle(fmt, mode, shared):
    from ccut_b200.experts import ExpertPipeline

    lw = inputs.make_layer(small_cfg(fmt, mode, hidden=256, inter=128, experts=8, top_k=2, shared=shared), seed=21)
    L = gpu_layer(lw)
    pipe = ExpertPipeline({3: L})
    xb = lw.make_x(9)
    x = formats.bf16_bits_to_f32(xb)
    projs = {"gate_proj": None, "up_proj": None, "down_proj": None} if shared else None
    gates = (1.0, 0.5) if shared else (1.0,)
    for gate in gates:
        y = pipe.step(3, x, lw.router, top_k=2, norm_topk_prob=mode == "topk_softmax", shared_projs=projs,
                      shared_gate=gate)
        assert isinstance(y, np.ndarray) and y.shape == (9, 256) and y.dtype == np.float32
        r = L.route(x_device(xb))  # the same routing kernels as the step
        ids, w = r.ids.cpu().numpy().astype(np.int64), r.weights.cpu().numpy()
        if gate == 1.0:
            ref = oracle_forward(lw, xb, ids=ids, weights=w)[0]
        else:
            ref = moe.moe_forward(x, lw.router, 2, mode, lw.w_lookup, lw.shared_cat(), shared_gate=gate, ids=ids,
                                  weights=w)[0]
        assert rel_err_rows(y, ref) <= TOL, gate
    assert L.shared_gate == 1.0  # the per-call gate is not kept
    assert pipe.metrics.steps == len(gates) and pipe.metrics.compute_ns > 0
    assert len(pipe.history.predict(2)) == 2
    yt = pipe.step(3, x_device(xb), lw.router, top_k=2, norm_topk_prob=mode == "topk_softmax", shared_projs=projs)
    assert yt.is_cuda
