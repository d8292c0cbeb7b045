"""A MoE layer loaded from a safetensors checkpoint into HBM (ccut_b200.checkpoint) runs
the same as the layer built from the same tensors in memory, and matches the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from ccut_b200 import checkpoint as ck
from oracle import inputs
from tests.ckpt_helpers import write_checkpoint
from tests.gpu_helpers import TOL, gpu_layer, oracle_forward, rel_err_rows, small_cfg, x_device

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from ccut_b200 import build
    build.build()


@pytest.mark.parametrize("kernel", ["tc", "mma"])
@pytest.mark.parametrize("fmt,mode,shared", [("awq_int4_g128", "softmax_topk", 2), ("fp8_b128", "topk_softmax", 1),
                                             ("awq_int4_g128", "topk_softmax", 0), ("fp8_channel", "topk_softmax", 1),
                                             ("int4_sym_g128", "softmax_topk", 1)])
def test_checkpoint_layer_matches_in_memory_layer(tmp_path, fmt, mode, shared, kernel):
    cfg = small_cfg(fmt, mode, hidden=384, inter=256, experts=8, top_k=2, shared=shared)
    lw = inputs.make_layer(cfg, seed=31)
    # the per-channel formats come in compressed-tensors checkpoints only
    root = write_checkpoint(tmp_path / "m", lw, layer=7, ct=fmt in ("fp8_channel", "int4_sym_g128"))
    L = ck.load_moe_layer(root, 7, kernel=kernel)
    ref_layer = gpu_layer(lw, kernel=kernel)
    for T in (1, 9, 70):
        xb = lw.make_x(T)
        x = x_device(xb)
        out, r = L.forward(x, out_dtype=torch.float32, return_routing=True)
        assert torch.equal(out, ref_layer.forward(x, out_dtype=torch.float32))
        ref, _, _ = oracle_forward(lw, xb, ids=r.ids.cpu().numpy().astype(np.int64), weights=r.weights.cpu().numpy())
        assert rel_err_rows(out.cpu().numpy(), ref) <= TOL
    assert L.workspace_status() == 0
