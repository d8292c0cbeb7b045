"""Parity at the BASELINE.json layer sizes and at the routing limits.

Full-size layers (configs 0, 1 and 3: H = 2048, 64 or 128 experts) are checked against the
oracle on a token subset (the oracle dequantizes only the experts those tokens touch), and
through a size-independent property: a token's output does not depend on the batch it
came in.  A decode-sized and a prefill-sized batch run different kernels (mma.sync vs
tcgen05), so the property also ties the two kernels together at full size."""

from __future__ import annotations

import numpy as np
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


_LAYERS: dict = {}


def _layer(name):
    if name not in _LAYERS:
        _LAYERS.clear()  # one full-size layer resident at a time
        lw = inputs.make_layer(name, seed=0)
        _LAYERS[name] = (lw, gpu_layer(lw))
    return _LAYERS[name]


@pytest.mark.parametrize("name", ["cfg0", "cfg1", "cfg3"])
def test_full_size_layer_matches_oracle(name):
    lw, L = _layer(name)
    xb = lw.make_x(12)
    y, r = L.forward(x_device(xb), return_routing=True)
    ref, _, _ = oracle_forward(lw, xb, ids=r.ids.cpu().numpy(), weights=r.weights.cpu().numpy())
    assert rel_err_rows(y.float().cpu().numpy(), ref) <= TOL
    assert L.workspace_status() == 0


@pytest.mark.parametrize("name", ["cfg0", "cfg1"])
def test_full_size_output_is_batch_independent(name):
    lw, L = _layer(name)
    xb = lw.make_x(2048)  # prefill: the tcgen05 kernel
    big = L.forward(x_device(xb)).float().cpu().numpy()
    small = L.forward(x_device(xb[:64])).float().cpu().numpy()  # decode: the mma.sync kernel
    one = L.forward(x_device(xb[5:6])).float().cpu().numpy()
    assert rel_err_rows(small, big[:64]) <= TOL
    assert rel_err_rows(one, big[5:6]) <= TOL


def test_full_size_dequant_export_bit_exact():
    lw, L = _layer("cfg1")
    for e in (0, 37, 63):
        got = L.dequant(e, "down").cpu().numpy()
        assert np.array_equal(got.view(np.uint32), inputs.dequant(lw.experts[e].down).view(np.uint32))


@pytest.mark.parametrize("kernel", ["tc", "mma"])
def test_routing_limits_256_experts_top16(kernel):
    cfg = small_cfg("awq_int4_g128", "topk_softmax", hidden=256, inter=128, experts=256, top_k=16)
    lw = inputs.make_layer(cfg, seed=17)
    L = gpu_layer(lw, kernel=kernel)
    xb = lw.make_x(33)
    y, r = L.forward(x_device(xb), return_routing=True)
    ids = r.ids.cpu().numpy()
    assert ids.shape == (33, 16) and all(len(set(row)) == 16 for row in ids.tolist())
    ref, _, _ = oracle_forward(lw, xb, ids=ids, weights=r.weights.cpu().numpy())
    assert rel_err_rows(y.float().cpu().numpy(), ref) <= TOL


def test_routing_beyond_limits_is_rejected():
    cfg = small_cfg("fp8_b128", hidden=128, inter=128, experts=8, top_k=2)
    L = gpu_layer(inputs.make_layer(cfg, seed=1))
    logits = torch.zeros(4, 300, device="cuda")
    with pytest.raises((ValueError, NotImplementedError)):
        L.topk(logits)
