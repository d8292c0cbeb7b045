"""The reference-shaped drop-ins (``ccut_b200.blocks.moe``, ``ccut_b200.quant``) on the GPU
against the reference's golden vectors and the CPU oracle."""

from __future__ import annotations

from types import SimpleNamespace

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


@pytest.mark.parametrize("k", [1, 2, 6, 8])
@pytest.mark.parametrize("norm", [True, False])
def test_topk_softmax_matches_reference_golden(golden_dir, k, norm):
    from ccut_b200.blocks.moe import topk_softmax

    g = np.load(golden_dir / "topk.npz")
    tag = "norm" if norm else "soft"
    w, ids = topk_softmax(g["logits"], k, norm_topk_prob=norm)
    assert ids.dtype == np.int64 and np.array_equal(ids, g[f"ids_{tag}_k{k}"])
    np.testing.assert_allclose(w, g[f"w_{tag}_k{k}"], rtol=1e-6, atol=1e-7)
    wt, it = topk_softmax(torch.from_numpy(g["logits"]).cuda(), k, norm)
    assert it.is_cuda and torch.equal(it.cpu(), torch.from_numpy(ids))


def test_topk_values_and_ties():
    from ccut_b200.blocks.moe import topk

    x = np.array([[1.0, 3.0, 3.0, 2.0], [5.0, 5.0, 5.0, 5.0]], dtype=np.float32)
    vals, idx = topk(x, 3)
    assert np.array_equal(idx, [[1, 2, 3], [0, 1, 2]])
    assert np.array_equal(vals, [[3.0, 3.0, 2.0], [5.0, 5.0, 5.0]])


@pytest.mark.parametrize("fmt,shared", [("fp8_b128", 2), ("awq_int4_g128", 0)])
def test_moe_forward_dropin(fmt, shared):
    from ccut_b200.blocks.moe import moe_forward

    mode = "softmax_topk" if shared else "topk_softmax"
    cfg = small_cfg(fmt, mode, hidden=256, inter=128, experts=8, top_k=2, shared=shared)
    lw = inputs.make_layer(cfg, seed=41)
    L = gpu_layer(lw)
    xb = lw.make_x(19)
    h = formats.bf16_bits_to_f32(xb)  # fp32 activations, bf16-representable
    spec = SimpleNamespace(top_k=2, norm_topk_prob=mode == "topk_softmax", has_shared_expert=bool(shared))
    out = moe_forward(h, lw.router, L, 0, spec, shared_projs={} if shared else None)
    assert isinstance(out, np.ndarray) and out.dtype == np.float32
    r = L.route(x_device(xb))
    ref, _, _ = oracle_forward(lw, xb, ids=r.ids.cpu().numpy(), weights=r.weights.cpu().numpy())
    assert rel_err_rows(out, ref) <= TOL
    with pytest.raises(ValueError):
        moe_forward(h, lw.router, L, 0, SimpleNamespace(top_k=3, norm_topk_prob=spec.norm_topk_prob,
                                                        has_shared_expert=bool(shared)), {} if shared else None)


def test_moe_combine_dropin_given_routing():
    from ccut_b200.blocks.moe import moe_combine

    cfg = small_cfg("fp8_b128", hidden=256, inter=128, experts=8, top_k=3, shared=1)
    lw = inputs.make_layer(cfg, seed=43)
    L = gpu_layer(lw)
    xb = lw.make_x(11)
    x = formats.bf16_bits_to_f32(xb)
    rng = np.random.default_rng(1)
    ids = np.stack([rng.permutation(8)[:3] for _ in range(11)]).astype(np.int64)
    w = rng.random((11, 3)).astype(np.float32)
    out = moe_combine(x, ids, w, w_lookup=L)
    ref = moe.moe_combine(x, ids, w, lw.w_lookup)  # routed experts only, as in the reference
    assert rel_err_rows(out, ref) <= TOL
    # a caller's expert function gets the exported (bit-exact) weights and the token rows;
    # expert_outputs is accepted and not read, as in the reference
    calls = []

    def fn(rows, wg, wu, wd):
        calls.append(rows.shape[0])
        return moe.expert_ffn(rows, wg, wu, wd)

    out_fn = moe_combine(x, ids, w, expert_outputs={0: None}, expert_fn=fn, w_lookup=L)
    assert sum(calls) == ids.size and len(calls) == len(np.unique(ids))
    assert rel_err_rows(out_fn, ref) <= 1e-5  # the same fp32 matrices: summation order only
    out_t = moe_combine(torch.from_numpy(x).cuda(), torch.from_numpy(ids), torch.from_numpy(w), expert_fn=fn,
                        w_lookup=L)
    assert isinstance(out_t, torch.Tensor) and rel_err_rows(out_t.cpu().numpy(), ref) <= 1e-5


@pytest.mark.parametrize("layout", ["frags", "rows"])
def test_quant_methods_apply(layout):
    from ccut_b200.quant import AwqInt4G128Method, Fp8Block128Method

    cfg = small_cfg("awq_int4_g128", hidden=256, inter=128, experts=1)
    a = inputs.make_layer(cfg, seed=5).experts[0].gate  # K = 256, N = 128
    x = np.random.default_rng(2).standard_normal((9, 256)).astype(np.float32)
    xr = formats.bf16_bits_to_f32(formats.bf16_bits_from_f32(x))
    m = AwqInt4G128Method(256, 128, layout=layout)
    y = m.apply(a.qweight.tobytes(), {"scales": a.scales, "qzeros": a.qzeros}, x)
    assert rel_err_rows(y, xr @ inputs.dequant(a)) <= 2e-3
    with pytest.raises(ValueError):
        m.apply(a.qweight, {"scales": a.scales}, x)
    f = inputs.make_layer(small_cfg("fp8_b128", hidden=256, inter=128, experts=1), seed=6).experts[0].up
    mf = Fp8Block128Method(256, 128, layout=layout)
    yf = mf.apply(f.weight, {"weight_scale_inv": f.scale}, torch.from_numpy(x).cuda())
    assert yf.is_cuda
    assert rel_err_rows(yf.cpu().numpy(), xr @ inputs.dequant(f)) <= 2e-3
