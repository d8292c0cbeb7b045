"""The reference's own weight formats on the GPU: per-channel FP8 (``fp8_channel``) and
signed int4 with fp32 scales (``int4_sym_g128``).

- Pack -> export is bit-exact against the oracle's restatement of ``fp8_dequant_mat`` /
  ``int4_dequant_row`` in both tile layouts, for routed experts and shared-expert slices.
- Both GEMM kernels multiply the exact codes and apply the fp32 scale per 128-k group: the
  down projection of one-hot rows returns the dequantized rows exactly.
- Layer outputs match the oracle within 1e-2 (both kernels, shared experts, several batch
  sizes); the quant-linear methods picked by ``make_method_for_spec`` match the reference's
  own ``apply`` outputs (fixtures made by ``tests/golden/make_golden_channel.py``); and the
  layer built from the reference ``moe_forward`` fixture's tensors reproduces its outputs."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import formats, inputs
from tests.gpu_helpers import TOL, gpu_layer, oracle_forward, rel_err_rows, small_cfg, x_device

pytestmark = pytest.mark.gpu

FMTS = ["fp8_channel", "int4_sym_g128"]


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from ccut_b200 import build
    build.build()


@pytest.mark.parametrize("layout", ["rows", "frags"])
@pytest.mark.parametrize("fmt", FMTS)
def test_dequant_export_bit_exact(fmt, layout):
    cfg = small_cfg(fmt, hidden=384, inter=256, experts=3, shared=1, shared_inter=512)
    lw = inputs.make_layer(cfg, seed=31)
    L = gpu_layer(lw)
    for e, ew in enumerate(lw.experts):
        for which in ("gate", "up", "down"):
            ref = inputs.dequant(getattr(ew, which))
            got = L.dequant(e, which, layout=layout).cpu().numpy()
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), f"expert {e} {which}"
    sh = lw.shared[0]  # two slices of 256 intermediate channels
    for s in range(2):
        for which in ("gate", "up", "down"):
            full = inputs.dequant(getattr(sh, which))
            ref = full[:, 256 * s:256 * (s + 1)] if which != "down" else full[256 * s:256 * (s + 1)]
            got = L.dequant(3 + s, which, layout=layout).cpu().numpy()
            assert np.array_equal(got.view(np.uint32), np.ascontiguousarray(ref).view(np.uint32)), (s, which)


@pytest.mark.parametrize("kernel", ["tc", "mma"])
@pytest.mark.parametrize("fmt", FMTS)
def test_down_product_is_the_exact_dequantized_weight(fmt, kernel):
    from ccut_b200.layer import Routing

    E, H, I = 4, 256, 384
    lw = inputs.make_layer(small_cfg(fmt, hidden=H, inter=I, experts=E, top_k=1), seed=5)
    if fmt == "fp8_channel":  # the smallest scale of the distribution on some channels
        lw.experts[1].down.scale[:7] = np.float32(1e-3)
    L = gpu_layer(lw, kernel=kernel)
    T = E * I if kernel == "tc" else E * 48  # mma.sync: decode-sized groups
    ids = torch.tensor([[t % E] for t in range(T)], dtype=torch.int32, device="cuda")
    w = torch.ones((T, 1), dtype=torch.float32, device="cuda")
    perm = L.permute(Routing(ids, w))
    row_token = perm.row_token[:T].cpu().numpy()
    h = torch.zeros((T, I), dtype=torch.bfloat16)
    hot = (row_token // E) % I
    h[np.arange(T), hot] = 1.0
    hcode = h.to("cuda").view(torch.int16) if kernel == "tc" else h.to(torch.float16).to("cuda").view(torch.int16)
    y = L.down(hcode, perm, T, 1).cpu().numpy()
    offs = perm.offsets.cpu().numpy()
    for e in range(E):
        wd = inputs.dequant(lw.experts[e].down)  # fp32 [I, H], the reference's dequant
        for r in range(offs[e], offs[e + 1]):
            assert np.array_equal(y[r], wd[hot[r]]), (e, r)


@pytest.mark.parametrize("kernel", ["tc", "mma"])
@pytest.mark.parametrize("fmt", FMTS)
def test_layer_matches_oracle(fmt, kernel):
    cfg = small_cfg(fmt, "topk_softmax", hidden=512, inter=256, experts=8, top_k=2, shared=1)
    lw = inputs.make_layer(cfg, seed=13)
    L = gpu_layer(lw, kernel=kernel)
    for T in (1, 7, 64, 300):
        xb = lw.make_x(T)
        out, r = L.forward(x_device(xb), out_dtype=torch.float32, return_routing=True)
        ids, wts = r.ids.cpu().numpy().astype(np.int64), r.weights.cpu().numpy()
        ref, _, _ = oracle_forward(lw, xb, ids=ids, weights=wts)
        assert rel_err_rows(out.cpu().numpy(), ref) <= TOL, T
    assert L.workspace_status() == 0


@pytest.mark.parametrize("layout", ["rows", "frags"])
def test_quant_linear_fp8_channel_matches_reference(golden_dir, layout):
    from ccut_b200 import quant, quant_spec as S

    g = np.load(golden_dir / "fp8_channel_linear.npz")
    N, K = g["w"].shape
    xb = formats.bf16_bits_to_f32(formats.bf16_bits_from_f32(g["x"]))  # the kernels read bf16 activations
    ref = xb @ formats.fp8_channel_dequant(g["w"], g["scale"]).T
    for key in ("fp8_static_channel_sym", "fp8_dynamic_token_sym"):
        spec = S.LayerQuantSpec("t.fp8", S.get_quant_key(key), scales=(S.ScaleDesc("t.fp8.weight_scale", "F32", (N,)),))
        m = quant.make_method_for_spec(spec, layout=layout)
        m.create_weights(spec)
        y = m.apply(g["w"].tobytes(), {"t.fp8.weight_scale": g["scale"]}, g["x"])
        assert y.shape == (g["x"].shape[0], N)
        assert rel_err_rows(y, ref) <= 1e-4  # exact operands: only the fp32 summation order differs
        assert rel_err_rows(y, g[f"y_{key}"]) <= TOL  # the reference's fp32 activations
    out = quant.dequantize("fp8_channel", g["w"], {"weight_scale": g["scale"]}, K, N).cpu().numpy()
    assert np.array_equal(out.view(np.uint32), g["dequant_out_in"].view(np.uint32))


@pytest.mark.parametrize("layout", ["rows", "frags"])
def test_quant_linear_int4_sym_matches_reference(golden_dir, layout):
    from ccut_b200 import quant, quant_spec as S

    g = np.load(golden_dir / "int4_sym_linear.npz")
    N, K = g["packed"].shape[0], g["packed"].shape[1] * 2
    xb = formats.bf16_bits_to_f32(formats.bf16_bits_from_f32(g["x"]))
    ref = xb @ formats.int4_sym_dequant(g["packed"], g["scale"]).T
    spec = S.LayerQuantSpec("t.int4", S.get_quant_key("int4_w4a16_sym"),
                            scales=(S.ScaleDesc("t.int4.weight_scale", "F32", (K,)),))
    m = quant.make_method_for_spec(spec, layout=layout)
    m.create_weights(spec)
    y = m.apply(g["packed"].tobytes(), {"t.int4.weight_scale": g["scale"]}, g["x"])
    assert rel_err_rows(y, ref) <= 1e-4
    assert rel_err_rows(y, g["y"]) <= TOL
    out = quant.dequantize("int4_sym_g128", g["packed"], {"weight_scale": g["scale"]}, K, N).cpu().numpy()
    assert np.array_equal(out.view(np.uint32), g["dequant_out_in"].view(np.uint32))


@pytest.mark.parametrize("kernel", ["tc", "mma"])
def test_forward_matches_reference_moe_forward_fp8_channel(golden_dir, kernel):
    """The reference ``moe_forward`` as-is with per-channel FP8: routed experts stored
    ``[in, out]`` with per-input scales (one per 128-row group), a shared expert with a
    general per-output-channel scale."""
    from ccut_b200 import MoeLayer
    from tests.golden.make_golden_channel import FIXTURE_CFG, fixture_layer

    g = np.load(golden_dir / "moe_forward_fp8ch.npz")
    router, routed, shared, xs = fixture_layer()
    c = FIXTURE_CFG

    def routed_mat(cw, s_in):  # per-input scale -> one scale per output channel per 128-k group
        return {"weight": cw, "scales": np.repeat(s_in[::128, None], cw.shape[0], axis=1)}

    experts = [{n: routed_mat(*proj[n]) for n in ("gate", "up", "down")} for proj in routed]
    sh = {n: {"weight": shared[n][0], "scale": shared[n][1]} for n in ("gate", "up", "down")}
    for norm in (False, True):
        L = MoeLayer("fp8_channel", c["hidden"], c["inter"], c["num_experts"], c["top_k"],
                     "topk_softmax" if norm else "softmax_topk", router, experts, shared=[sh],
                     shared_inter=c["shared_inter"], kernel=kernel)
        for T, xb in xs.items():
            out = L.forward(x_device(xb), out_dtype=torch.float32).cpu().numpy()
            assert rel_err_rows(out, g[f"y_norm{int(norm)}_T{T}"]) <= TOL, (norm, T)
