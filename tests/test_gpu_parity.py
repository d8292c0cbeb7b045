"""Parity of the CUDA path (through the C ABI) with the CPU oracle and the reference's
own outputs (golden fixtures).

Bars: bit-exact for dequantized weights, routing ids (on identical logits) and the
permutation; max relative error per token row <= 1e-2 for the layer output (bf16 out,
fp32 accumulation)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import formats, inputs, routing
from tests.gpu_helpers import (TOL, gpu_layer, ids_match_except_near_ties, oracle_forward, oracle_scores,
                               rel_err_rows, small_cfg, x_device)

pytestmark = pytest.mark.gpu

FMTS = ["awq_int4_g128", "fp8_b128"]


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from ccut_b200 import build
    build.build()


# ---------------------------------------------------------------- dequant export
LAYOUTS = ["rows", "frags"]
KERNELS = ["tc", "mma"]


@pytest.mark.parametrize("layout", LAYOUTS)
@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("order", ["awq", "sequential"])
def test_dequant_export_bit_exact(fmt, order, layout):
    if fmt == "fp8_b128" and order == "sequential":
        pytest.skip("nibble order is an AWQ-only parameter")
    cfg = small_cfg(fmt, hidden=384, inter=256, experts=3, shared=1)
    lw = inputs.make_layer(cfg, seed=21)
    if order == "sequential":  # repack the same nibbles in sequential order
        for ew in lw.experts + lw.shared:
            for m in (ew.gate, ew.up, ew.down):
                m.qweight = formats.awq_pack(formats.awq_unpack(m.qweight, "awq"), "sequential")
                m.qzeros = formats.awq_pack(formats.awq_unpack(m.qzeros, "awq"), "sequential")
        L = gpu_layer(lw, nibble_order="sequential")
        deq = lambda m: formats.awq_dequant(m.qweight, m.qzeros, m.scales, order="sequential")  # noqa: E731
    else:
        L = gpu_layer(lw)
        deq = inputs.dequant
    for e, ew in enumerate(lw.experts + lw.shared):
        for which in ("gate", "up", "down"):
            ref = deq(getattr(ew, which)).astype(np.float32)
            got = L.dequant(e, which, layout=layout).cpu().numpy()
            assert got.shape == ref.shape
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), f"expert {e} {which}"


@pytest.mark.parametrize("layout", [0, 1])
def test_dequant_export_e4m3_all_codes_and_nan(layout):
    """Every e4m3 code (incl. the two NaN codes) through pack -> export."""
    import ctypes as C
    from ccut_b200 import _lib
    lib = _lib.load()
    K = N = 128
    codes = np.arange(K * N, dtype=np.int64) % 256
    w = codes.astype(np.uint8).reshape(N, K)
    s = np.array([[0.37]], dtype=np.float32)
    wd, sd = torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda()
    nbytes = lib.ccut_packed_matrix_bytes(_lib.FMT_FP8_E4M3_B128, K, N)
    packed = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.call("ccut_pack_matrix", _lib.FMT_FP8_E4M3_B128, layout, C.c_void_p(wd.data_ptr()), None,
              C.c_void_p(sd.data_ptr()), K, N, 0, C.c_void_p(packed.data_ptr()), 1, 0, st)
    out = torch.empty((K, N), dtype=torch.float32, device="cuda")
    _lib.call("ccut_dequant_matrix", _lib.FMT_FP8_E4M3_B128, layout, C.c_void_p(packed.data_ptr()), K, N, 1, 0,
              C.c_void_p(out.data_ptr()), st)
    got = out.cpu().numpy().T  # [N, K]
    ref = formats.fp8_block_dequant(w, s)
    nan = np.isnan(ref)
    assert np.array_equal(nan, np.isnan(got)) and nan.any()
    assert np.array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32))


# ---------------------------------------------------------------- routing
@pytest.mark.parametrize("k", [1, 2, 6, 8])
def test_topk_ids_bit_exact_on_reference_logits(golden_dir, k):
    g = np.load(golden_dir / "topk.npz")
    lg = g["logits"]
    for mode, tag in (("softmax_topk", "soft"), ("topk_softmax", "norm")):
        cfg = small_cfg("fp8_b128", mode, hidden=128, inter=128, experts=64, top_k=k)
        L = gpu_layer(inputs.make_layer(cfg, seed=1))
        r = L.topk(torch.from_numpy(lg).cuda())
        assert np.array_equal(r.ids.cpu().numpy().astype(np.int64), g[f"ids_{tag}_k{k}"])
        np.testing.assert_allclose(r.weights.cpu().numpy(), g[f"w_{tag}_k{k}"], rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("mode,E,k", [("softmax_topk", 64, 6), ("topk_softmax", 128, 8), ("softmax_topk", 256, 8),
                                      ("topk_softmax", 8, 1), ("softmax_topk", 32, 16)])
def test_topk_ids_bit_exact_random(mode, E, k):
    rng = np.random.default_rng(E * 31 + k)
    lg = rng.standard_normal((777, E)).astype(np.float32)
    lg[5, :] = 1.25  # a fully tied row
    lg[6, 3:9] = 9.0  # ties at the top
    cfg = small_cfg("awq_int4_g128", mode, hidden=128, inter=128, experts=E, top_k=k)
    L = gpu_layer(inputs.make_layer(cfg, seed=2))
    r = L.topk(torch.from_numpy(lg).cuda())
    w_ref, ids_ref = routing.route(lg, k, mode)
    assert np.array_equal(r.ids.cpu().numpy().astype(np.int64), ids_ref)
    np.testing.assert_allclose(r.weights.cpu().numpy(), w_ref, rtol=1e-5, atol=1e-7)


def test_grouped_sigmoid_topk_matches_oracle():
    rng = np.random.default_rng(17)
    E, k = 256, 8
    lg = rng.standard_normal((300, E)).astype(np.float32) * 2
    cfg = small_cfg("fp8_b128", "sigmoid_group", hidden=128, inter=128, experts=E, top_k=k, n_group=8,
                    topk_group=4, routed_scaling=2.5)
    L = gpu_layer(inputs.make_layer(cfg, seed=3))
    r = L.topk(torch.from_numpy(lg).cuda())
    w_ref, ids_ref = routing.grouped_sigmoid_topk(lg, k, 8, 4, 2.5)
    got = r.ids.cpu().numpy().astype(np.int64)
    s = 1 / (1 + np.exp(-lg.astype(np.float64)))
    bad = ids_match_except_near_ties(got, ids_ref, s, k)
    assert bad.size == 0
    same = (got == ids_ref).all(axis=1)
    assert same.mean() > 0.98
    np.testing.assert_allclose(r.weights.cpu().numpy()[same], w_ref[same], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("fmt,mode", [("fp8_b128", "softmax_topk"), ("awq_int4_g128", "topk_softmax")])
def test_route_logits_and_ids(fmt, mode):
    cfg = small_cfg(fmt, mode, hidden=512, inter=128, experts=64, top_k=6)
    lw = inputs.make_layer(cfg, seed=4)
    L = gpu_layer(lw)
    for T in (1, 7, 64, 300):
        xb = lw.make_x(T)
        r = L.route(x_device(xb), want_logits=True)
        lg_ref = formats.bf16_bits_to_f32(xb) @ lw.router.T
        np.testing.assert_allclose(r.logits.cpu().numpy(), lg_ref, rtol=1e-4, atol=1e-5)
        # identical logits -> bit-exact ids
        w_ref, ids_ref = routing.route(r.logits.cpu().numpy(), cfg.top_k, mode)
        assert np.array_equal(r.ids.cpu().numpy().astype(np.int64), ids_ref)
        np.testing.assert_allclose(r.weights.cpu().numpy(), w_ref, rtol=1e-5, atol=1e-7)
        # from x: equal to the oracle except at near-ties
        _, ids_x = routing.route(lg_ref, cfg.top_k, mode)
        assert ids_match_except_near_ties(r.ids.cpu().numpy(), ids_x, oracle_scores(lw, xb), cfg.top_k).size == 0


def test_route_logits_prefill_sizes():
    """From 256 tokens on the router is split once into bf16 planes and the logits GEMM is
    pipelined: partial expert tiles (E = 72) and odd token counts against the fp32 oracle."""
    cfg = small_cfg("awq_int4_g128", "topk_softmax", hidden=384, inter=128, experts=72, top_k=4)
    lw = inputs.make_layer(cfg, seed=14)
    L = gpu_layer(lw)
    for T in (255, 256, 513, 1100):
        xb = lw.make_x(T)
        r = L.route(x_device(xb), want_logits=True)
        lg_ref = formats.bf16_bits_to_f32(xb) @ lw.router.T
        np.testing.assert_allclose(r.logits.cpu().numpy(), lg_ref, rtol=1e-4, atol=1e-5)
        w_ref, ids_ref = routing.route(r.logits.cpu().numpy(), cfg.top_k, "topk_softmax")
        assert np.array_equal(r.ids.cpu().numpy().astype(np.int64), ids_ref)


# ---------------------------------------------------------------- permutation
def test_permute_stable_counting_sort():
    cfg = small_cfg("fp8_b128", hidden=128, inter=128, experts=16, top_k=4, shared=1)
    L = gpu_layer(inputs.make_layer(cfg, seed=5))
    rng = np.random.default_rng(6)
    T, k, E = 333, 4, 16
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    ids[:40] = np.array([3, 0, 1, 2])  # pile onto a few experts; expert 15 may stay empty
    w = rng.random((T, k)).astype(np.float32)
    p = L.permute(type("R", (), {"ids": torch.from_numpy(ids).cuda(), "weights": torch.from_numpy(w).cuda()})())
    offs, rt, rw, pr = (p.offsets.cpu().numpy(), p.row_token.cpu().numpy(), p.row_weight.cpu().numpy(),
                        p.pair_row.cpu().numpy())
    flat = ids.reshape(-1)
    order = np.argsort(flat, kind="stable")  # stable by (t, j)
    counts = np.bincount(flat, minlength=E)
    assert np.array_equal(offs[:E + 1], np.concatenate([[0], np.cumsum(counts)]))
    assert offs[E + 1] == T * k + T
    assert np.array_equal(rt[:T * k], order // k)
    assert np.array_equal(rw[:T * k], w.reshape(-1)[order])
    inv = np.empty(T * k, dtype=np.int64)
    inv[order] = np.arange(T * k)
    assert np.array_equal(pr, inv)
    assert np.array_equal(rt[T * k:], np.arange(T)) and np.all(rw[T * k:] == 1.0)


# ---------------------------------------------------------------- whole layer
CASES = [
    # fmt, routing, experts, top_k, shared, hidden, inter, tokens
    ("awq_int4_g128", "softmax_topk", 8, 2, 0, 256, 128, (1, 3, 17, 64)),
    ("fp8_b128", "softmax_topk", 8, 2, 2, 256, 128, (1, 3, 17, 64)),
    ("awq_int4_g128", "topk_softmax", 16, 4, 1, 384, 256, (1, 5, 130)),
    ("fp8_b128", "topk_softmax", 16, 6, 0, 512, 384, (2, 33, 200)),
    ("fp8_b128", "sigmoid_group", 32, 4, 1, 256, 128, (9, 100)),
]


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("fmt,mode,E,k,S,H,I,Ts", CASES)
def test_forward_matches_oracle(fmt, mode, E, k, S, H, I, Ts, kernel):
    kw = dict(n_group=4, topk_group=2, routed_scaling=2.5) if mode == "sigmoid_group" else {}
    cfg = small_cfg(fmt, mode, hidden=H, inter=I, experts=E, top_k=k, shared=S, **kw)
    lw = inputs.make_layer(cfg, seed=E + k + S)
    L = gpu_layer(lw, kernel=kernel)
    for T in Ts:
        xb = lw.make_x(T)
        out, r = L.forward(x_device(xb), out_dtype=torch.float32, return_routing=True)
        ids, w = r.ids.cpu().numpy().astype(np.int64), r.weights.cpu().numpy()
        ref, ids_ref, _ = oracle_forward(lw, xb)
        assert ids_match_except_near_ties(ids, ids_ref, oracle_scores(lw, xb), k).size == 0
        ref_same, _, _ = oracle_forward(lw, xb, ids=ids, weights=w)
        err = rel_err_rows(out.cpu().numpy(), ref_same)
        assert err <= TOL, f"T={T}: max row rel err {err:.3e}"
        # bf16 output (the weighted rows pass through bf16 once before the fp32 sum)
        outb = L.forward(x_device(xb)).float().cpu().numpy()
        assert rel_err_rows(outb, ref_same) <= TOL
    assert L.workspace_status() == 0


@pytest.mark.parametrize("kernel", KERNELS)
def test_forward_matches_reference_moe_forward_as_is(golden_dir, kernel):
    """Against the reference's own moe_forward (FP8 per-row scales) on equivalent weights."""
    g = np.load(golden_dir / "moe_forward_fp8.npz")
    for norm in (False, True):
        cfg = small_cfg("fp8_b128", "topk_softmax" if norm else "softmax_topk", top_k=int(g["top_k"]))
        lw = inputs.make_layer(cfg, seed=int(g["seed"]))
        for ew in lw.experts:
            for m in (ew.gate, ew.up, ew.down):
                m.scale[:] = m.scale[0:1, :]
        L = gpu_layer(lw, kernel=kernel)
        for T in (1, 5, 17):
            xb = g[f"x_T{T}"]
            out = L.forward(x_device(xb), out_dtype=torch.float32).cpu().numpy()
            assert rel_err_rows(out, g[f"y_norm{int(norm)}_T{T}"]) <= TOL


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("fmt", FMTS)
def test_forward_matches_reference_combine(golden_dir, fmt, kernel):
    g = np.load(golden_dir / f"combine_{fmt}.npz")
    cfg = small_cfg(fmt, str(g["routing"]), top_k=int(g["top_k"]))
    lw = inputs.make_layer(cfg, seed=int(g["seed"]))
    L = gpu_layer(lw, kernel=kernel)
    for T in (1, 5, 17):
        out, r = L.forward(x_device(g[f"x_T{T}"]), out_dtype=torch.float32, return_routing=True)
        assert np.array_equal(r.ids.cpu().numpy().astype(np.int64), g[f"ids_T{T}"])
        assert rel_err_rows(out.cpu().numpy(), g[f"y_T{T}"]) <= TOL


@pytest.mark.parametrize("kernel", KERNELS)
def test_stages_compose_to_forward(kernel):
    cfg = small_cfg("awq_int4_g128", "softmax_topk", experts=8, top_k=2, shared=1)
    lw = inputs.make_layer(cfg, seed=8)
    L = gpu_layer(lw, kernel=kernel)
    x = x_device(lw.make_x(37))
    r = L.route(x)
    p = L.permute(r)
    y = L.expert_ffn(x, p)
    out = L.combine(y, p, 37, out_dtype=torch.float32)
    full = L.forward(x, out_dtype=torch.float32)
    assert torch.equal(out, full)


@pytest.mark.parametrize("fmt", FMTS)
def test_dynamic_schedule_matches_static(fmt):
    """The decode GEMM hands out work items from a counter in the workspace (dynamic
    schedule) or by CTA index (static, chosen by a workspace too small for the counters);
    both compute every item whole, so the down projection is bit-identical either way, and
    every call leaves the counters at zero for the next one.  The whole layer stays within
    tolerance of the oracle."""
    import ctypes as C

    from ccut_b200 import _lib
    from ccut_b200.layer import _ptr, _stream

    cfg = small_cfg(fmt, "softmax_topk", hidden=1024, inter=512, experts=16, top_k=4, shared=1)
    lw = inputs.make_layer(cfg, seed=21)
    L = gpu_layer(lw, kernel="mma")
    for T in (1, 7, 64):
        xb = lw.make_x(T)
        x = x_device(xb)
        p = L.permute(L.route(x))
        h = L.gate_up(x, p)
        assert torch.equal(L.gate_up(x, p), h)
        y_dyn = L.down(h, p, T)
        ws_dyn = L._ws["down"]
        assert int(ws_dyn[256:512].count_nonzero()) == 0  # counters back at zero
        y_st = torch.empty_like(y_dyn)
        ws = torch.zeros(256, dtype=torch.uint8, device="cuda")
        _lib.call("ccut_moe_down", C.byref(L.desc), _ptr(h), T, L.top_k, _ptr(p.offsets), _ptr(p.row_weight),
                  _ptr(y_st), _ptr(ws), ws.numel(), _stream())
        R = T * L.top_k + T
        assert torch.equal(y_dyn[:R], y_st[:R])
        out, r = L.forward(x, out_dtype=torch.float32, return_routing=True)
        ref, _, _ = oracle_forward(lw, xb, ids=r.ids.cpu().numpy().astype(np.int64), weights=r.weights.cpu().numpy())
        assert rel_err_rows(out.cpu().numpy(), ref) <= TOL
    assert L.workspace_status() == 0


# ---------------------------------------------------------------- edge cases
def test_empty_batch():
    lw = inputs.make_layer(small_cfg("fp8_b128"), seed=9)
    L = gpu_layer(lw)
    out = L.forward(torch.empty((0, 256), dtype=torch.bfloat16, device="cuda"))
    assert out.shape == (0, 256)


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("fmt", FMTS)
def test_all_tokens_on_one_expert_and_empty_experts(fmt, kernel):
    cfg = small_cfg(fmt, "topk_softmax", experts=8, top_k=1, shared=1)
    lw = inputs.make_layer(cfg, seed=10)
    lw.router[:] = 0.0
    lw.router[5, :] = 0.05  # every token routes to expert 5 (x>0 dominated rows aside)
    L = gpu_layer(lw, kernel=kernel)
    xb = formats.bf16_bits_from_f32(np.abs(formats.bf16_bits_to_f32(lw.make_x(150))) + 0.1)
    out, r = L.forward(x_device(xb), out_dtype=torch.float32, return_routing=True)
    ids = r.ids.cpu().numpy().astype(np.int64)
    assert (ids == 5).all()
    ref, _, _ = oracle_forward(lw, xb, ids=ids, weights=r.weights.cpu().numpy())
    assert rel_err_rows(out.cpu().numpy(), ref) <= TOL


@pytest.mark.parametrize("layout", [0, 1])
def test_quant_linear_matches_reference_weight_only(golden_dir, layout):
    """QuantizeMethodBase.apply parity: AWQ (z = 8) linear vs the reference's signed int4 W4A16."""
    import ctypes as C
    from ccut_b200 import _lib
    g = np.load(golden_dir / "int4_linear.npz")
    K, N = g["qweight"].shape[0], g["scales"].shape[1]
    # N = 24 is not a tile multiple: pad the output channels to 128 with zero scales
    Np = 128
    q = np.zeros((K, Np), dtype=np.uint8)
    q[:, :N] = formats.awq_unpack(g["qweight"])
    z = np.full((K // 128, Np), 8, dtype=np.uint8)
    s = np.zeros((K // 128, Np), dtype=np.float16)
    s[:, :N] = g["scales"]
    lib = _lib.load()
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    qd = torch.from_numpy(formats.awq_pack(q)).cuda()
    zd = torch.from_numpy(formats.awq_pack(z)).cuda()
    sd = torch.from_numpy(s).cuda()
    packed = torch.empty(lib.ccut_packed_matrix_bytes(1, K, Np), dtype=torch.uint8, device="cuda")
    _lib.call("ccut_pack_matrix", 1, layout, C.c_void_p(qd.data_ptr()), C.c_void_p(zd.data_ptr()),
              C.c_void_p(sd.data_ptr()), K, Np, 0, C.c_void_p(packed.data_ptr()), 1, 0, st)
    x = torch.from_numpy(g["x"]).cuda().to(torch.bfloat16)
    M = x.shape[0]
    y = torch.empty((M, Np), dtype=torch.float32, device="cuda")
    ws = torch.empty(lib.ccut_quant_linear_workspace_bytes(1, M, K), dtype=torch.uint8, device="cuda")
    _lib.call("ccut_quant_linear", 1, layout, C.c_void_p(packed.data_ptr()), K, Np, C.c_void_p(x.data_ptr()), M,
              C.c_void_p(y.data_ptr()), C.c_void_p(ws.data_ptr()), ws.numel(), st)
    ref = formats.bf16_bits_to_f32(formats.bf16_bits_from_f32(g["x"])) @ formats.awq_dequant(
        g["qweight"], g["qzeros"], g["scales"])
    got = y.cpu().numpy()[:, :N]
    # fragment kernel: exact operands, only the fp32 summation order differs; row (tcgen05)
    # kernel: the dequantized weight operand is rounded to f16 (<= 2^-11 relative)
    assert rel_err_rows(got, ref) <= (1e-4 if layout == 1 else 2e-3)
    assert rel_err_rows(got, g["y"]) <= TOL  # the reference's fp32 x (ours is bf16-rounded)


def test_argument_validation():
    lw = inputs.make_layer(small_cfg("fp8_b128"), seed=12)
    L = gpu_layer(lw)
    with pytest.raises(ValueError):
        L.forward(torch.zeros((4, 128), dtype=torch.bfloat16, device="cuda"))
    with pytest.raises(ValueError):
        L.forward(torch.zeros((4, 256), dtype=torch.float16, device="cuda"))
    with pytest.raises(NotImplementedError):
        gpu_layer(lw).__class__("int3", 256, 128, 8, 2, "softmax_topk", lw.router, lw.experts)
