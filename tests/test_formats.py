"""The reference's own weight formats on the host side: the oracle's per-channel FP8 and
signed int4 dequant against fixtures the reference generated, the checkpoint-form
conversions of ``ccut_b200.formats`` (bit-exact against the oracle), ``QuantKey`` dispatch,
and the compressed-tensors symmetric int4 repack."""

from __future__ import annotations

import numpy as np
import pytest

from ccut_b200 import formats as F
from ccut_b200 import quant, quant_spec
from oracle import formats, moe
from tests.golden.make_golden_channel import FIXTURE_CFG, fixture_layer


def _load(golden_dir, name):
    return np.load(golden_dir / name)


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def test_oracle_fp8_channel_matches_reference(golden_dir):
    g = _load(golden_dir, "fp8_channel_linear.npz")
    d = formats.fp8_channel_dequant(g["w"], g["scale"])
    assert np.array_equal(_bits(d), _bits(g["dequant_out_in"]))
    for key in ("fp8_static_channel_sym", "fp8_dynamic_token_sym"):  # the reference's w8a8 label = w8a16
        np.testing.assert_allclose(g["x"] @ d.T, g[f"y_{key}"], rtol=1e-5, atol=1e-6)


def test_oracle_int4_sym_matches_reference(golden_dir):
    g = _load(golden_dir, "int4_sym_linear.npz")
    d = formats.int4_sym_dequant(g["packed"], g["scale"])
    assert np.array_equal(_bits(d), _bits(g["dequant_out_in"]))
    np.testing.assert_allclose(g["x"] @ d.T, g["y"], rtol=1e-5, atol=1e-6)
    assert not np.array_equal(g["scale"].astype(np.float16).astype(np.float32), g["scale"])  # fp32-only scales


def _canon_dequant(fmt, t):
    """fp32 [N, K] of a canonical matrix, as the kernels' exact codes times the fp32 scale."""
    if fmt == "int4_sym_g128":
        q = formats.awq_unpack(np.asarray(t["qweight"])).astype(np.float32) - 8.0
        return (q * np.repeat(np.asarray(t["scales"], np.float32), 128, axis=0)).astype(np.float32).T
    v = formats.fp8_e4m3_decode(np.asarray(t["weight"]))
    return (v * np.repeat(np.asarray(t["scales"], np.float32), 128, axis=0).T).astype(np.float32)


def test_int4_sym_reference_form_converts_exactly(golden_dir):
    g = _load(golden_dir, "int4_sym_linear.npz")
    t = F.canonical("int4_sym_g128", {"weight": g["packed"], "weight_scale": g["scale"]})
    assert t["qweight"].dtype == np.int32 and t["scales"].dtype == np.float32
    assert np.array_equal(_bits(_canon_dequant("int4_sym_g128", t)), _bits(g["dequant_out_in"]))
    assert F.repacked("int4_sym_g128", {"weight": g["packed"]})


def test_int4_sym_rejects_scales_varying_inside_a_group():
    packed = np.zeros((128, 128), np.uint8)
    s = np.full(256, 0.01, np.float32)
    s[5] = 0.02
    with pytest.raises(ValueError):
        F.int4_sym_from_reference(packed, s)
    with pytest.raises(ValueError):
        F.int4_sym_from_reference(packed, np.full(200, 0.01, np.float32))


@pytest.mark.parametrize("form", ["vector", "column", "scalar", "grouped"])
def test_fp8_channel_scale_forms(golden_dir, form):
    g = _load(golden_dir, "fp8_channel_linear.npz")
    w, s = g["w"], g["scale"]
    N, K = w.shape
    if form == "scalar":
        s = s[:1]
    ref = formats.fp8_channel_dequant(w, np.broadcast_to(s, (N,)) if s.size == 1 else s)
    mat = {"vector": {"weight": w, "scale": s}, "column": {"weight": w, "weight_scale": s.reshape(-1, 1)},
           "scalar": {"weight": w, "scale": np.float32(s[0])},
           "grouped": {"weight": w, "scales": np.repeat(s[None, :], K // 128, axis=0)}}[form]
    t = F.canonical("fp8_channel", mat)
    assert t["scales"].shape == (K // 128, N)
    assert np.array_equal(_bits(_canon_dequant("fp8_channel", t)), _bits(ref))


def test_slices_cut_the_right_channels():
    rng = np.random.default_rng(1)
    w = rng.integers(0, 256, (256, 384), dtype=np.uint8)
    w[(w & 0x7F) == 0x7F] = 0  # no NaN codes: the comparison is of values
    s = rng.random(256).astype(np.float32)
    t = F.canonical("fp8_channel", {"weight": w, "scale": s})
    full = _canon_dequant("fp8_channel", t)
    assert np.array_equal(_canon_dequant("fp8_channel", F.slice_out("fp8_channel", t, 128, 128)), full[128:256])
    assert np.array_equal(_canon_dequant("fp8_channel", F.slice_in("fp8_channel", t, 128, 256)), full[:, 128:384])
    p = rng.integers(0, 256, (256, 192), dtype=np.uint8)
    ti = F.canonical("int4_sym_g128", {"weight": p, "scale": np.repeat(rng.random(3).astype(np.float32), 128)})
    full = _canon_dequant("int4_sym_g128", ti)
    assert np.array_equal(_canon_dequant("int4_sym_g128", F.slice_out("int4_sym_g128", ti, 128, 128)), full[128:])
    assert np.array_equal(_canon_dequant("int4_sym_g128", F.slice_in("int4_sym_g128", ti, 128, 256)), full[:, 128:])


def test_moe_forward_fp8ch_fixture_matches_oracle(golden_dir):
    """The reference moe_forward (routed experts with per-input scales, shared expert with
    per-output scales) equals the oracle's layer on the same fp32 matrices."""
    g = _load(golden_dir, "moe_forward_fp8ch.npz")
    router, routed, shared, xs = fixture_layer()
    c = FIXTURE_CFG

    def deq_routed(cw, s_in):  # [in, out]: per-row scale of the reference's [in, out] storage
        return (formats.fp8_e4m3_decode(cw).T * s_in[:, None]).astype(np.float32)

    mats = [tuple(deq_routed(*proj[n]) for n in ("gate", "up", "down")) for proj in routed]
    sh = tuple(formats.fp8_channel_dequant(*shared[n]).T for n in ("gate", "up", "down"))
    for norm in (False, True):
        for T, xb in xs.items():
            y, _, _ = moe.moe_forward(formats.bf16_bits_to_f32(xb), router, c["top_k"],
                                      "topk_softmax" if norm else "softmax_topk", lambda e: mats[e], shared=sh)
            np.testing.assert_allclose(y, g[f"y_norm{int(norm)}_T{T}"], rtol=2e-5, atol=2e-6)


def test_quant_key_dispatch():
    want = {"fp8_static_channel_sym": "fp8_channel", "fp8_dynamic_token_sym": "fp8_channel",
            "fp8_static_tensor_sym": "fp8_channel", "int4_w4a16_sym": "int4_sym_g128",
            "awq_int4_g128": "awq_int4_g128", "fp8_block128": "fp8_b128"}
    for name in quant_spec.registered_keys():
        key = quant_spec.get_quant_key(name)
        if name in want:
            assert quant.format_for_key(key) == want[name], name
        elif key.is_quantized():
            with pytest.raises(NotImplementedError):
                quant.format_for_key(key)
    with pytest.raises(KeyError):
        quant_spec.get_quant_key("int3")
    assert quant_spec.get_quant_key("FP8_Block128").compute_path() == "w8a16"
    assert quant_spec.get_quant_key("awq_int4_g128").compute_path() == "w4a16"


def test_make_method_for_spec_picks_the_format_method():
    S = quant_spec
    cases = {"fp8_static_channel_sym": quant.Fp8ChannelMethod, "int4_w4a16_sym": quant.Int4SymMethod,
             "awq_int4_g128": quant.AwqInt4G128Method, "fp8_block128": quant.Fp8Block128Method}
    for name, cls in cases.items():
        spec = S.LayerQuantSpec(f"l.{name}", S.get_quant_key(name), scales=(S.ScaleDesc(f"l.{name}.s", "F32"),))
        m = quant.make_method_for_spec(spec, 256, 128, device="cpu")
        assert type(m) is cls and m.scale_name == f"l.{name}.s"
        m.create_weights(spec)
        with pytest.raises(ValueError):
            m.create_weights(S.LayerQuantSpec("l", S.get_quant_key(name)))  # no scale tensors
    assert isinstance(quant.make_method_for_spec(S.LayerQuantSpec("l", S.get_quant_key("bf16")), device="cpu"),
                      quant.UnquantizedMethod)
    skipped = S.LayerQuantSpec("l", S.get_quant_key("bf16"), skipped=True)  # an ignored layer
    assert isinstance(quant.make_method_for_spec(skipped, device="cpu"), quant.UnquantizedMethod)
    with pytest.raises(NotImplementedError):
        quant.make_method_for_spec(S.LayerQuantSpec("l", S.get_quant_key("nf4_w4a16"), scales=(S.ScaleDesc("s", "F32"),)))
    # a compressed-tensors spec: the activation key overrides the act side, the weight side picks
    act = S.QuantKey(S.QuantDType.FP32, S.ScaleStrategy.PER_TOKEN)
    spec = S.LayerQuantSpec("l", S.get_quant_key("fp8_static_channel_sym"), activation_key=act,
                            scales=(S.ScaleDesc("l.weight_scale", "F32"),))
    assert spec.effective_key().act_scale == "token" and spec.effective_key().is_w8a8()
    assert type(quant.make_method_for_spec(spec, device="cpu")) is quant.Fp8ChannelMethod


def test_ct_int4_symmetric_repack_keeps_fp32_scales(golden_dir):
    g = _load(golden_dir, "ct_int4.npz")
    t = quant.ct_int4_to_sym(g["sym_weight_packed"], g["sym_weight_scale"], g["sym_weight_shape"])
    assert t["scales"].dtype == np.float32
    np.testing.assert_array_equal(_canon_dequant("int4_sym_g128", t), g["sym_weight"].astype(np.float32))


def test_quant_linear_helpers_for_channel_formats():
    rng = np.random.default_rng(4)
    w = rng.integers(0, 256, (256, 128), dtype=np.uint8)
    s = rng.random(256).astype(np.float32)
    t = {"weight": w, "weight_scale": s}
    perm = rng.permutation(256)
    p = quant.permute_out_channels("fp8_channel", t, perm)
    assert np.array_equal(p["weight"], w[perm]) and np.array_equal(p["weight_scale"], s[perm])
    c = quant.cat_checkpoint_tensors("fp8_channel", [t, t])
    assert c["weight"].shape == (512, 128) and c["weight_scale"].shape == (512,)
    pd = quant.pad_out_channels("fp8_channel", {"weight": w[:200], "weight_scale": s[:200]}, 256)
    assert pd["weight"].shape == (256, 128) and pd["weight_scale"].shape == (256,)
    pk = rng.integers(0, 256, (128, 64), dtype=np.uint8)
    ti = {"weight": pk, "weight_scale": np.full(128, 0.5, np.float32)}
    assert quant.cat_checkpoint_tensors("int4_sym_g128", [ti, ti])["weight"].shape == (256, 64)
    with pytest.raises(ValueError):
        quant.cat_checkpoint_tensors("int4_sym_g128", [ti, {"weight": pk, "weight_scale": np.ones(128, np.float32)}])
    pi = quant.pad_out_channels("int4_sym_g128", {"weight": pk[:100], "weight_scale": ti["weight_scale"]}, 128)
    assert np.all(formats.int4_sym_dequant(pi["weight"], pi["weight_scale"])[100:] == 0)
