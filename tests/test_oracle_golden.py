"""Pin the CPU oracle to fixtures produced by running the reference itself.

The fixtures (``tests/golden/*.npz``) were written by ``tests/golden/make_golden.py``,
which imports the reference's own ``ccut`` modules.  Tolerances: bit-exact for decode
tables, dequantized weights and routing ids; fp32 matmul-order tolerance elsewhere.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import formats, inputs, moe, routing


def _load(golden_dir, name):
    return np.load(golden_dir / name, allow_pickle=False)


def test_e4m3_table_bit_exact(golden_dir):
    g = _load(golden_dir, "e4m3_table.npz")
    ours = formats.fp8_e4m3_decode(g["codes"])
    ref = g["values"]
    nan = np.isnan(ref)
    assert np.array_equal(nan, np.isnan(ours))
    assert nan.sum() == 2 and nan[0x7F] and nan[0xFF]
    assert np.array_equal(ours[~nan].view(np.uint32), ref[~nan].view(np.uint32))


def test_fp8_rowscale_dequant_bit_exact(golden_dir):
    g = _load(golden_dir, "fp8_rowscale.npz")
    ours = formats.fp8_e4m3_decode(g["w"]) * g["scale"][:, None]
    assert np.array_equal(ours.astype(np.float32).view(np.uint32), g["out"].view(np.uint32))


def test_fp8_block_dequant_equals_rowscale_when_block_scale_is_uniform(golden_dir):
    g = _load(golden_dir, "fp8_rowscale.npz")
    w = g["w"]  # [16, 40]
    s = np.float32(0.0173)
    blk = formats.fp8_block_dequant(w, np.full((1, 1), s, dtype=np.float32))
    row = formats.fp8_e4m3_decode(w) * s
    assert np.array_equal(blk.view(np.uint32), row.astype(np.float32).view(np.uint32))


def test_awq_dequant_matches_reference_int4(golden_dir):
    g = _load(golden_dir, "int4_linear.npz")
    w = formats.awq_dequant(g["qweight"], g["qzeros"], g["scales"])  # [K, N]
    ref = g["dequant_out_in"]  # [N, K]
    assert np.array_equal(w.T.astype(np.float32).view(np.uint32), ref.view(np.uint32))
    y = g["x"] @ w
    np.testing.assert_allclose(y, g["y"], rtol=1e-5, atol=1e-6)


def test_awq_pack_roundtrip_and_orders():
    rng = np.random.default_rng(3)
    v = rng.integers(0, 16, size=(5, 32), dtype=np.uint8)
    for order in ("awq", "sequential"):
        assert np.array_equal(formats.awq_unpack(formats.awq_pack(v, order), order), v)
    # AWQ interleave: slot 1 of the first word holds column 2
    word = formats.awq_pack(v, "awq").view(np.uint32)[0, 0]
    assert (word >> 4) & 0xF == v[0, 2]
    with pytest.raises(ValueError):
        formats.awq_pack(np.full((1, 8), 16, dtype=np.uint8))


def test_fp8_encode_matches_torch_and_roundtrips():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(4)
    x = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * 40,
        formats.FP8_E4M3_TABLE[np.isfinite(formats.FP8_E4M3_TABLE)],
        np.array([448.0, -448.0, 0.0, -0.0, 1e-9, -2.0 ** -10], dtype=np.float32),
    ]).astype(np.float32)
    x = np.clip(x, -448, 448)
    ours = formats.fp8_e4m3_encode(x)
    theirs = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(ours, theirs)


@pytest.mark.parametrize("k", [1, 2, 6, 8])
def test_topk_softmax_ids_bit_exact_and_weights(golden_dir, k):
    g = _load(golden_dir, "topk.npz")
    lg = g["logits"]
    w, ids = routing.topk_softmax(lg, k, norm_topk_prob=False)
    assert np.array_equal(ids, g[f"ids_soft_k{k}"])
    np.testing.assert_allclose(w, g[f"w_soft_k{k}"], rtol=2e-6, atol=1e-7)
    w, ids = routing.topk_softmax(lg, k, norm_topk_prob=True)
    assert np.array_equal(ids, g[f"ids_norm_k{k}"])
    np.testing.assert_allclose(w, g[f"w_norm_k{k}"], rtol=2e-6, atol=1e-7)


def test_silu_mul_and_expert_ffn(golden_dir):
    g = _load(golden_dir, "silu_ffn.npz")
    np.testing.assert_allclose(moe.silu_mul(g["gate"], g["up"]), g["silu_mul"], rtol=1e-6, atol=1e-7)
    y = moe.expert_ffn(g["x"], g["wg"], g["wu"], g["wd"])
    np.testing.assert_allclose(y, g["y"], rtol=1e-5, atol=1e-6)


def _small(fmt, routing_mode, k, shared=0):
    return inputs.MoeLayerConfig(
        f"small_{fmt}", hidden=256, inter=128, num_experts=8, top_k=k,
        num_shared=shared, shared_inter=128, fmt=fmt, routing=routing_mode,
    )


@pytest.mark.parametrize("fmt", ["awq_int4_g128", "fp8_b128"])
def test_moe_combine_matches_reference(golden_dir, fmt):
    g = _load(golden_dir, f"combine_{fmt}.npz")
    k = int(g["top_k"])
    mode = str(g["routing"])
    layer = inputs.make_layer(_small(fmt, mode, k), seed=int(g["seed"]))
    for T in (1, 5, 17):
        xb = layer.make_x(T)
        assert np.array_equal(xb, g[f"x_T{T}"]), "seeded generator drifted"
        xf = formats.bf16_bits_to_f32(xb)
        out, ids, w = moe.moe_forward(xf, layer.router, k, mode, layer.w_lookup)
        assert np.array_equal(ids, g[f"ids_T{T}"])
        np.testing.assert_allclose(w, g[f"w_T{T}"], rtol=2e-6, atol=1e-7)
        ref = g[f"y_T{T}"]
        err = np.abs(out - ref).max(axis=1) / np.maximum(np.abs(ref).max(axis=1), 1e-30)
        assert err.max() < 1e-5


@pytest.mark.parametrize("norm", [False, True])
def test_moe_forward_matches_reference_as_is(golden_dir, norm):
    """The reference's own ``moe_forward`` (FP8 per-row) equals the oracle on FP8-block
    weights whose scales are constant along N."""
    g = _load(golden_dir, "moe_forward_fp8.npz")
    cfg = _small("fp8_b128", "topk_softmax" if norm else "softmax_topk", int(g["top_k"]))
    layer = inputs.make_layer(cfg, seed=int(g["seed"]))
    for ew in layer.experts:
        for mat in (ew.gate, ew.up, ew.down):
            mat.scale[:] = mat.scale[0:1, :]
    for T in (1, 5, 17):
        xb = layer.make_x(T)
        assert np.array_equal(xb, g[f"x_T{T}"])
        xf = formats.bf16_bits_to_f32(xb)
        out, _, _ = moe.moe_forward(xf, layer.router, cfg.top_k, cfg.routing, layer.w_lookup)
        ref = g[f"y_norm{int(norm)}_T{T}"]
        err = np.abs(out - ref).max(axis=1) / np.maximum(np.abs(ref).max(axis=1), 1e-30)
        assert err.max() < 1e-5


def test_grouped_sigmoid_properties():
    rng = np.random.default_rng(9)
    lg = rng.standard_normal((33, 64)).astype(np.float32)
    w, ids = routing.grouped_sigmoid_topk(lg, 8, n_group=8, topk_group=4, routed_scaling=2.5)
    assert ids.shape == (33, 8)
    np.testing.assert_allclose(w.sum(axis=1), 2.5, rtol=1e-5)
    for t in range(33):
        assert len(set(ids[t].tolist())) == 8
        assert len({int(e) // 8 for e in ids[t]}) <= 4
    # brute force: ids are the 8 best sigmoid scores among the 4 groups with best top-2 sums
    s = 1 / (1 + np.exp(-lg.astype(np.float64)))
    for t in range(33):
        gs = [np.sort(s[t, g * 8:(g + 1) * 8])[-2:].sum() for g in range(8)]
        keep = sorted(range(8), key=lambda g: (-gs[g], g))[:4]
        cand = [e for e in range(64) if e // 8 in keep]
        best = sorted(cand, key=lambda e: (-s[t, e], e))[:8]
        assert ids[t].tolist() == best


def test_layer_generator_is_deterministic_and_sized():
    cfg = _small("awq_int4_g128", "softmax_topk", 2, shared=1)
    a, b = inputs.make_layer(cfg, seed=5), inputs.make_layer(cfg, seed=5)
    assert np.array_equal(a.experts[3].down.qweight, b.experts[3].down.qweight)
    assert np.array_equal(a.make_x(4), b.make_x(4))
    assert a.experts[0].gate.qweight.shape == (256, 16)
    assert a.experts[0].down.scales.shape == (1, 256)
    assert inputs.CONFIGS["cfg0"].expert_bytes() == 4_494_336
    assert inputs.CONFIGS["cfg1"].expert_bytes() == 8_652_864
    assert inputs.CONFIGS["cfg3"].expert_bytes() == 2_451_456
    assert inputs.CONFIGS["cfg4"].expert_bytes() == 44_050_944


# ---------------------------------------------------------------- attention / RMSNorm
def test_gqa_attention_oracle_matches_reference(golden_dir):
    """oracle.attention.gqa_attention against the reference's gqa_attention_fast
    (ccut/blocks/attn_gqa.py:127-153) on causal, unmasked and grouped cases."""
    from oracle import attention

    g = np.load(golden_dir / "attn_norm.npz")
    i = 0
    while f"gqa{i}_q" in g:
        q, k, v = (formats.bf16_bits_to_f32(g[f"gqa{i}_{n}"]) for n in "qkv")
        start = int(g[f"gqa{i}_start"])
        s, kv = q.shape[2], k.shape[2]
        mask = attention.causal_mask(s, start)[None, None] if start >= 0 else None
        got = attention.gqa_attention(q, k, v, mask)
        np.testing.assert_allclose(got, g[f"gqa{i}_out"], rtol=1e-5, atol=1e-5)
        i += 1
    assert i == 4


def test_rms_norm_oracle_matches_reference(golden_dir):
    from oracle import attention

    g = np.load(golden_dir / "attn_norm.npz")
    for i in range(2):
        x = formats.bf16_bits_to_f32(g[f"rms{i}_x"])
        w = g[f"rms{i}_w"]
        y = attention.rms_norm(x, w if w.size else None, float(g[f"rms{i}_eps"]))
        np.testing.assert_allclose(y, g[f"rms{i}_y"], rtol=1e-6, atol=1e-6)


def test_rope_oracle_matches_reference(golden_dir):
    """oracle.attention.apply_rope against the reference's apply_rope (ccut/blocks/rope.py:130-175)."""
    from oracle import attention

    g = np.load(golden_dir / "attn_norm.npz")
    for i in range(2):
        q, k = (formats.bf16_bits_to_f32(g[f"rope{i}_{n}"]) for n in "qk")
        qo, ko = attention.apply_rope(q, k, g[f"rope{i}_inv_freq"], g[f"rope{i}_pos"], float(g[f"rope{i}_attn"]),
                                      str(g[f"rope{i}_type"]))
        np.testing.assert_allclose(qo, g[f"rope{i}_q_out"], rtol=1e-6, atol=1e-6)
        np.testing.assert_allclose(ko, g[f"rope{i}_k_out"], rtol=1e-6, atol=1e-6)


def test_mla_oracle_matches_reference(golden_dir):
    """oracle.attention.mla_attention (and its latent-space form) against the reference's
    mla_decode / mla_prefill (ccut/blocks/attn_mla.py:85-167)."""
    from oracle import attention

    g = np.load(golden_dir / "attn_norm.npz")
    for i in range(2):
        args = [g[f"mla{i}_{n}"] for n in ("c", "kpe", "qn", "qp", "ku", "vu")]
        scale, start = float(g[f"mla{i}_scale"]), int(g[f"mla{i}_start"])
        ref = g[f"mla{i}_out"]
        np.testing.assert_allclose(attention.mla_attention(*args, scale, start), ref, rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(attention.mla_attention_absorbed(*args, scale, start), ref, rtol=1e-4, atol=1e-5)


def test_mla_latent_form_at_deepseek_sizes():
    """The latent-space regrouping the MLA kernel computes equals the reference's expanded form
    at the DeepSeek-V2-Lite sizes (rank 512, rope 64, nope 128, v 128, 16 heads): decode over a
    long cache and a causal prefill after a prefix."""
    from oracle import attention

    rng = np.random.default_rng(9)
    for prefix, seq in ((200, 1), (30, 12)):
        kv = prefix + seq
        c = rng.standard_normal((kv, 512)).astype(np.float32)
        kpe = rng.standard_normal((kv, 64)).astype(np.float32)
        qn = rng.standard_normal((seq, 16, 128)).astype(np.float32)
        qp = rng.standard_normal((seq, 16, 64)).astype(np.float32)
        ku = (rng.standard_normal((512, 16 * 128)) * 0.05).astype(np.float32)
        vu = (rng.standard_normal((512, 16 * 128)) * 0.05).astype(np.float32)
        scale = 1.0 / np.sqrt(192.0)
        ref = attention.mla_attention(c, kpe, qn, qp, ku, vu, scale, prefix)
        got = attention.mla_attention_absorbed(c, kpe, qn, qp, ku, vu, scale, prefix)
        np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-5 * np.abs(ref).max())


def test_topk_softmax_wide_routers_match_reference(golden_dir):
    """The oracle's topk_softmax against the reference's at 128 experts top-8 (normalised)
    and 256 experts top-16 (both modes), with exact ties: ids bit-exact, weights to fp32."""
    g = np.load(golden_dir / "routing_wide.npz")
    for i in range(3):
        k, norm = int(g[f"c{i}_k"]), bool(g[f"c{i}_norm"])
        w, ids = routing.topk_softmax(g[f"c{i}_logits"], k, norm_topk_prob=norm)
        assert np.array_equal(ids, g[f"c{i}_ids"]), i
        np.testing.assert_allclose(w, g[f"c{i}_w"], rtol=1e-6, atol=1e-7)
