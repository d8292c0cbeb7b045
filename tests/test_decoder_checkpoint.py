"""Whole-decoder checkpoints on the CPU (``ccut_b200.checkpoint.decoder_spec_from_config``,
``load_decoder_weights``): which layers are MoE, the tensor names and shapes, tied
embeddings, quantized and BF16 attention projections, and the errors."""

from __future__ import annotations

import json

import numpy as np
import pytest

from ccut_b200 import checkpoint as ck
from oracle import inputs
from tests.ckpt_helpers import write_decoder_checkpoint
from tests.model_helpers import make_tiny, quantized_attention, quantized_layers

_FP8 = {"quant_method": "fp8", "weight_block_size": [128, 128]}


def _cfg(**kw):
    base = {"hidden_size": 256, "num_hidden_layers": 6, "num_attention_heads": 4, "vocab_size": 32,
            "num_experts": 8, "quantization_config": _FP8}
    return base | kw


def test_moe_layer_selection_and_spec():
    assert ck.decoder_spec_from_config(_cfg()).moe_layers == (True,) * 6
    assert ck.decoder_spec_from_config(_cfg(mlp_only_layers=[0, 3])).moe_layers == (False, True, True, False, True,
                                                                                     True)
    assert ck.decoder_spec_from_config(_cfg(decoder_sparse_step=2)).moe_layers == (False, True) * 3
    assert ck.decoder_spec_from_config(_cfg(first_k_dense_replace=2, num_experts=None, n_routed_experts=8)
                                       ).moe_layers == (False, False, True, True, True, True)
    assert ck.decoder_spec_from_config(_cfg(num_experts=0)).moe_layers == (False,) * 6
    s = ck.decoder_spec_from_config(_cfg(num_key_value_heads=2, head_dim=128, rms_norm_eps=1e-5,
                                         attn_logit_softcapping=30.0, tie_word_embeddings=True))
    assert (s.kv_heads, s.head_dim, s.eps, s.softcap, s.tie_word_embeddings, s.fmt) == (2, 128, 1e-5, 30.0, True,
                                                                                         "fp8_b128")
    assert ck.decoder_spec_from_config(_cfg()).head_dim == 64
    with pytest.raises(KeyError):
        ck.decoder_spec_from_config(_cfg(kv_lora_rank=512))  # MLA without its head sizes
    m = ck.decoder_spec_from_config(_cfg(kv_lora_rank=512, qk_nope_head_dim=128, qk_rope_head_dim=64, v_head_dim=128))
    assert m.mla["kv_lora_rank"] == 512 and m.head_dim == 64 and m.mla["softmax_scale"] == pytest.approx(192 ** -0.5)
    with pytest.raises(NotImplementedError):
        ck.decoder_spec_from_config(_cfg(linear_num_key_heads=16))
    with pytest.raises(KeyError):
        ck.decoder_spec_from_config({k: v for k, v in _cfg().items() if k != "vocab_size"})
    with pytest.raises(NotImplementedError):
        ck.decoder_spec_from_config(_cfg(quantization_config=None))


@pytest.mark.parametrize("fmt, quant_attn", [("fp8_b128", True), ("awq_int4_g128", False)])
def test_load_decoder_weights(tmp_path, fmt, quant_attn):
    t = make_tiny(41, kv_heads=2, qk_norm="head", layers=3)
    q = quantized_layers(t, fmt, seed=41)
    mats, attn = quantized_attention(t, fmt, seed=42) if quant_attn else (None, t.attn)
    dl = inputs.make_layer(inputs.scaled_config("cfg1" if fmt == "fp8_b128" else "cfg0", hidden=t.hidden, inter=256,
                                                num_experts=1, top_k=1, num_shared=0), seed=43)
    root = write_decoder_checkpoint(tmp_path / "m", t, fmt, q, mats, dense={1: dl.experts[0]}, dense_inter=256)
    w = ck.load_decoder_weights(root)
    s = w["spec"]
    assert s.moe_layers == (True, False, True) and s.inter == 256 and s.fmt == fmt
    assert np.array_equal(w["embed"], t.embed) and np.array_equal(w["lm_head"], t.lm_head)
    assert np.array_equal(w["final_norm"], t.final_norm)
    for i, lay in enumerate(w["layers"]):
        assert np.array_equal(lay["ln1"], t.attn[i].ln1) and np.array_equal(lay["q_norm"], t.attn[i].q_norm)
        for p in "qkvo":
            kind, m = lay[p]
            assert kind == ("quant" if quant_attn else "dense")
            if not quant_attn:
                assert np.array_equal(m, getattr(t.attn[i], "w" + p))
        kind, f = lay["ffn"]
        assert kind == ("dense" if i == 1 else "moe")
        if kind == "moe":
            spec, router, experts, shared, bias = f
            assert np.array_equal(router, q[i].router) and len(experts) == 8 and len(shared) == 1 and bias is None
    # tied embeddings, a missing norm, a projection of the wrong shape
    root2 = write_decoder_checkpoint(tmp_path / "tied", t, fmt, q, mats, dense={1: dl.experts[0]}, dense_inter=256,
                                     tie=True)
    w2 = ck.load_decoder_weights(root2)
    assert w2["lm_head"] is w2["embed"]
    root3 = write_decoder_checkpoint(tmp_path / "nonorm", t, fmt, q, mats, dense={1: dl.experts[0]}, dense_inter=256,
                                     drop=("model.layers.2.post_attention_layernorm.weight",))
    with pytest.raises(KeyError):
        ck.load_decoder_weights(root3)
    cfg = json.loads((root / "config.json").read_text())
    (root / "config.json").write_text(json.dumps(cfg | {"num_key_value_heads": 4}))
    with pytest.raises(ValueError):
        ck.load_decoder_weights(root)
    (root / "config.json").write_text(json.dumps(cfg | {"intermediate_size": 0}))
    with pytest.raises(ValueError):
        ck.load_decoder_weights(root)


@pytest.mark.parametrize("fmt", ["awq_int4_g128", "fp8_b128"])
def test_cat_checkpoint_tensors(fmt):
    """Fusing the q / k / v projections: the concatenated checkpoint tensors dequantize to the
    three matrices side by side (the oracle's dequant)."""
    from ccut_b200.quant import cat_checkpoint_tensors
    from ccut_b200.synthetic import _gen_matrix

    rng = np.random.default_rng(3)
    mats = [_gen_matrix(rng, fmt, 256, n) for n in (256, 128, 128)]  # [in, out] shapes 256 -> n
    if fmt == "awq_int4_g128":
        dicts = [{"qweight": m.qweight, "qzeros": m.qzeros, "scales": m.scales} for m in mats]
        t = cat_checkpoint_tensors(fmt, dicts)
        fused = inputs.AwqMatrix(t["qweight"], t["qzeros"], t["scales"])
    else:
        dicts = [{"weight": m.weight, "weight_scale_inv": m.scale} for m in mats]
        t = cat_checkpoint_tensors(fmt, dicts)
        fused = inputs.Fp8Matrix(t["weight"], t["weight_scale_inv"])
    want = np.concatenate([inputs.dequant(m) for m in mats], axis=1)  # [in, sum(out)]
    assert np.array_equal(inputs.dequant(fused), want)
    with pytest.raises(NotImplementedError):
        cat_checkpoint_tensors("int8", dicts)


def test_load_decoder_checks_engine_config_first(tmp_path):
    """The engine's [quant] / [experts] settings are checked before any weight is uploaded."""
    t = make_tiny(45, kv_heads=2, qk_norm=None, layers=1)
    q = quantized_layers(t, "fp8_b128", seed=45)
    root = write_decoder_checkpoint(tmp_path / "m", t, "fp8_b128", q)
    with pytest.raises(NotImplementedError):
        ck.load_decoder(root, app_config={"quant": {"quantization": "mxfp8"}})
    with pytest.raises(ValueError):
        ck.load_decoder(root, app_config={"experts": {"expert_ring_slots": 0}})
