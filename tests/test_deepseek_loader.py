"""MLA checkpoints (DeepSeek-V2 / V3) on the CPU: config parsing, the YaRN table and softmax
scale, the rope-channel reordering of the quantized formats, and the oracle's decoder over
what ``load_decoder_weights`` reads, against ``transformers``' ``DeepseekV3ForCausalLM``
(``tests/golden/deepseek_tiny.npz``, made by ``tests/golden/make_golden_deepseek.py``)."""

from __future__ import annotations

import json

import numpy as np
import pytest

from ccut_b200.checkpoint import _rope_perm, decoder_spec_from_config, load_decoder_weights
from ccut_b200.quant import pad_out_channels, permute_out_channels
from ccut_b200.rope_tables import yarn_mscale, yarn_rope_table
from ccut_b200 import synthetic
from oracle import formats, inputs
from oracle import model as omodel
from tests.deepseek_helpers import DS_CASES, DS_SEEDS, deepseek_tiny, oracle_decoder, write_deepseek_checkpoint


@pytest.fixture(scope="module")
def golden(golden_dir):
    return np.load(golden_dir / "deepseek_tiny.npz")


def _rel(a, b) -> float:
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / np.abs(b).max())


@pytest.mark.parametrize("case", sorted(DS_CASES))
def test_rope_and_scale_match_transformers(golden, case):
    cfg, _, _ = deepseek_tiny(DS_SEEDS[case], **DS_CASES[case])
    spec = decoder_spec_from_config(cfg)
    assert spec.mla["rope_interleave"] and spec.head_dim == 64 and spec.rope_scaling["type"] == "yarn"
    inv, f = yarn_rope_table(spec.head_dim, spec.rope_theta, spec.rope_scaling)
    np.testing.assert_allclose(inv, golden[f"{case}_inv_freq"], rtol=1e-6)
    assert f == pytest.approx(float(golden[f"{case}_rope_factor"]), rel=1e-12)
    assert spec.mla["softmax_scale"] == pytest.approx(float(golden[f"{case}_softmax_scale"]), rel=1e-12)


@pytest.mark.parametrize("case", sorted(DS_CASES))
def test_oracle_over_loaded_weights_matches_transformers(tmp_path, golden, case):
    """The oracle's MLA decoder over the tensors ``load_decoder_weights`` reads (rope channels
    reordered from the interleaved layout, YaRN, the mscale softmax scale, grouped sigmoid
    routing with its bias, a dense first layer) against transformers' logits, for one causal
    pass and for a prefill followed by single-token steps and a chunk."""
    w = load_decoder_weights(write_deepseek_checkpoint(tmp_path / case, case))
    assert w["spec"].moe_layers == (False, True)
    layers, ffns, spec = oracle_decoder(w)
    toks, ref = golden[f"{case}_tokens"], golden[f"{case}_logits"]
    lg, _ = omodel.model_forward(toks, w["embed"], layers, ffns, w["final_norm"], w["lm_head"], spec,
                                 omodel.KvCache(), 0)
    assert _rel(lg, ref) < 1e-4
    cache, pos = omodel.KvCache(), 0
    for n in (5, 1, 1, 5):
        lg, _ = omodel.model_forward(toks[pos: pos + n], w["embed"], layers, ffns, w["final_norm"], w["lm_head"],
                                     spec, cache, pos)
        assert _rel(lg, ref[pos: pos + n]) < 1e-4, (case, pos)
        pos += n


def test_interleaved_rope_channels_matter(tmp_path, golden):
    """Reading the same checkpoint as if its rope channels were already in the half layout
    (``rope_interleave = false``) moves the logits away from transformers': the reordering is
    what the comparison above pins."""
    case = "fp8_bf16_attn"
    root = write_deepseek_checkpoint(tmp_path / case, case)
    cfg = json.loads((root / "config.json").read_text())
    cfg["rope_interleave"] = False
    (root / "config.json").write_text(json.dumps(cfg))
    w = load_decoder_weights(root)
    layers, ffns, spec = oracle_decoder(w)
    lg, _ = omodel.model_forward(golden[f"{case}_tokens"], w["embed"], layers, ffns, w["final_norm"], w["lm_head"],
                                 spec, omodel.KvCache(), 0)
    assert _rel(lg, golden[f"{case}_logits"]) > 1e-3


def _deq(fmt, t):
    if fmt == "awq_int4_g128":
        return formats.awq_dequant(t["qweight"], t["qzeros"], t["scales"]).T
    return formats.fp8_block_dequant(np.asarray(t["weight"]), np.asarray(t["weight_scale_inv"]))


def _tensors(fmt, m):
    if fmt == "awq_int4_g128":
        return {"qweight": m.qweight, "qzeros": m.qzeros, "scales": m.scales}
    return {"weight": m.weight, "weight_scale_inv": m.scale}


@pytest.mark.parametrize("fmt", ["awq_int4_g128", "fp8_b128"])
def test_permute_and_pad_output_channels(fmt):
    """The byte moves of ``permute_out_channels`` / ``pad_out_channels`` dequantize (oracle) to
    the permuted / zero-padded matrix exactly."""
    rng = np.random.default_rng(5)
    m = synthetic._gen_matrix(rng, fmt, 256, 576)  # kv_a_proj_with_mqa's 512 + 64 outputs
    t = _tensors(fmt, m)
    ref = np.ascontiguousarray(inputs.dequant(m).T)  # [576, 256]
    perm = _rope_perm(576, [512], 64)
    assert sorted(perm.tolist()) == list(range(576)) and perm[512:516].tolist() == [512, 514, 516, 518]
    got = _deq(fmt, permute_out_channels(fmt, t, perm))
    assert np.array_equal(got, ref[perm])
    padded = _deq(fmt, pad_out_channels(fmt, t, 640))
    assert padded.shape == (640, 256) and np.array_equal(padded[:576], ref) and not padded[576:].any()
    if fmt == "awq_int4_g128":
        perm2 = rng.permutation(576)  # AWQ moves any permutation
        assert np.array_equal(_deq(fmt, permute_out_channels(fmt, t, perm2)), ref[perm2])
    else:
        with pytest.raises(ValueError):  # rows leaving their 128-row scale block
            permute_out_channels(fmt, t, _rope_perm(576, [224], 64))
    with pytest.raises(ValueError):
        pad_out_channels(fmt, t, 500)


def test_mla_config_parsing():
    cfg, _, _ = deepseek_tiny(DS_SEEDS["awq_quant_attn"], **DS_CASES["awq_quant_attn"])
    spec = decoder_spec_from_config(cfg)
    assert spec.mla == {"kv_lora_rank": 512, "q_lora_rank": 128, "qk_nope_head_dim": 64, "qk_rope_head_dim": 64,
                        "v_head_dim": 64, "softmax_scale": pytest.approx(128 ** -0.5 * yarn_mscale(4.0, 0.8) ** 2),
                        "rope_interleave": True}
    assert spec.kv_heads == 1 and spec.inter == 256
    # the newer rope_parameters key, and a YaRN factor from the two context lengths
    c2 = {k: v for k, v in cfg.items() if k != "rope_theta"}  # transformers 5 writes it under rope_parameters
    rs = dict(c2.pop("rope_scaling"))
    rs.pop("factor")
    c2["rope_parameters"] = {**{k: v for k, v in rs.items() if k != "type"}, "rope_type": "yarn", "rope_theta": 5e4}
    s2 = decoder_spec_from_config(c2)
    assert s2.rope_scaling["factor"] == 4.0 and s2.rope_theta == 5e4 and s2.mla["softmax_scale"] == spec.mla[
        "softmax_scale"]
    # no scaling: the plain scale
    c3 = {k: v for k, v in cfg.items() if k != "rope_scaling"}
    assert decoder_spec_from_config(c3).mla["softmax_scale"] == pytest.approx(128 ** -0.5)
    with pytest.raises(KeyError):
        decoder_spec_from_config({k: v for k, v in cfg.items() if k != "v_head_dim"})
