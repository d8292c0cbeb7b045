"""Seeded tiny DeepSeek-V3-style checkpoints for the MLA loader tests (test fixtures).

``deepseek_tiny(seed, ...)`` draws, from ``numpy.random.default_rng(seed)``, a two-layer model
with multi-head latent attention (kv rank 512, rope 64, YaRN scaling with ``mscale`` /
``mscale_all_dim``, interleaved rope channels), a dense MLP in layer 0
(``first_k_dense_replace = 1``) and in layer 1 a MoE block with grouped sigmoid routing
(two groups, one kept, ``e_score_correction_bias``, ``routed_scaling_factor``) and one shared
expert.  MLP, expert and (with ``quant_attn``) attention matrices are seeded AWQ / FP8
matrices (``ccut_b200.synthetic``; AWQ attention scales divided by 4); the other tensors are
bf16.  It returns the
``config.json`` dict, the checkpoint tensors and the same weights as the fp32 state dict of
``transformers``' ``DeepseekV3ForCausalLM`` (dequantized by the oracle; experts in its fused
``gate_up_proj`` / ``down_proj`` layout), from which ``tests/golden/make_golden_deepseek.py``
made the reference logits.  ``oracle_decoder`` builds the oracle's decoder from what
``load_decoder_weights`` reads back.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np

from ccut_b200 import synthetic
from oracle import formats, inputs
from oracle import model as omodel
from oracle import moe
from tests.ckpt_helpers import _matrix_tensors, write_safetensors

# name -> keyword arguments of deepseek_tiny
DS_CASES = {
    "fp8_bf16_attn": {"fmt": "fp8_b128", "q_rank": 0, "d_nope": 32, "d_v": 48, "quant_attn": False},
    "awq_quant_attn": {"fmt": "awq_int4_g128", "q_rank": 128, "d_nope": 64, "d_v": 64, "quant_attn": True},
    "fp8_quant_attn": {"fmt": "fp8_b128", "q_rank": 0, "d_nope": 64, "d_v": 64, "quant_attn": True},
}
DS_SEEDS = {"fp8_bf16_attn": 51, "awq_quant_attn": 52, "fp8_quant_attn": 53}

_V, _H, _HEADS, _R, _DR, _E, _I, _I_DENSE = 512, 256, 4, 512, 64, 8, 128, 256


def _bf16(a):
    return omodel.round_bf16(np.asarray(a, np.float32))


def _quant_config(fmt: str) -> dict:
    if fmt == "awq_int4_g128":
        return {"quant_method": "awq", "bits": 4, "group_size": 128, "zero_point": True, "version": "gemm"}
    return {"quant_method": "fp8", "fmt": "e4m3", "weight_block_size": [128, 128], "activation_scheme": "dynamic"}


def deepseek_tiny(seed: int, fmt: str, q_rank: int = 0, d_nope: int = 32, d_v: int = 48, quant_attn: bool = False):
    """``(config, tensors, hf_state)``: see the module docstring."""
    rng = np.random.default_rng(seed)
    cfg = {"architectures": ["DeepseekV3ForCausalLM"], "model_type": "deepseek_v3", "vocab_size": _V,
           "hidden_size": _H, "intermediate_size": _I_DENSE, "moe_intermediate_size": _I, "num_hidden_layers": 2,
           "num_attention_heads": _HEADS, "num_key_value_heads": _HEADS, "n_shared_experts": 1,
           "n_routed_experts": _E, "routed_scaling_factor": 2.5, "kv_lora_rank": _R, "q_lora_rank": q_rank or None,
           "qk_rope_head_dim": _DR, "v_head_dim": d_v, "qk_nope_head_dim": d_nope, "n_group": 2, "topk_group": 1,
           "num_experts_per_tok": 2, "first_k_dense_replace": 1, "norm_topk_prob": True, "scoring_func": "sigmoid",
           "topk_method": "noaux_tc", "max_position_embeddings": 1024, "rope_theta": 10000.0,
           "rope_scaling": {"type": "yarn", "factor": 4.0, "original_max_position_embeddings": 256, "beta_fast": 32,
                            "beta_slow": 1, "mscale": 1.0, "mscale_all_dim": 0.8},
           "rope_interleave": True, "tie_word_embeddings": False, "rms_norm_eps": 1e-6, "hidden_act": "silu",
           "quantization_config": _quant_config(fmt)}
    bf = synthetic.bf16_bits_from_f32
    t: dict = {}
    hf: dict = {}

    def dense(name: str, out_dim: int, in_dim: int):
        a = _bf16(rng.standard_normal((out_dim, in_dim), dtype=np.float32) / np.float32(np.sqrt(in_dim)))
        t[f"{name}.weight"] = ("BF16", bf(a))
        hf[f"{name}.weight"] = a

    def quant(name: str, out_dim: int, in_dim: int, hf_name: str | None = None, awq_scale: float = 1.0):
        m = synthetic._gen_matrix(rng, fmt, in_dim, out_dim)
        if fmt == "awq_int4_g128" and awq_scale != 1.0:
            m.scales = (m.scales * np.float16(awq_scale)).astype(np.float16)
        t.update(_matrix_tensors(name, m))
        deq = np.ascontiguousarray(inputs.dequant(m).T)  # [out, in]
        if hf_name is not None:
            hf[hf_name] = deq
        return deq

    def vec(name: str, n: int, lo: float = 0.5, hi: float = 1.5):
        a = _bf16(rng.uniform(lo, hi, n).astype(np.float32))
        t[name] = ("BF16", bf(a))
        hf[name] = a

    def attn(name: str, o: int, i: int):
        if quant_attn:  # AWQ attention scales / 4: weights near 1 / sqrt(in), as trained projections are
            quant(name, o, i, f"{name}.weight", awq_scale=0.25)
        else:
            dense(name, o, i)

    emb = _bf16(rng.standard_normal((_V, _H), dtype=np.float32))
    t["model.embed_tokens.weight"] = ("BF16", bf(emb))
    hf["model.embed_tokens.weight"] = emb
    for i in range(2):
        pre = f"model.layers.{i}"
        vec(f"{pre}.input_layernorm.weight", _H)
        sa = f"{pre}.self_attn"
        q_out = _HEADS * (d_nope + _DR)
        if q_rank:
            attn(f"{sa}.q_a_proj", q_rank, _H)
            vec(f"{sa}.q_a_layernorm.weight", q_rank)
            attn(f"{sa}.q_b_proj", q_out, q_rank)
        else:
            attn(f"{sa}.q_proj", q_out, _H)
        attn(f"{sa}.kv_a_proj_with_mqa", _R + _DR, _H)
        vec(f"{sa}.kv_a_layernorm.weight", _R)
        attn(f"{sa}.kv_b_proj", _HEADS * (d_nope + d_v), _R)
        attn(f"{sa}.o_proj", _H, _HEADS * d_v)
        vec(f"{pre}.post_attention_layernorm.weight", _H)
        mlp = f"{pre}.mlp"
        if i == 0:
            quant(f"{mlp}.gate_proj", _I_DENSE, _H, f"{mlp}.gate_proj.weight")
            quant(f"{mlp}.up_proj", _I_DENSE, _H, f"{mlp}.up_proj.weight")
            quant(f"{mlp}.down_proj", _H, _I_DENSE, f"{mlp}.down_proj.weight")
            continue
        router = (rng.standard_normal((_E, _H), dtype=np.float32) * np.float32(0.1)).astype(np.float32)
        bias = rng.uniform(0.0, 0.05, _E).astype(np.float32)
        t[f"{mlp}.gate.weight"] = (None, router)
        t[f"{mlp}.gate.e_score_correction_bias"] = (None, bias)
        hf[f"{mlp}.gate.weight"], hf[f"{mlp}.gate.e_score_correction_bias"] = router, bias
        gate_up, down = [], []
        for e in range(_E):
            g = quant(f"{mlp}.experts.{e}.gate_proj", _I, _H)
            u = quant(f"{mlp}.experts.{e}.up_proj", _I, _H)
            d = quant(f"{mlp}.experts.{e}.down_proj", _H, _I)
            gate_up.append(np.concatenate([g, u]))
            down.append(d)
        hf[f"{mlp}.experts.gate_up_proj"] = np.stack(gate_up)
        hf[f"{mlp}.experts.down_proj"] = np.stack(down)
        for p, (o, n) in (("gate", (_I, _H)), ("up", (_I, _H)), ("down", (_H, _I))):
            quant(f"{mlp}.shared_experts.{p}_proj", o, n, f"{mlp}.shared_experts.{p}_proj.weight")
    vec("model.norm.weight", _H)
    lm = _bf16(rng.standard_normal((_V, _H), dtype=np.float32) / np.float32(np.sqrt(_H)))
    t["lm_head.weight"] = ("BF16", bf(lm))
    hf["lm_head.weight"] = lm
    return cfg, t, hf


def write_deepseek_checkpoint(root: Path, case: str) -> Path:
    import json

    cfg, tensors, _ = deepseek_tiny(DS_SEEDS[case], **DS_CASES[case])
    root.mkdir(parents=True, exist_ok=True)
    (root / "config.json").write_text(json.dumps(cfg))
    write_safetensors(root / "model.safetensors", tensors, {"format": "pt"})
    return root


def _deq(m, fmt: str) -> np.ndarray:
    """A ``load_decoder_weights`` matrix -> fp32 ``[out, in]`` (the oracle's dequant)."""
    kind, a = m
    if kind == "dense":
        return np.asarray(a, np.float32)
    if fmt == "awq_int4_g128":
        return np.ascontiguousarray(formats.awq_dequant(a["qweight"], a["qzeros"], a["scales"]).T)
    return formats.fp8_block_dequant(np.asarray(a["weight"]), np.asarray(a["weight_scale_inv"]))


def oracle_decoder(w: dict, projections: str | None = None):
    """``(MlaWeights per layer, ffn callables, DecoderSpec)`` of the oracle for what
    ``load_decoder_weights`` returned.  ``projections`` mirrors what ``load_decoder`` keeps on
    the device: None, the exact matrices; ``"quantized"`` (``quantized_projections=True``),
    ``kv_a`` rounded to bf16 (it is always dequantized to bf16); ``"bf16"``, q / q_a / kv_a / o
    rounded.  ``kv_b`` stays exact (fp32 on the device)."""
    from ccut_b200.rope_tables import yarn_rope_table

    spec = w["spec"]
    m, fmt = spec.mla, spec.fmt
    dn, dr, dv = m["qk_nope_head_dim"], m["qk_rope_head_dim"], m["v_head_dim"]
    exact = lambda a: a  # noqa: E731
    rb = _bf16 if projections == "bf16" else exact
    rkv = _bf16 if projections else exact
    layers, ffns = [], []
    for lay in w["layers"]:
        qa = rb(_deq(lay["q_a"], fmt)) if "q_a" in lay else None
        layers.append(omodel.MlaWeights(lay["ln1"], rb(_deq(lay["q"], fmt)), rkv(_deq(lay["kv_a"], fmt)),
                                        _deq(lay["kv_b"], fmt), rb(_deq(lay["o"], fmt)), lay["ln2"], spec.heads, dn,
                                        dr, dv, lay["kv_a_norm"], qa, lay.get("q_a_norm"), m["softmax_scale"]))
        kind, f = lay["ffn"]
        if kind == "dense":
            wg, wu, wd = (_deq(("quant", f[p]), fmt).T.copy() for p in ("gate", "up", "down"))
            ffns.append(lambda x, wg=wg, wu=wu, wd=wd: moe.expert_ffn(x, wg, wu, wd))
            continue
        ms, router, experts, shared, bias = f
        ex = [tuple(_deq(("quant", e[p]), fmt).T.copy() for p in ("gate", "up", "down")) for e in experts]
        sh = tuple(_deq(("quant", shared[0][p]), fmt).T.copy() for p in ("gate", "up", "down")) if shared else None
        kw = {"n_group": ms.n_group, "topk_group": ms.topk_group, "routed_scaling": ms.routed_scaling, "bias": bias}
        lookup = lambda e, ex=ex: ex[e]  # noqa: E731
        f = omodel.moe_ffn(router, ms.top_k, ms.routing, lookup, sh, route_kw=kw)
        f.args = (router, ms.top_k, ms.routing, lookup, sh, kw)  # for tests that force another routing
        ffns.append(f)
    inv, f = yarn_rope_table(dr, spec.rope_theta, spec.rope_scaling)
    dspec = omodel.DecoderSpec(spec.hidden, spec.heads, 1, dr, inv, attn_factor=f * f, scaling_type="yarn",
                               eps=spec.eps)
    return layers, ffns, dspec
