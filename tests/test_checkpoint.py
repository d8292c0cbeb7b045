"""Checkpoint loader on the host: safetensors header parsing, config resolution, expert
indexing and the error classes (no GPU; the upload into HBM is covered by
tests/test_gpu_checkpoint.py)."""

from __future__ import annotations

import json
import struct

import numpy as np
import pytest

from ccut_b200 import checkpoint as ck
from oracle import inputs
from tests.ckpt_helpers import merged_shared, write_checkpoint, write_safetensors
from tests.gpu_helpers import small_cfg


def _layer(fmt, shared=2, mode="softmax_topk"):
    return inputs.make_layer(small_cfg(fmt, mode, hidden=256, inter=128, experts=8, top_k=2, shared=shared), seed=5)


def test_safetensors_round_trip(tmp_path):
    rng = np.random.default_rng(0)
    t = {"a": (None, rng.standard_normal((3, 5)).astype(np.float32)),
         "b": (None, rng.integers(0, 2**31, (7,), dtype=np.int64).astype(np.int32)),
         "c": ("F8_E4M3", rng.integers(0, 256, (2, 4, 8), dtype=np.uint8)),
         "d": ("BF16", rng.integers(0, 2**16, (6,), dtype=np.uint16)),
         "e": (None, np.float16([1.5, -2.0]))}
    write_safetensors(tmp_path / "x.safetensors", t, {"k": "v"})
    sh = ck.SafetensorsShard(tmp_path / "x.safetensors")
    assert sh.names == list(t) and sh.metadata == {"k": "v"}
    for name, (dt, a) in t.items():
        got = sh.array(name)
        assert got.shape == a.shape and np.array_equal(got.view(np.uint8), np.ascontiguousarray(a).view(np.uint8))
        assert not got.flags.writeable
    assert sh.info("c").dtype == "F8_E4M3"
    with pytest.raises(KeyError):
        sh.array("missing")


def test_safetensors_rejects_corrupt_files(tmp_path):
    p = tmp_path / "bad.safetensors"
    p.write_bytes(b"\x01\x02")
    with pytest.raises(ValueError):
        ck.SafetensorsShard(p)
    hdr = json.dumps({"w": {"dtype": "F32", "shape": [4], "data_offsets": [0, 12]}}).encode()
    p.write_bytes(struct.pack("<Q", len(hdr)) + hdr + b"\0" * 16)  # 4 floats need 16 bytes, not 12
    with pytest.raises(ValueError):
        ck.SafetensorsShard(p)
    hdr = json.dumps({"w": {"dtype": "F32", "shape": [8], "data_offsets": [0, 32]}}).encode()
    p.write_bytes(struct.pack("<Q", len(hdr)) + hdr + b"\0" * 16)  # data section shorter than declared
    with pytest.raises(ValueError):
        ck.SafetensorsShard(p)


def test_expert_pattern():
    rx = ck.expert_pattern("model.layers.{layer}.mlp.experts.{expert}.{proj}_proj")
    m = rx.match("model.layers.12.mlp.experts.63.down_proj.qweight")
    assert m and (m["layer"], m["expert"], m["proj"]) == ("12", "63", "down")
    assert rx.match("model.layers.1.mlp.shared_experts.gate_proj.weight") is None
    assert rx.match("xmodel.layers.1.mlp.experts.0.up_proj.weight") is None  # anchored


def test_config_resolution():
    base = {"hidden_size": 2048, "moe_intermediate_size": 1408, "n_routed_experts": 64, "num_experts_per_tok": 6,
            "n_shared_experts": 2, "norm_topk_prob": False,
            "quantization_config": {"quant_method": "awq", "bits": 4, "group_size": 128, "zero_point": True}}
    s = ck.moe_spec_from_config(base)
    assert (s.fmt, s.hidden, s.inter, s.num_experts, s.top_k, s.routing, s.shared_inter) == \
        ("awq_int4_g128", 2048, 1408, 64, 6, "softmax_topk", 2816)
    qwen = {"text_config": {"hidden_size": 2048, "moe_intermediate_size": 768, "num_experts": 128,
                            "num_experts_per_tok": 8, "norm_topk_prob": True,
                            "quantization_config": {"quant_method": "awq", "bits": 4, "group_size": 128}}}
    s = ck.moe_spec_from_config(qwen)
    assert (s.num_experts, s.routing, s.shared_inter) == (128, "topk_softmax", 0)
    v3 = {"hidden_size": 7168, "moe_intermediate_size": 2048, "n_routed_experts": 256, "num_experts_per_tok": 8,
          "n_shared_experts": 1, "norm_topk_prob": True, "scoring_func": "sigmoid", "n_group": 8, "topk_group": 4,
          "routed_scaling_factor": 2.5,
          "quantization_config": {"quant_method": "fp8", "fmt": "e4m3", "weight_block_size": [128, 128]}}
    s = ck.moe_spec_from_config(v3)
    assert (s.fmt, s.routing, s.n_group, s.topk_group, s.routed_scaling, s.shared_inter) == \
        ("fp8_b128", "sigmoid_group", 8, 4, 2.5, 2048)
    # DeepSeek-V2 (not Lite): group-limited greedy softmax routing, routed scaling 16
    for extra in ({"topk_method": "group_limited_greedy", "n_group": 8, "topk_group": 3},
                  {"routed_scaling_factor": 16.0}):
        with pytest.raises(NotImplementedError):
            ck.moe_spec_from_config({**base, **extra})
    lite = ck.moe_spec_from_config({**base, "topk_method": "greedy", "n_group": 1, "routed_scaling_factor": 1.0})
    assert lite.routing == "softmax_topk"
    for bad in ({"quant_method": "gptq", "bits": 4}, {"quant_method": "awq", "bits": 8, "group_size": 128},
                {"quant_method": "awq", "bits": 4, "group_size": 64},
                {"quant_method": "fp8", "weight_block_size": [1, 128]}, {"quant_method": "fp8"}):
        with pytest.raises(NotImplementedError):
            ck.quant_format({"quantization_config": bad})
    with pytest.raises(NotImplementedError):
        ck.quant_format({"hidden_size": 8})
    with pytest.raises(ValueError):
        ck.moe_spec_from_config({"hidden_size": 8, "quantization_config": base["quantization_config"]})


@pytest.mark.parametrize("ct", [False, True])
@pytest.mark.parametrize("fmt", ["awq_int4_g128", "fp8_b128"])
def test_load_layer_weights_matches_the_written_layer(tmp_path, fmt, ct):
    """The layer read back equals the written one; ``ct``: written in compressed-tensors form
    (int4 repacked into AWQ's layout, FP8 block scales under ``weight_scale``)."""
    lw = _layer(fmt)
    root = write_checkpoint(tmp_path / "m", lw, layer=3, router_bf16=True, ct=ct)
    spec, router, experts, shared, bias = ck.load_layer_weights(root, 3)
    c = lw.cfg
    assert (spec.fmt, spec.hidden, spec.inter, spec.num_experts, spec.top_k, spec.shared_inter) == \
        (fmt, c.hidden, c.inter, c.num_experts, c.top_k, c.num_shared * c.shared_inter)
    assert bias is None and len(experts) == c.num_experts and len(shared) == 1
    # the router went through bf16
    from oracle import formats
    assert np.array_equal(router, formats.bf16_bits_to_f32(inputs.synthetic.bf16_bits_from_f32(lw.router)))
    fields = ("qweight", "qzeros", "scales") if fmt == "awq_int4_g128" else ("weight", "weight_scale_inv")
    src = {"weight_scale_inv": "scale"}
    for e in (0, 5, 7):
        for proj in ("gate", "up", "down"):
            for f in fields:
                assert np.array_equal(experts[e][proj][f], getattr(getattr(lw.experts[e], proj), src.get(f, f)))
    ms = merged_shared(lw)
    for proj in ("gate", "up", "down"):
        for f in fields:
            assert np.array_equal(shared[0][proj][f], getattr(ms[proj], src.get(f, f)))


@pytest.mark.parametrize("fmt", ["fp8_channel", "int4_sym_g128"])
def test_load_compressed_tensors_channel_formats(tmp_path, fmt):
    """compressed-tensors per-channel FP8 (the reference's own checkpoints) and symmetric int4
    with fp32 group scales read back as tensors that dequantize to the written matrices."""
    from ccut_b200 import formats as F
    from oracle import formats

    lw = _layer(fmt, shared=1)
    root = write_checkpoint(tmp_path / "m", lw, layer=3, ct=True)
    spec, router, experts, shared, bias = ck.load_layer_weights(root, 3)
    assert spec.fmt == fmt and len(experts) == lw.cfg.num_experts and len(shared) == 1

    def deq(t):  # fp32 [N, K] of a loaded matrix, through the canonical form
        c = F.canonical(fmt, t)
        if fmt == "fp8_channel":
            return formats.fp8_e4m3_decode(c["weight"]) * np.repeat(c["scales"], 128, axis=0).T
        q = formats.awq_unpack(c["qweight"]).astype(np.float32) - 8.0
        return (q * np.repeat(c["scales"], 128, axis=0)).T

    for e in (0, 5, 7):
        for proj in ("gate", "up", "down"):
            ref = inputs.dequant(getattr(lw.experts[e], proj)).T
            assert np.array_equal(deq(experts[e][proj]).astype(np.float32), ref)
    for proj in ("gate", "up", "down"):
        assert np.array_equal(deq(shared[0][proj]).astype(np.float32), inputs.dequant(getattr(lw.shared[0], proj)).T)


def test_load_errors(tmp_path):
    lw = _layer("fp8_b128")
    # a missing block scale
    root = write_checkpoint(tmp_path / "a", lw, drop=("model.layers.3.mlp.experts.1.up_proj.weight_scale_inv",))
    with pytest.raises(ValueError, match="scale"):
        ck.load_layer_weights(root, 3)
    # a missing expert
    root = write_checkpoint(tmp_path / "b", lw, drop=tuple(f"model.layers.3.mlp.experts.6.down_proj.{s}"
                                                             for s in ("weight", "weight_scale_inv")))
    with pytest.raises(ValueError, match="missing"):
        ck.load_layer_weights(root, 3)
    # the wrong layer
    root = write_checkpoint(tmp_path / "c", lw)
    with pytest.raises(ValueError):
        ck.load_layer_weights(root, 4)
    # a per-token shared-expert gate (Qwen2-MoE) is not run by this path
    lw2 = _layer("awq_int4_g128")
    root = write_checkpoint(tmp_path / "d", lw2)
    from tests.ckpt_helpers import write_safetensors as ws
    ws(root / "extra.safetensors", {"model.layers.3.mlp.shared_expert_gate.weight": (None, np.zeros((1, 256), np.float32))})
    idx = json.loads((root / "model.safetensors.index.json").read_text())
    idx["weight_map"]["model.layers.3.mlp.shared_expert_gate.weight"] = "extra.safetensors"
    (root / "model.safetensors.index.json").write_text(json.dumps(idx))
    with pytest.raises(NotImplementedError):
        ck.load_layer_weights(root, 3)
    # no config.json
    with pytest.raises(FileNotFoundError):
        ck.CheckpointReader(tmp_path / "nowhere")


def test_single_file_checkpoint_without_index(tmp_path):
    lw = _layer("awq_int4_g128", shared=0, mode="topk_softmax")
    root = write_checkpoint(tmp_path / "m", lw, layer=0)
    # fold the two shards into one model.safetensors
    t = {}
    for f in sorted(root.glob("model-*.safetensors")):
        sh = ck.SafetensorsShard(f)
        t.update({n: (sh.info(n).dtype, np.array(sh.array(n))) for n in sh.names})
        f.unlink()
    (root / "model.safetensors.index.json").unlink()
    write_safetensors(root / "model.safetensors", t)
    spec, router, experts, shared, _ = ck.load_layer_weights(root, 0)
    assert spec.routing == "topk_softmax" and shared == [] and len(experts) == lw.cfg.num_experts
    assert np.array_equal(experts[2]["down"]["scales"], lw.experts[2].down.scales)
