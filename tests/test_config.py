"""The reference's [experts] / [quant] settings (ccut/config.py:91-108, engine.toml:26-42) as
this path reads them: the values it runs, the ones it refuses and the out-of-range ones."""

from __future__ import annotations

import pytest

from ccut_b200 import config

AWQ = {"quantization_config": {"quant_method": "awq", "bits": 4, "group_size": 128, "zero_point": True,
                               "version": "gemm"}}
FP8 = {"quantization_config": {"quant_method": "fp8", "fmt": "e4m3", "weight_block_size": [128, 128]}}


def test_defaults_and_checkpoint_format():
    # the reference's engine.toml defaults
    app = {"experts": {"expert_residency": "zero", "expert_ring_slots": 2}, "quant": {"quantization": "auto",
           "quant_ignore": [], "fp8_compute_mode": "w8a16", "kv_cache_dtype": "auto"}}
    r = config.resolve(app, AWQ)
    assert r["format"] == "awq_int4_g128" and r["kv_cache_dtype"] == "bf16" and r["residency"] == "hbm"
    assert config.resolve(None, FP8)["format"] == "fp8_b128"
    assert config.quant_settings({"quant": {"kv_cache_dtype": "bf16"}}, FP8)["format"] == "fp8_b128"
    # the reference computes its w8a8 label as w8a16 (dequantized weights, 16-bit activations)
    assert config.quant_settings({"quant": {"fp8_compute_mode": "w8a8"}}, FP8)["fp8_compute_mode"] == "w8a8"
    assert config.expert_settings({"experts": {"expert_residency": "page_cache_only", "expert_ring_slots": 8}})[
        "expert_ring_slots"] == 8


@pytest.mark.parametrize("section, key, value, exc", [
    ("quant", "quantization", "nvfp4_per_token", NotImplementedError),
    ("quant", "quantization", "int4", ValueError),
    ("quant", "fp8_compute_mode", "w4a4", ValueError),
    ("quant", "kv_cache_dtype", "fp8", NotImplementedError),
    ("quant", "kv_cache_dtype", "fp16", ValueError),
    ("experts", "expert_residency", "always", ValueError),
    ("experts", "expert_parallel_size", 0, ValueError),
    ("experts", "expert_parallel_size", "2", ValueError),
    ("engine", "tensor_parallel_size", 2, ValueError),
    ("engine", "pipeline_parallel_size", 2, ValueError),
    ("experts", "expert_ring_slots", 9, ValueError),
])
def test_refused_settings(section, key, value, exc):
    with pytest.raises(exc):
        config.resolve({section: {key: value}}, AWQ)


def test_unquantized_checkpoint_is_refused():
    with pytest.raises(NotImplementedError):
        config.resolve({}, {"hidden_size": 128})


def test_expert_residency_hbm_and_expert_parallel_size():
    assert config.expert_settings(None)["expert_residency"] == "hbm"
    r = config.resolve({"experts": {"expert_residency": "hbm", "expert_parallel_size": 8}}, FP8)
    assert r["residency"] == "hbm" and r["expert_parallel_size"] == 8


def test_cross_validate_admits_expert_parallelism_only():
    app = {"engine": {"tensor_parallel_size": 1, "pipeline_parallel_size": 1}, "experts": {"expert_parallel_size": 4}}
    assert config.cross_validate(app, world_size=4, num_experts=64)["expert_parallel_size"] == 4
    with pytest.raises(ValueError):
        config.cross_validate(app, world_size=2)  # the size must be the process group's
    with pytest.raises(ValueError):
        config.cross_validate({"experts": {"expert_parallel_size": 16}}, num_experts=8)
    with pytest.raises(ValueError):
        config.cross_validate({"engine": {"tensor_parallel_size": 2}, "experts": {"expert_parallel_size": 2}})
