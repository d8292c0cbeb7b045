"""compressed-tensors checkpoints on the CPU: the int4 ``pack-quantized`` repack into AWQ's
layout against the ``compressed_tensors`` library's own packing and dequantization
(``tests/golden/ct_int4.npz``, made by ``tests/golden/make_golden_ct.py``), its checks, and
which ``quantization_config`` schemes resolve to this path's formats."""

from __future__ import annotations

import numpy as np
import pytest

from ccut_b200 import checkpoint as ck
from ccut_b200.quant import ct_int4_to_awq
from oracle import formats
from tests.ckpt_helpers import ct_quant_config


@pytest.mark.parametrize("case", ["sym", "asym"])
def test_ct_int4_repack_matches_library(golden_dir, case):
    """AWQ tensors from the library's packed int4 dequantize (oracle) to the library's own
    dequantized weight, bit for bit."""
    g = np.load(golden_dir / "ct_int4.npz")
    zp = g[f"{case}_weight_zero_point"] if f"{case}_weight_zero_point" in g else None
    t = ct_int4_to_awq(g[f"{case}_weight_packed"], g[f"{case}_weight_scale"], zp, g[f"{case}_weight_shape"])
    N, K = g[f"{case}_weight_shape"]
    assert t["qweight"].shape == (K, N // 8) and t["qzeros"].shape == (K // 128, N // 8)
    assert t["scales"].shape == (K // 128, N) and t["scales"].dtype == np.float16
    w = formats.awq_dequant(t["qweight"], t["qzeros"], t["scales"]).T
    assert np.array_equal(w, g[f"{case}_weight"])
    if zp is None:
        assert np.all(formats.awq_unpack(t["qzeros"]) == 8)


def test_ct_int4_checks(golden_dir):
    g = np.load(golden_dir / "ct_int4.npz")
    wp, s, shape = g["asym_weight_packed"], g["asym_weight_scale"], g["asym_weight_shape"]
    zp = g["asym_weight_zero_point"]
    with pytest.raises(ValueError):  # a scale fp16 cannot hold
        ct_int4_to_awq(wp, s + np.float32(1e-7), zp, shape)
    with pytest.raises(ValueError):
        ct_int4_to_awq(wp.astype(np.int64), s, zp, shape)
    with pytest.raises(ValueError):
        ct_int4_to_awq(wp, s[:, :1], zp, shape)
    with pytest.raises(ValueError):
        ct_int4_to_awq(wp, s, zp[:, :1], shape)
    with pytest.raises(ValueError):
        ct_int4_to_awq(wp[:, :8], s, zp, shape)
    with pytest.raises(ValueError):
        ct_int4_to_awq(wp, s, zp, shape, group_size=64)


def test_compressed_tensors_config_resolution():
    base = {"hidden_size": 256}
    assert ck.quant_format({**base, "quantization_config": ct_quant_config("awq_int4_g128")}) == "awq_int4_g128"
    assert ck.quant_format({**base, "quantization_config": ct_quant_config("fp8_b128")}) == "fp8_b128"

    def variant(fmt, **w):
        q = ct_quant_config(fmt)
        grp = q["config_groups"]["group_0"]
        grp["weights"] = {**grp["weights"], **w}
        return {**base, "quantization_config": q}

    assert ck.quant_format({**base, "quantization_config": ct_quant_config("fp8_channel")}) == "fp8_channel"
    assert ck.quant_format({**base, "quantization_config": ct_quant_config("int4_sym_g128")}) == "int4_sym_g128"
    assert ck.quant_format(variant("fp8_b128", strategy="tensor")) == "fp8_channel"  # one scale for all channels
    assert ck.quant_format(variant("fp8_b128", strategy="channel")) == "fp8_channel"
    for cfg in (variant("awq_int4_g128", group_size=64), variant("awq_int4_g128", strategy="channel"),
                variant("awq_int4_g128", num_bits=8), variant("awq_int4_g128", actorder="group"),
                variant("fp8_b128", strategy="group"), variant("fp8_b128", block_structure=[64, 64])):
        with pytest.raises(NotImplementedError):
            ck.quant_format(cfg)
    q = ct_quant_config("awq_int4_g128")
    q["config_groups"]["group_0"]["input_activations"] = {"num_bits": 8, "type": "int", "strategy": "token"}
    with pytest.raises(NotImplementedError):  # W4A8: activations would be quantized
        ck.quant_format({**base, "quantization_config": q})
    q = ct_quant_config("awq_int4_g128")
    q["format"] = "naive-quantized"  # int4 values stored unpacked, one per int8
    with pytest.raises(NotImplementedError):
        ck.quant_format({**base, "quantization_config": q})
    q = ct_quant_config("awq_int4_g128")
    q["config_groups"]["group_1"] = q["config_groups"]["group_0"]
    with pytest.raises(NotImplementedError):
        ck.quant_format({**base, "quantization_config": q})
