"""Dense SwiGLU FFN (ccut_b200.dense.DenseFfn: the grouped expert GEMMs with one expert)
against the oracle's fp32 expert_ffn (ccut/blocks/moe.py:122-141), including an
intermediate size that is not a multiple of 128 (padded with zero channels)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from ccut_b200 import synthetic
from ccut_b200.dense import DenseFfn
from oracle import formats, inputs, moe
from tests.gpu_helpers import TOL, rel_err_rows, x_device

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from ccut_b200 import build
    build.build()


def _awq(rng, K, N):
    return inputs.AwqMatrix(rng.integers(0, 2**32, (K, N // 8), dtype=np.uint64).astype(np.uint32).view(np.int32),
                            rng.integers(0, 2**32, (K // 128, N // 8), dtype=np.uint64).astype(np.uint32).view(np.int32),
                            (np.abs(rng.standard_normal((K // 128, N))) * 0.02 + 1e-3).astype(np.float16))


def _fp8(rng, N, K):
    w = np.clip(rng.standard_normal((N, K)), -448, 448).astype(np.float32)
    codes = synthetic._encode_e4m3(w)
    s = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), ((N + 127) // 128, (K + 127) // 128))).astype(np.float32)
    return inputs.Fp8Matrix(np.asarray(codes, dtype=np.uint8), s)


@pytest.mark.parametrize("kernel", ["tc", "mma"])
@pytest.mark.parametrize("fmt,H,I", [("awq_int4_g128", 256, 384), ("fp8_b128", 256, 320), ("fp8_b128", 384, 10944 // 16)])
def test_dense_ffn_matches_oracle(fmt, H, I, kernel):
    rng = np.random.default_rng(H + I)
    if fmt == "awq_int4_g128":
        g, u, d = _awq(rng, H, I), _awq(rng, H, I), _awq(rng, I, H)
    else:
        g, u, d = _fp8(rng, I, H), _fp8(rng, I, H), _fp8(rng, H, I)
    ffn = DenseFfn(fmt, H, I, g, u, d, kernel=kernel)
    wg, wu, wd = inputs.dequant(g), inputs.dequant(u), inputs.dequant(d)
    for T in (1, 17, 130):
        xb = synthetic.bf16_bits_from_f32(rng.standard_normal((T, H)).astype(np.float32))
        out = ffn.forward(x_device(xb), out_dtype=torch.float32).cpu().numpy()
        ref = moe.expert_ffn(formats.bf16_bits_to_f32(xb), wg, wu, wd)
        assert rel_err_rows(out, ref) <= TOL, f"T={T}"
        outb = ffn.forward(x_device(xb)).float().cpu().numpy()
        assert rel_err_rows(outb, ref) <= TOL
    assert ffn.workspace_status() == 0


def test_dense_ffn_rejects_bad_shapes():
    rng = np.random.default_rng(0)
    with pytest.raises(ValueError):  # AWQ down projection input not a multiple of 128
        DenseFfn("awq_int4_g128", 256, 320, _awq(rng, 256, 320), _awq(rng, 256, 320),
                 inputs.AwqMatrix(np.zeros((320, 32), np.int32), np.zeros((3, 32), np.int32),
                                  np.zeros((3, 256), np.float16)))
    with pytest.raises(NotImplementedError):
        DenseFfn("int8", 256, 256, None, None, None)
