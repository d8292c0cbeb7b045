"""Independent pins for the formats the reference does not implement (its parity is
otherwise unpinned): the oracle's AWQ-g128 unpacking and dequant against vLLM's
``awq_pack`` (AutoAWQ GEMM layout), its DeepSeek-V3 grouped sigmoid routing against vLLM's
``grouped_topk``, and its FP8 128 x 128 block dequant against PyTorch's float8_e4m3fn
decode.  Fixtures: tests/golden/vllm_formats.npz (tests/golden/make_golden_vllm.py)."""

from __future__ import annotations

import numpy as np
import torch

from oracle import formats, routing


def test_awq_dequant_matches_vllm_packing(golden_dir):
    g = np.load(golden_dir / "vllm_formats.npz")
    q, z, s = g["awq_q"].astype(np.int64), g["awq_z"].astype(np.int64), g["awq_s"]
    direct = (q - np.repeat(z, 128, axis=0)).astype(np.float32) * np.repeat(s, 128, axis=0).astype(np.float32)
    got = formats.awq_dequant(g["awq_qweight"], g["awq_qzeros"], s)
    assert np.array_equal(got.view(np.uint32), direct.view(np.uint32))  # bit-exact
    assert np.array_equal(formats.awq_unpack(g["awq_qweight"], "awq"), q)


def test_grouped_sigmoid_routing_matches_vllm(golden_dir):
    g = np.load(golden_dir / "vllm_formats.npz")
    logits = g["route_logits"]
    w_ref, ids_ref = g["route_w"], g["route_ids"]
    w, ids = routing.grouped_sigmoid_topk(logits, 8, 8, 4, 2.5)
    # vLLM's top-k is unsorted: compare the chosen sets, and the weights matched by expert
    for t in range(logits.shape[0]):
        assert set(ids[t].tolist()) == set(ids_ref[t].tolist()), t
        mine = dict(zip(ids[t].tolist(), w[t].tolist()))
        for e, wr in zip(ids_ref[t].tolist(), w_ref[t].tolist()):
            assert abs(mine[e] - wr) <= 1e-6 * max(1.0, abs(wr))


def test_fp8_block_dequant_matches_torch_e4m3():
    rng = np.random.default_rng(5)
    N, K = 256, 384
    codes = rng.integers(0, 256, (N, K), dtype=np.int64).astype(np.uint8)
    codes[(codes & 0x7F) == 0x7F] = 0x3C  # NaN codes are covered by the reference's table test
    sc = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), (N // 128, K // 128))).astype(np.float32)
    f = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    ref = f * np.repeat(np.repeat(sc, 128, 0), 128, 1)
    got = formats.fp8_block_dequant(codes, sc)
    assert np.array_equal(got.view(np.uint32), ref.astype(np.float32).view(np.uint32))
