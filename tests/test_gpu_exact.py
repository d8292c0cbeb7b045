"""Exactness of the tcgen05 expert GEMM's weight operand, and parity at the benchmark's sizes
that the other GPU tests do not reach.

- The down GEMM fed one-hot intermediate rows returns rows of the dequantized down matrix
  exactly (equal fp32 values; only the sign of a zero may differ): the kernel multiplies the unscaled code ((q - z) for AWQ, the e4m3 value for FP8,
  both exact in bf16) and applies the fp32 group / block scale when it promotes each 128-k
  partial sum, so one product is fl32(code * s), the reference's dequantized weight
  (ccut/quant/kernels.py:150-171, :276-295), including FP8 blocks at the smallest scale.
- FP8 blocks at scale 1e-3 compared element by element with the oracle: each output element
  within 2^-7 of the sum of the magnitudes of its products (the bf16 SwiGLU rows round each
  product by at most 2^-9).
- The config-1 prefill (T = 2048, the benchmark's default workload) against the oracle on 64
  rows spread over the batch (every 256-token tile of the two shared-expert slices) and on
  every row of the routed expert with the most rows.
- The config-4 layer at full size (H = 7168, 256 experts, I = 2048, grouped sigmoid routing
  with a selection bias, one shared expert, FP8 blocks), generated on the GPU: the 4096-token
  prefill (tcgen05) and a 256-token decode (mma.sync) against the oracle on a token subset,
  dequantizing only the experts those tokens touch; the routing against the oracle's
  grouped sigmoid top-k except at near ties."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import formats, inputs, moe, routing
from tests.gpu_helpers import TOL, gpu_layer, oracle_forward, rel_err_rows, small_cfg, x_device

pytestmark = pytest.mark.gpu

FMTS = ["awq_int4_g128", "fp8_b128"]


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from ccut_b200 import build
    build.build()


def _set_small_fp8_scales(lw, value=1e-3):
    for ew in lw.experts + lw.shared:
        for m in (ew.gate, ew.up, ew.down):
            m.scale[...] = np.float32(value)


@pytest.mark.parametrize("fmt", FMTS)
def test_down_product_is_the_exact_dequantized_weight(fmt):
    from ccut_b200.layer import Routing

    E, H, I = 4, 256, 384
    lw = inputs.make_layer(small_cfg(fmt, hidden=H, inter=I, experts=E, top_k=1), seed=5)
    if fmt == "fp8_b128":  # the smallest scale of the format's range on some blocks
        lw.experts[1].down.scale[:, 0] = np.float32(1e-3)
        lw.experts[2].down.scale[...] = np.float32(1e-3)
    L = gpu_layer(lw, kernel="tc")
    T = E * I  # every intermediate index of every expert, over two token tiles per expert
    ids = torch.tensor([[t % E] for t in range(T)], dtype=torch.int32, device="cuda")
    w = torch.ones((T, 1), dtype=torch.float32, device="cuda")
    perm = L.permute(Routing(ids, w))
    row_token = perm.row_token[:T].cpu().numpy()
    h = torch.zeros((T, I), dtype=torch.bfloat16)
    hot = (row_token // E) % I  # one-hot position of each row
    h[np.arange(T), hot] = 1.0
    y = L.down(h.to("cuda").view(torch.int16), perm, T, 1).cpu().numpy()
    offs = perm.offsets.cpu().numpy()
    for e in range(E):
        wd = inputs.dequant(lw.experts[e].down)  # fp32 [I, H], the reference's dequant
        for r in range(offs[e], offs[e + 1]):
            # exact values; the one bit allowed to differ is the sign of a zero (an e4m3 -0
            # code dequantizes to -0, the tensor core's sum of products gives +0)
            assert np.array_equal(y[r], wd[hot[r]]) and not np.isnan(y[r]).any(), (e, r)


def test_fp8_small_block_scales_elementwise():
    cfg = small_cfg("fp8_b128", hidden=512, inter=256, experts=8, top_k=2, shared=1)
    lw = inputs.make_layer(cfg, seed=9)
    _set_small_fp8_scales(lw)
    L = gpu_layer(lw, kernel="tc")
    xb = lw.make_x(300)
    y, r = L.forward(x_device(xb), out_dtype=torch.float32, return_routing=True)
    ids, wts = r.ids.cpu().numpy(), r.weights.cpu().numpy()
    x = formats.bf16_bits_to_f32(xb)
    ref = np.zeros((300, 512), np.float32)
    mag = np.zeros((300, 512), np.float32)
    mats = [(inputs.dequant(ew.gate), inputs.dequant(ew.up), inputs.dequant(ew.down)) for ew in lw.experts]
    sh = tuple(inputs.dequant(m) for m in (lw.shared[0].gate, lw.shared[0].up, lw.shared[0].down))
    for t in range(300):
        parts = [(float(wts[t, j]), mats[int(ids[t, j])]) for j in range(2)] + [(1.0, sh)]
        for wt, (wg, wu, wd) in parts:
            hrow = moe.silu_mul(x[t:t + 1] @ wg, x[t:t + 1] @ wu)
            ref[t] += wt * (hrow @ wd)[0]
            mag[t] += abs(wt) * (np.abs(hrow) @ np.abs(wd))[0]
    err = np.abs(y.cpu().numpy() - ref)
    assert (err <= 2.0 ** -7 * mag + 1e-30).all(), float((err / np.maximum(mag, 1e-30)).max())


def test_cfg1_prefill_every_tile_matches_oracle():
    lw = inputs.make_layer("cfg1", seed=0)
    L = gpu_layer(lw)
    xb = lw.make_x(2048)  # the benchmark's default workload: the tcgen05 kernel
    y, r = L.forward(x_device(xb), return_routing=True)
    ids, wts = r.ids.cpu().numpy(), r.weights.cpu().numpy()
    counts = np.bincount(ids.ravel(), minlength=64)
    busiest = int(counts.argmax())
    rows = sorted(set(range(0, 2048, 32)) | set(np.nonzero((ids == busiest).any(axis=1))[0].tolist()))
    assert len(rows) >= 64 + 1
    ref, _, _ = oracle_forward(lw, xb[rows], ids=ids[rows], weights=wts[rows])
    assert rel_err_rows(y.float().cpu().numpy()[rows], ref) <= TOL
    assert L.workspace_status() == 0


class _DeviceExperts:
    """Oracle lookups of a GPU-generated layer: one expert's matrices copied to the host and
    dequantized at a time (the whole layer is 45 GB in fp32)."""

    def __init__(self, lw):
        self.lw = lw
        self._key, self._val = None, None

    @staticmethod
    def _host(m):
        return inputs.Fp8Matrix(m.weight.cpu().numpy(), m.scale.cpu().numpy())

    def _get(self, key, ew):
        if key != self._key:
            self._key = key
            self._val = tuple(inputs.dequant(self._host(m)) for m in (ew.gate, ew.up, ew.down))
        return self._val

    def w_lookup(self, e):
        return self._get(e, self.lw.experts[e])

    def shared(self):
        return self._get("shared", self.lw.shared[0])


def test_cfg4_full_size_prefill_and_decode_match_oracle():
    from ccut_b200.synthetic import make_layer_device

    lw = make_layer_device("cfg4", seed=3)
    c = lw.cfg
    bias = (np.random.default_rng(4).standard_normal(c.num_experts) * 0.01).astype(np.float32)
    L = gpu_layer(lw, bias=bias)
    ox = _DeviceExperts(lw)
    xb = lw.make_x(4096)
    x = formats.bf16_bits_to_f32(xb)
    for T, picks in ((4096, [0, 1, 777, 2048, 4095]), (256, [0, 100, 255])):
        y, r = L.forward(x_device(xb[:T]), return_routing=True)
        ids, wts = r.ids.cpu().numpy(), r.weights.cpu().numpy()
        # routing: the oracle's grouped sigmoid top-k with the same bias, except near ties
        logits = x[:T] @ lw.router.T
        _, ref_ids = routing.route(logits, c.top_k, c.routing, bias=bias, **c.route_kw)
        score = 1.0 / (1.0 + np.exp(-logits.astype(np.float64))) + bias
        bad = [t for t in range(T) if set(ids[t]) != set(ref_ids[t])
               and abs(np.sort(score[t])[::-1][c.top_k - 1] - np.sort(score[t])[::-1][c.top_k]) > 1e-5]
        assert len(bad) <= T // 100, bad[:8]
        ref = moe.moe_combine(x[picks], ids[picks], wts[picks], ox.w_lookup)
        ref += moe.expert_ffn(x[picks], *ox.shared())
        assert rel_err_rows(y.float().cpu().numpy()[picks], ref) <= TOL, T
    assert L.workspace_status() == 0
