"""GQA attention and RMSNorm on the GPU (ccut_gqa_attention, ccut_rms_norm through the
drop-ins ccut_b200.blocks.attn_gqa / .norm) against the reference's own outputs (golden
fixtures from ccut/blocks/attn_gqa.py:gqa_attention_fast and ccut/blocks/norm.py:rms_norm)
and against the oracle on larger cases: long kv ranges split over CTAs, causal prefill,
soft-capping, both head dims, bf16 outputs, empty kv."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention, formats

pytestmark = pytest.mark.gpu

# fp32 scores and softmax on bf16 inputs: only summation order and exp differ
RTOL, ATOL = 1e-4, 1e-4


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from ccut_b200 import build
    build.build()


def _bf16(rng, shape, scale=1.0):
    bits = formats.bf16_bits_from_f32((rng.standard_normal(shape) * scale).astype(np.float32))
    return bits, formats.bf16_bits_to_f32(bits)


def _dev(bits):
    return torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16)


def test_gqa_matches_reference_golden(golden_dir):
    from ccut_b200.blocks import attn_gqa

    g = np.load(golden_dir / "attn_norm.npz")
    for i in range(4):
        q, k, v = (g[f"gqa{i}_{n}"] for n in "qkv")
        start = int(g[f"gqa{i}_start"])
        s, kv = q.shape[2], k.shape[2]
        mask = attn_gqa.build_causal_mask(s, start)[None, None] if start >= 0 else None
        got = attn_gqa.gqa_attention_fast(_dev(q), _dev(k), _dev(v), mask).cpu().numpy()
        np.testing.assert_allclose(got, g[f"gqa{i}_out"], rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("b,h,kvh,s,L,d,causal,softcap", [
    (2, 32, 4, 1, 3000, 128, True, None),   # decode over a long kv range: many splits
    (1, 32, 4, 70, 70, 128, True, None),    # causal prefill from position 0
    (2, 8, 8, 4, 257, 64, True, 30.0),      # plain heads, head dim 64, soft cap
    (1, 16, 2, 3, 100, 128, False, None),   # no mask
    (3, 4, 1, 9, 9, 64, True, None),        # all heads on one kv head
])
def test_gqa_matches_oracle(b, h, kvh, s, L, d, causal, softcap):
    from ccut_b200.blocks import attn_gqa

    rng = np.random.default_rng(b * 1000 + h * 10 + s)
    qb, q = _bf16(rng, (b, h, s, d))
    kb, k = _bf16(rng, (b, kvh, L, d))
    vb, v = _bf16(rng, (b, kvh, L, d))
    start = L - s if causal else None
    mask = attention.causal_mask(s, start)[None, None] if causal else None
    ref = attention.gqa_attention(q, k, v, mask, softcap=softcap)
    got = attn_gqa.gqa_attention_fast(_dev(qb), _dev(kb), _dev(vb), start_pos=start, softcap=softcap)
    np.testing.assert_allclose(got.cpu().numpy(), ref, rtol=RTOL, atol=ATOL)
    # numpy in -> numpy out, the reference's mask argument instead of start_pos
    got_np = attn_gqa.gqa_attention_fast(q, k, v, attn_gqa.build_causal_mask(s, start) if causal else None,
                                         softcap=softcap)
    assert isinstance(got_np, np.ndarray)
    np.testing.assert_allclose(got_np, ref, rtol=RTOL, atol=ATOL)


def test_gqa_bf16_output_and_edges():
    from ccut_b200 import _lib
    from ccut_b200.blocks import attn_gqa
    from ccut_b200.layer import _ptr, _stream

    rng = np.random.default_rng(7)
    b, h, kvh, s, L, d = 2, 8, 2, 1, 500, 128
    qb, q = _bf16(rng, (b, h, s, d))
    kb, k = _bf16(rng, (b, kvh, L, d))
    vb, v = _bf16(rng, (b, kvh, L, d))
    ref = attention.gqa_attention(q, k, v)
    out = torch.empty((b, h, s, d), dtype=torch.bfloat16, device="cuda")
    lib = _lib.load()
    ws = torch.empty(max(lib.ccut_gqa_attention_workspace_bytes(b, h, kvh, s, L, d), 256), dtype=torch.uint8,
                     device="cuda")
    qd, kd, vd = _dev(qb), _dev(kb), _dev(vb)  # kept alive until the kernel has run
    _lib.call("ccut_gqa_attention", _ptr(qd), _ptr(kd), _ptr(vd), b, h, kvh, s, L, d, -1, 0.0, 0.0,
              _ptr(out), _lib.OUT_BF16, _ptr(ws), ws.numel(), _stream())
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, rtol=1e-2, atol=1e-2)
    # no kv positions: zeros (the reference's 1e-30 clamp on an empty sum)
    z = attn_gqa.gqa_attention_fast(_dev(qb), _dev(kb)[:, :, :0], _dev(vb)[:, :, :0])
    assert z.shape == (b, h, s, d) and torch.count_nonzero(z) == 0
    with pytest.raises(NotImplementedError):  # a non-causal additive mask
        attn_gqa.gqa_attention_fast(q, k, v, np.full((s, L), -1.0, np.float32))
    with pytest.raises(NotImplementedError):
        attn_gqa.gqa_attention_fast(q[..., :96], k[..., :96], v[..., :96])
    with pytest.raises(ValueError):
        attn_gqa.gqa_attention_fast(q, k[:, :1].repeat(3, axis=1), v[:, :1].repeat(3, axis=1))


def test_rms_norm_matches_reference_golden(golden_dir):
    from ccut_b200.blocks import norm

    g = np.load(golden_dir / "attn_norm.npz")
    for i in range(2):
        x = formats.bf16_bits_to_f32(g[f"rms{i}_x"])
        w = g[f"rms{i}_w"]
        y = norm.rms_norm(x, w if w.size else None, float(g[f"rms{i}_eps"]))
        np.testing.assert_allclose(y, g[f"rms{i}_y"], rtol=1e-5, atol=1e-5)


def test_rms_norm_bf16_and_batched_shapes():
    from ccut_b200.blocks import norm

    rng = np.random.default_rng(3)
    xb, x = _bf16(rng, (4, 33, 2048), 2.0)
    w = rng.uniform(0.5, 1.5, 2048).astype(np.float32)
    ref = attention.rms_norm(x, w, 1e-6)
    got = norm.rms_norm(_dev(xb), torch.from_numpy(w).cuda())
    assert got.dtype == torch.bfloat16 and got.shape == (4, 33, 2048)
    np.testing.assert_allclose(got.float().cpu().numpy(), ref, rtol=1e-2, atol=1e-2)
    got32 = norm.rms_norm(torch.from_numpy(x).cuda(), w)
    np.testing.assert_allclose(got32.cpu().numpy(), ref, rtol=1e-5, atol=1e-5)


def test_rope_matches_reference_golden(golden_dir):
    """ccut_apply_rope against the reference's apply_rope (ccut/blocks/rope.py:130-175):
    no scaling (head dim 128) and yarn (attention factor on q, positions ~4000)."""
    from ccut_b200.blocks import rope

    g = np.load(golden_dir / "attn_norm.npz")
    for i in range(2):
        q, k = (formats.bf16_bits_to_f32(g[f"rope{i}_{n}"]) for n in "qk")
        args = (g[f"rope{i}_inv_freq"], g[f"rope{i}_pos"], float(g[f"rope{i}_attn"]), str(g[f"rope{i}_type"]))
        qo, ko = rope.apply_rope(q, k, *args)  # numpy (fp32) in
        np.testing.assert_allclose(qo, g[f"rope{i}_q_out"], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(ko, g[f"rope{i}_k_out"], rtol=1e-5, atol=1e-5)
        qt, kt = rope.apply_rope(_dev(g[f"rope{i}_q"]), _dev(g[f"rope{i}_k"]), *args)  # bf16 tensors in
        np.testing.assert_allclose(qt.cpu().numpy(), g[f"rope{i}_q_out"], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(kt.cpu().numpy(), g[f"rope{i}_k_out"], rtol=1e-5, atol=1e-5)
