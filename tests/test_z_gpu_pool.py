"""Attention over a cache pool on the GPU (``ccut_gqa_attention_pool``,
``ccut_mla_attention_pool``, ``KvPool``): one launch for sequences of different lengths
against the oracle per sequence, slots outside the pool, and the engine backend with pooled
caches (GQA and MLA models) against the same backend with separate caches."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention, formats
from tests.gpu_helpers import gpu_layer
from tests.model_helpers import make_tiny, quantized_layers

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from ccut_b200 import build
    build.build()


def _bf16(a):
    return formats.bf16_bits_to_f32(formats.bf16_bits_from_f32(np.asarray(a, np.float32)))


@pytest.mark.parametrize("d", [64, 128])
def test_pool_attention_matches_oracle(d):
    from ccut_b200 import _lib
    from ccut_b200.layer import _ptr, _stream
    from ccut_b200.model import KvPool

    rng = np.random.default_rng(d)
    n_slots, layers, kvh, L, heads = 4, 2, 2, 300, 8
    pool = KvPool(n_slots, layers, kvh, L, d)
    kv_host = _bf16(rng.standard_normal((2, n_slots, layers, kvh, L, d)))
    pool.k.copy_(torch.from_numpy(kv_host[0]).cuda().to(torch.bfloat16))
    pool.v.copy_(torch.from_numpy(kv_host[1]).cuda().to(torch.bfloat16))
    slots, starts = [2, 0, 3, -1, 7, 1], [10, 250, 0, 5, 5, -3]  # the last three read nothing
    B, layer = len(slots), 1
    qh = _bf16(rng.standard_normal((B, heads, 1, d)))
    q = torch.from_numpy(qh).cuda().to(torch.bfloat16)
    sl = torch.tensor(slots, dtype=torch.int32, device="cuda")
    st = torch.tensor(starts, dtype=torch.int32, device="cuda")
    out = torch.empty((B, heads, 1, d), dtype=torch.float32, device="cuda")
    lib = _lib.load()
    ws = torch.empty(max(lib.ccut_gqa_attention_workspace_bytes(B, heads, kvh, 1, L, d), 256), dtype=torch.uint8,
                     device="cuda")
    _lib.call("ccut_gqa_attention_pool", _ptr(q), _ptr(pool.k[0, layer]), _ptr(pool.v[0, layer]), _ptr(sl), _ptr(st),
              B, heads, kvh, 1, L, d, int(pool.k.stride(0)), n_slots, 0.0, 0.0, _ptr(out), _lib.OUT_F32, _ptr(ws),
              ws.numel(), _stream())
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for b, (slot, start) in enumerate(zip(slots, starts)):
        if not (0 <= slot < n_slots and start >= 0):
            assert np.count_nonzero(got[b]) == 0
            continue
        k = kv_host[0, slot, layer][None, :, : start + 1]
        v = kv_host[1, slot, layer][None, :, : start + 1]
        np.testing.assert_allclose(got[b:b + 1], attention.gqa_attention(qh[b:b + 1], k, v), rtol=1e-4, atol=1e-4)


def test_backend_pooled_matches_separate_caches():
    """A decode step of three requests through one pooled attention launch per layer gives the
    logits and greedy tokens of the same requests with separate caches."""
    from ccut_b200.backend import GenericBackend
    from ccut_b200.model import DecoderLayer, MoeDecoder, rope_table

    t = make_tiny(37, kv_heads=2, qk_norm="head")
    q = quantized_layers(t, "fp8_b128", seed=37)
    layers = [DecoderLayer(w.ln1, w.wq, w.wk, w.wv, w.wo, w.ln2, gpu_layer(ol.lw), w.q_norm, w.k_norm, heads=t.heads,
                           kv_heads=t.kv_heads, head_dim=t.head_dim) for w, ol in zip(t.attn, q)]
    inv, af = rope_table(t.head_dim, t.theta)
    dec = MoeDecoder(t.embed, layers, t.final_norm, t.lm_head, inv_freq=inv, attention_factor=af, eps=t.eps)
    rng = np.random.default_rng(13)
    prompts = [[int(x) for x in rng.integers(0, t.vocab, n)] for n in (9, 30, 3)]
    sep = GenericBackend(dec, max_seqs=3, max_len=128)
    pooled = GenericBackend(dec, max_seqs=3, max_len=128, pool=True)
    a, b = [list(p) for p in prompts], [list(p) for p in prompts]
    for step in range(4):
        for x, y in zip(sep.logits_batch(a), pooled.logits_batch(b)):
            x, y = x.cpu().numpy(), y.cpu().numpy()
            assert np.abs(x - y).max() <= 1e-2 * np.abs(x).max(), step
        for s, tok in zip(a, sep.generate_batch([(s, {"temperature": 0.0}) for s in a])):
            s.append(tok)
        for s, tok in zip(b, pooled.generate_batch([(s, {"temperature": 0.0}) for s in b])):
            s.append(tok)
    assert sorted(s.cache.slot for s in pooled._seqs) == [0, 1, 2]


def test_mla_pool_attention_matches_oracle():
    """One ``ccut_mla_attention_pool`` launch over latent caches of different lengths (some
    split over CTAs) against the oracle's MLA attention per sequence; rows of slots outside
    the pool or with a negative start come out zero."""
    from ccut_b200 import _lib
    from ccut_b200.layer import _ptr, _stream
    from ccut_b200.model import KvPool

    rng = np.random.default_rng(5)
    n_slots, layers, L, heads, dn, dv = 4, 2, 1100, 16, 128, 128
    pool = KvPool(n_slots, layers, 1, L, 576, values=False)
    kv_host = _bf16(rng.standard_normal((n_slots, layers, 1, L, 576)))
    pool.k.copy_(torch.from_numpy(kv_host).cuda().to(torch.bfloat16))
    slots, starts = [2, 0, 3, -1, 7, 1], [10, 1099, 0, 5, 5, -3]  # the last three read nothing
    B, layer = len(slots), 1
    qn = _bf16(rng.standard_normal((B, heads, dn)))
    qp = _bf16(rng.standard_normal((B, heads, 64)))
    ku = _bf16(rng.standard_normal((512, heads * dn)) * 0.05)
    vu = _bf16(rng.standard_normal((512, heads * dv)) * 0.05)
    scale = float(1.0 / np.sqrt(dn + 64))
    q_lat = np.einsum("bhd,rhd->bhr", qn, ku.reshape(512, heads, dn))
    q = torch.from_numpy(np.concatenate([q_lat, qp], axis=-1).astype(np.float32)).cuda().contiguous()
    sl = torch.tensor(slots, dtype=torch.int32, device="cuda")
    st = torch.tensor(starts, dtype=torch.int32, device="cuda")
    out = torch.empty((B * heads, 512), dtype=torch.float32, device="cuda")
    lib = _lib.load()
    ws = torch.empty(max(lib.ccut_mla_attention_workspace_bytes(B, heads, 1, L), 256), dtype=torch.uint8,
                     device="cuda")
    _lib.call("ccut_mla_attention_pool", _ptr(q), _ptr(pool.k[0, layer]), _ptr(sl), _ptr(st), B, heads, 1, L, 512, 64,
              int(pool.k.stride(0)), n_slots, scale, _ptr(out), _lib.OUT_F32, _ptr(ws), ws.numel(), _stream())
    torch.cuda.synchronize()
    o_lat = out.cpu().numpy().reshape(B, heads, 512)
    for b, (slot, start) in enumerate(zip(slots, starts)):
        if not (0 <= slot < n_slots and start >= 0):
            assert np.count_nonzero(o_lat[b]) == 0
            continue
        rows = kv_host[slot, layer, 0, : start + 1]
        ref = attention.mla_attention(rows[:, :512], rows[:, 512:], qn[b][None], qp[b][None], ku, vu, scale, start)[0]
        got = np.einsum("hr,rhd->hd", o_lat[b], vu.reshape(512, heads, dv))
        err = np.abs(got - ref).max() / np.abs(ref).max()
        assert err <= 1e-3, (b, err)


def test_backend_pooled_mla_matches_separate_caches():
    """Decode steps of three requests of an MLA model through one pooled latent-attention
    launch per layer give the greedy tokens of the same requests with separate caches."""
    from ccut_b200.backend import GenericBackend
    from ccut_b200.model import MlaDecoderLayer, MoeDecoder, rope_table
    from tests.model_helpers import MLA_TINY

    t = make_tiny(38, mla=MLA_TINY)
    q = quantized_layers(t, "fp8_b128", seed=38)
    layers = [MlaDecoderLayer(w.ln1, w.wq, w.wkv_a, w.wkv_b, w.wo, w.ln2, gpu_layer(ol.lw), w.kv_norm, heads=w.heads,
                              qk_nope_head_dim=w.d_nope, qk_rope_head_dim=w.d_rope, v_head_dim=w.d_v)
              for w, ol in zip(t.attn, q)]
    inv, af = rope_table(t.rope_dim, t.theta)
    dec = MoeDecoder(t.embed, layers, t.final_norm, t.lm_head, inv_freq=inv, attention_factor=af, eps=t.eps)
    rng = np.random.default_rng(14)
    prompts = [[int(x) for x in rng.integers(0, t.vocab, n)] for n in (9, 30, 3)]
    sep = GenericBackend(dec, max_seqs=3, max_len=128)
    pooled = GenericBackend(dec, max_seqs=3, max_len=128, pool=True)
    a, b = [list(p) for p in prompts], [list(p) for p in prompts]
    for _ in range(4):
        la, lb = sep.logits_batch(a), pooled.logits_batch(b)
        for x, y in zip(la, lb):
            x, y = x.cpu().numpy(), y.cpu().numpy()
            assert np.abs(x - y).max() <= 1e-2 * np.abs(x).max()
        for s, tok in zip(a, sep.generate_batch([(s, {"temperature": 0.0}) for s in a])):
            s.append(tok)
        for s, tok in zip(b, pooled.generate_batch([(s, {"temperature": 0.0}) for s in b])):
            s.append(tok)
    assert a == b
