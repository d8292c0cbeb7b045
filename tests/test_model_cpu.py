"""Decoder stack and engine backend on the CPU: the oracle against the reference's own layer
forward, the sampling transform against the reference's, and the host logic of
``ccut_b200.model`` / ``ccut_b200.backend`` (weight layouts, cache positions, prefix reuse,
errors).

The host-logic tests run ``MoeDecoder`` on CPU tensors with its three device calls (RMSNorm,
RoPE, attention) replaced by short torch functions written here and a torch MoE block; the
product runs those calls through the CUDA library (``tests/test_z_gpu_engine.py``).
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import json

from tests.model_helpers import MLA_TINY, make_tiny, rope_inv_freq
from oracle import model as omodel


# ---- oracle pins --------------------------------------------------------------------------
def _golden_tiny(g, ci):
    qk = str(g[f"m{ci}_qk_norm"])
    return make_tiny(int(g[f"m{ci}_seed"]), norm_topk_prob=bool(g[f"m{ci}_norm"]), qk_norm=None if qk == "none" else qk)


def test_oracle_decoder_matches_reference_layer(golden_dir):
    """oracle.model against the reference's model_forward_layer (ccut/models/generic.py:403-447)
    decoding token by token: hidden state after every layer and the logits of every step."""
    g = np.load(golden_dir / "model_decode.npz")
    for ci in range(2):
        t = _golden_tiny(g, ci)
        spec = t.spec(g[f"m{ci}_inv_freq"])
        cache, ffns = omodel.KvCache(), t.dense_ffns()
        for s, tok in enumerate(g[f"m{ci}_tokens"]):
            lg, hs = omodel.model_forward([tok], t.embed, t.attn, ffns, t.final_norm, t.lm_head, spec, cache, s)
            for i in range(t.layers):
                np.testing.assert_allclose(hs[i][0], g[f"m{ci}_h"][s, i], rtol=1e-5, atol=1e-5)
            np.testing.assert_allclose(lg[0], g[f"m{ci}_logits"][s], rtol=1e-5, atol=1e-5)


def _golden_mla(g, ci):
    return make_tiny(int(g[f"c{ci}_seed"]), norm_topk_prob=bool(g[f"c{ci}_norm"]), mla=json.loads(str(g[f"c{ci}_mla"])))


def test_oracle_mla_decoder_matches_reference_blocks(golden_dir):
    """oracle.model's MLA layer against the reference's MLA blocks assembled into a layer
    (tests/golden/make_golden_mla_model.py): a prefill chunk, single-token steps and a second
    chunk, with and without kv_a_layernorm, with a q_a / q_b pair and an explicit scale."""
    g = np.load(golden_dir / "mla_decoder.npz")
    for ci in range(2):
        t = _golden_mla(g, ci)
        spec = t.spec(g[f"c{ci}_inv_freq"])
        cache, ffns = omodel.KvCache(), t.dense_ffns()
        tokens, pos = g[f"c{ci}_tokens"], 0
        for n in g["chunks"]:
            lg, hs = omodel.model_forward(tokens[pos: pos + n], t.embed, t.attn, ffns, t.final_norm, t.lm_head, spec,
                                          cache, pos)
            for i in range(t.layers):
                np.testing.assert_allclose(hs[i], g[f"c{ci}_h"][pos: pos + n, i], rtol=2e-5, atol=2e-5)
            np.testing.assert_allclose(lg, g[f"c{ci}_logits"][pos: pos + n], rtol=2e-5, atol=2e-5)
            pos += int(n)
        assert cache.k[0].shape == (1, pos, MLA_TINY["rank"]) and cache.v[0].shape == (1, pos, MLA_TINY["d_rope"])


def test_rope_tables_match_reference(golden_dir):
    from ccut_b200.model import rope_table

    g = np.load(golden_dir / "model_decode.npz")
    inv, attn = rope_table(64, 10000.0)
    assert np.array_equal(inv, g["m0_inv_freq"]) and attn == float(g["m0_attn_factor"])
    np.testing.assert_allclose(rope_inv_freq(64, 10000.0), g["m0_inv_freq"], rtol=1e-6)
    lin, _ = rope_table(64, 10000.0, {"type": "linear", "factor": 4.0})
    np.testing.assert_allclose(lin, inv / 4.0, rtol=1e-7)
    # the reference's build_rope for yarn (its own formula), dynamic and linear, bit for bit
    # (tests/golden/rope_tables.npz, made by tests/golden/make_golden_rope.py)
    r = np.load(golden_dir / "rope_tables.npz")
    for i in range(int(r["n"])):
        got, af = rope_table(int(r[f"r{i}_head_dim"]), float(r[f"r{i}_theta"]), json.loads(str(r[f"r{i}_scaling"])))
        assert np.array_equal(got, r[f"r{i}_inv_freq"]) and af == float(r[f"r{i}_attn_factor"]), i
    with pytest.raises(ValueError):
        rope_table(64, 10000.0, {"type": "longrope", "factor": 4.0})


def test_sampling_transform_matches_reference(golden_dir):
    """ccut_b200.sampling.temperature_topk against the reference's (ccut/blocks/heads.py:76-126):
    the same kept tokens and the same probabilities, the top-p edge case included."""
    from ccut_b200.sampling import temperature_topk

    g = np.load(golden_dir / "model_decode.npz")
    for j, (temp, top_k, top_p, min_p) in enumerate(g["samp_params"]):
        ref = g[f"samp{j}_probs"]
        got = temperature_topk(g["samp_logits"], temp, int(top_k), top_p, min_p)
        assert np.array_equal(got > 0, ref > 0), j
        np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-7)
        tg = temperature_topk(torch.from_numpy(g["samp_logits"]), temp, int(top_k), top_p, min_p)
        np.testing.assert_allclose(tg.numpy(), ref, rtol=1e-5, atol=1e-7)


def test_sample_greedy_and_seeded():
    from ccut_b200.sampling import sample

    logits = torch.tensor([0.5, 3.0, 3.0, -1.0])
    assert sample(logits, {"temperature": 0.0}) == 1  # ties to the lowest index
    g1, g2 = torch.Generator().manual_seed(5), torch.Generator().manual_seed(5)
    a = [sample(logits, {"temperature": 1.0, "top_k": 3}, g1) for _ in range(20)]
    b = [sample(logits, {"temperature": 1.0, "top_k": 3}, g2) for _ in range(20)]
    assert a == b and set(a) <= {0, 1, 2}
    assert {sample(logits + torch.tensor([0, 0, -0.1, 0]), {"temperature": 0.7, "top_k": 1}, g1)
            for _ in range(5)} == {1}
    # values equal to the k-th largest stay in (the reference's threshold test is ``x < thr``)
    assert {sample(logits, {"temperature": 0.7, "top_k": 1}, g1) for _ in range(40)} == {1, 2}


# ---- host logic with torch stand-ins for the device calls ---------------------------------
def _norm(x, weight=None, eps=1e-6):
    x32 = x.float()
    y = x32 * torch.rsqrt((x32 * x32).mean(-1, keepdim=True) + eps)
    if weight is not None:
        y = y * weight.float()
    return y.to(torch.bfloat16) if x.dtype == torch.bfloat16 else y


def _rope(q, k, inv_freq, positions, attention_factor=1.0, scaling_type="none", seq_len=0):
    f = positions.float()[:, None, :, None] * inv_freq.float()[None, None, None, :]
    c, s = torch.cos(f), torch.sin(f)

    def rot(x, scale):
        x = x.float() * scale
        h = x.shape[-1] // 2
        return torch.cat([x[..., :h] * c - x[..., h:] * s, x[..., h:] * c + x[..., :h] * s], -1)

    qs = attention_factor if scaling_type in ("yarn", "linear") and attention_factor != 1.0 else 1.0
    return rot(q, qs), rot(k, 1.0)


def _attend(q, k, v, start_pos, softcap):
    _, H, S, d = q.shape
    g = H // k.shape[0]
    L = start_pos + S
    kk = k[:, :L].float().repeat_interleave(g, 0)
    vv = v[:, :L].float().repeat_interleave(g, 0)
    sc = torch.einsum("hsd,hld->hsl", q[0].float(), kk) / math.sqrt(d)
    if softcap:
        sc = torch.tanh(sc / softcap) * softcap
    mask = torch.arange(L)[None, :] > (start_pos + torch.arange(S))[:, None]
    p = torch.softmax(sc.masked_fill(mask, float("-inf")), -1)
    return torch.einsum("hsl,hld->hsd", p, vv)[None].to(torch.bfloat16)


def _mla(q, kv, causal_start, scale):
    """``ccut_mla_attention`` for one sequence: q fp32 [S, H, 576], kv bf16 [n, 576] -> the
    latent output [S * H, 512]."""
    S, H, _ = q.shape
    n = kv.shape[0]
    kvf = kv.float()
    sc = torch.einsum("shk,nk->shn", q.float(), kvf) * scale
    vis = torch.full((S,), n) if causal_start < 0 else torch.clamp(causal_start + torch.arange(S) + 1, max=n)
    mask = torch.arange(n)[None, :] >= vis[:, None]
    p = torch.softmax(sc.masked_fill(mask[:, None, :], float("-inf")), -1)
    return torch.einsum("shn,nr->shr", p, kvf[:, :512]).reshape(S * H, 512)


def _mla_pool(q, pool, layer, slots, starts, scale):
    """``ccut_mla_attention_pool``: row b over its slot's latent rows ``<= starts[b]`` (zero
    rows for a slot outside the pool or a negative start)."""
    outs = []
    for b in range(q.shape[0]):
        slot, st = int(slots[b]), int(starts[b])
        if not (0 <= slot < pool.slots and st >= 0):
            outs.append(torch.zeros((q.shape[1], 512)))
            continue
        outs.append(_mla(q[b:b + 1], pool.k[slot, layer, 0, : st + 1], st, scale))
    return torch.cat(outs)


class _TorchMoe:
    """MoE block with the tiny model's dense experts (softmax routing as the reference)."""

    def __init__(self, t, i):
        self.router = torch.from_numpy(t.router[i])
        self.experts = [tuple(torch.from_numpy(m) for m in e) for e in t.experts[i]]
        self.shared = tuple(torch.from_numpy(m) for m in t.shared[i]) if t.shared[i] is not None else None
        self.k, self.norm = t.top_k, t.norm_topk_prob
        self.calls = []

    def _mlp(self, x, wg, wu, wd):
        gt = x @ wg
        return (gt / (1 + torch.exp(-gt)) * (x @ wu)) @ wd

    def forward(self, x, out_dtype=torch.bfloat16):
        assert x.dtype == torch.bfloat16 and x.dim() == 2
        self.calls.append(x.shape[0])
        xf = x.float()
        lg = xf @ self.router.T
        if self.norm:
            vals, ids = torch.topk(lg, self.k, dim=1)
            w = torch.softmax(vals, 1)
        else:
            w, ids = torch.topk(torch.softmax(lg, 1), self.k, dim=1)
        out = torch.zeros_like(xf)
        for t in range(x.shape[0]):
            for j in range(self.k):
                out[t] += w[t, j] * self._mlp(xf[t:t + 1], *self.experts[int(ids[t, j])])[0]
        if self.shared is not None:
            out += self._mlp(xf, *self.shared)
        return out.to(out_dtype)


@pytest.fixture
def torch_ops(monkeypatch):
    import ccut_b200.model as m

    monkeypatch.setattr(m, "rms_norm", _norm)
    monkeypatch.setattr(m, "apply_rope", _rope)
    monkeypatch.setattr(m, "_attend", _attend)
    monkeypatch.setattr(m, "_mla_attend", _mla)
    monkeypatch.setattr(m, "_mla_attend_pool", _mla_pool)
    return m


def _build(m, t, **kw):
    layers = [m.DecoderLayer(w.ln1, w.wq, w.wk, w.wv, w.wo, w.ln2, _TorchMoe(t, i), w.q_norm, w.k_norm, heads=t.heads,
                             kv_heads=t.kv_heads, head_dim=t.head_dim, device="cpu") for i, w in enumerate(t.attn)]
    inv, attn = m.rope_table(t.head_dim, t.theta)
    return m.MoeDecoder(t.embed, layers, t.final_norm, t.lm_head, inv_freq=inv, attention_factor=attn, eps=t.eps,
                        device="cpu", **kw)


def _mla_layers(m, t, ffns=None):
    return [m.MlaDecoderLayer(w.ln1, w.wq, w.wkv_a, w.wkv_b, w.wo, w.ln2, ffns[i] if ffns else _TorchMoe(t, i),
                              w.kv_norm, heads=w.heads, qk_nope_head_dim=w.d_nope, qk_rope_head_dim=w.d_rope,
                              v_head_dim=w.d_v, q_a=w.wq_a, q_a_norm=w.q_a_norm, softmax_scale=w.scale, device="cpu")
            for i, w in enumerate(t.attn)]


def _build_mla(m, t, **kw):
    inv, attn = m.rope_table(t.rope_dim, t.theta)
    return m.MoeDecoder(t.embed, _mla_layers(m, t), t.final_norm, t.lm_head, inv_freq=inv, attention_factor=attn,
                        eps=t.eps, device="cpu", **kw)


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-12))


@pytest.mark.parametrize("kv_heads, qk_norm", [(1, "flat"), (2, "head"), (4, None)])
def test_decoder_host_logic_matches_oracle(torch_ops, kv_heads, qk_norm):
    """Prefill of 5 tokens, then 3 single-token steps and a 2-token chunk: logits of every
    position against the oracle's decoder (bf16 at the same points)."""
    m = torch_ops
    t = make_tiny(21, kv_heads=kv_heads, qk_norm=qk_norm, norm_topk_prob=kv_heads == 2)
    dec = _build(m, t)
    cache = dec.new_cache(32)
    spec, ocache, ffns = t.spec(), omodel.KvCache(), t.dense_ffns()
    rng = np.random.default_rng(3)
    pos = 0
    for n in (5, 1, 1, 1, 2):
        toks = rng.integers(0, t.vocab, n)
        got = dec.forward(toks, cache, all_logits=True)
        ref, _ = omodel.model_forward(toks, t.embed, t.attn, ffns, t.final_norm, t.lm_head, spec, ocache, pos,
                                      bf16_acts=True)
        assert got.shape == (n, t.vocab) and _rel(got.numpy(), ref) < 5e-3
        pos += n
        assert cache.length == pos
        last = dec.forward(toks[-1:], cache, start_pos=pos - 1)  # recompute the last position
        assert last.shape == (t.vocab,) and _rel(last.numpy(), ref[-1]) < 5e-3
    # a wrong position (one past) changes the logits: the comparison above is position-sensitive
    c2 = dec.new_cache(32)
    dec.forward([3, 9], c2)
    c3 = dec.new_cache(32)
    dec.forward([3, 3, 9], c3)
    assert _rel(dec.forward([5], c2).numpy(), dec.forward([5], c3).numpy()) > 1e-3


def test_decoder_checks(torch_ops):
    m = torch_ops
    t = make_tiny(22)
    dec = _build(m, t)
    cache = dec.new_cache(4)
    with pytest.raises(ValueError):
        dec.forward([], cache)
    with pytest.raises(ValueError):
        dec.forward([1, 2, 3, 4, 5], cache)  # past max_len
    with pytest.raises(ValueError):
        dec.forward([t.vocab], cache)
    with pytest.raises(ValueError):
        dec.forward([1], cache, start_pos=1)  # past the cached positions
    dec.forward([1, 2], cache)
    cache.truncate(1)
    with pytest.raises(ValueError):
        cache.truncate(2)
    w = t.attn[0]
    kw = dict(heads=t.heads, kv_heads=t.kv_heads, head_dim=t.head_dim, device="cpu")
    with pytest.raises(NotImplementedError):
        m.DecoderLayer(w.ln1, w.wq, w.wk, w.wv, w.wo, w.ln2, None, **{**kw, "head_dim": 96})
    with pytest.raises(ValueError):
        m.DecoderLayer(w.ln1, w.wq, w.wk.T, w.wv, w.wo, w.ln2, None, **kw)  # [in, out] by mistake
    with pytest.raises(ValueError):
        m.DecoderLayer(w.ln1, w.wq, w.wk, w.wv, w.wo, w.ln2, None, q_norm=np.ones(3), **kw)
    with pytest.raises(ValueError):
        m.DecoderLayer(w.ln1, w.wq, w.wk, w.wv, w.wo, w.ln2, None, **{**kw, "kv_heads": 3})
    with pytest.raises(ValueError):
        m.MoeDecoder(t.embed, [], t.final_norm, t.lm_head, inv_freq=np.ones(32), device="cpu")
    with pytest.raises(ValueError):
        m.MoeDecoder(t.embed, dec.layers, t.final_norm, t.lm_head, inv_freq=np.ones(31), device="cpu")


def test_backend_prefix_reuse(torch_ops):
    """generate_step as Engine._backend_step calls it (ccut/engine.py:305-333): a request grown
    one token per step runs one position per step; chunked prefill runs each chunk once; a
    diverging request reuses the shared prefix; the least recently used cache is evicted."""
    from ccut_b200.backend import GenericBackend, common_prefix

    m = torch_ops
    t = make_tiny(23)
    be = GenericBackend(_build(m, t), max_seqs=2, max_len=64, prefill_chunk=4)
    prompt = [5, 9, 13, 2, 8, 1, 4]
    ref = be.model.forward(prompt, be.model.new_cache(64))
    assert be.tokens_run == 0
    np.testing.assert_allclose(be.logits_for(prompt).numpy(), ref.numpy(), rtol=1e-5, atol=1e-5)
    assert be.tokens_run == 7
    ids = list(prompt)
    for step in range(3):
        ids.append(be.generate_step(ids, {"temperature": 0.0}))
        assert be.tokens_run == 8 + step
    full = be.model.forward(ids, be.model.new_cache(64))
    np.testing.assert_allclose(be.logits_for(ids).numpy(), full.numpy(), rtol=2e-2, atol=2e-2)
    assert be.tokens_run == 11  # the last position again, for its logits
    # a request sharing the first 4 prompt tokens with the cached one
    other = prompt[:4] + [30, 31]
    be.logits_for(other)
    assert be.tokens_run == 11 + 2
    # engine-style chunked prefill: the ids grow by chunks
    before = be.tokens_run
    long = list(range(40, 52))
    for n in (4, 8, 12):
        be.logits_for(long[:n])
    assert be.tokens_run - before == 4 + 4 + 4
    assert len(be._seqs) == 2
    assert common_prefix([1, 2, 3], [1, 2, 4, 5]) == 2 and common_prefix([1], [1, 2]) == 1
    assert common_prefix([], [3]) == 0
    with pytest.raises(ValueError):
        be.generate_step([], {})
    with pytest.raises(ValueError):
        be.generate_step(list(range(65)), {})


def test_backend_l1_interface(torch_ops):
    """forward_step / generate with the reference L1Backend's signatures
    (ccut/models/backend_transformers.py:75-124): greedy by default, stops at eos."""
    from ccut_b200.backend import GenericBackend

    m = torch_ops
    t = make_tiny(24)
    be = GenericBackend(_build(m, t), max_len=32)
    prompt = [3, 1, 4, 1, 5]
    out = be.generate(prompt, 4)
    ids = list(prompt)
    for _ in range(4):
        ids.append(be.generate_step(ids, {"temperature": 0.0}))
    assert out == ids[len(prompt):]
    seen = []
    be.eos_token_id = out[1]
    assert be.generate(prompt, 4, on_token=seen.append) == out[:2] and seen == out[:2]
    calls = []
    be.eos_token_id = None
    be.generate(prompt, 2, sampling=lambda lg, pos: calls.append((tuple(lg.shape), pos)) or 0)
    assert calls == [((1, t.vocab), 0), ((1, t.vocab), 1)]
    logits, past = be.forward_step(prompt)
    assert logits.shape == (1, t.vocab) and past.length == len(prompt)


def test_decoder_batch_matches_single_sequences(torch_ops):
    """forward_batch (one pass over several sequences, attention per sequence) against the same
    sequences run one at a time."""
    m = torch_ops
    t = make_tiny(25, kv_heads=2, qk_norm="head")
    dec = _build(m, t)
    rng = np.random.default_rng(8)
    prompts = [rng.integers(0, t.vocab, n) for n in (6, 1, 9)]
    singles, caches = [], []
    for p in prompts:
        c = dec.new_cache(32)
        singles.append(dec.forward(p, c, all_logits=True))
        caches.append(c)
    bcaches = [dec.new_cache(32) for _ in prompts]
    got = dec.forward_batch([(p, c, None) for p, c in zip(prompts, bcaches)], all_logits=True)
    for g, s in zip(got, singles):
        assert g.shape == s.shape and _rel(g.numpy(), s.numpy()) < 5e-3
    # one more token each, from different positions; last-token logits only
    nxt = [[int(x)] for x in rng.integers(0, t.vocab, 3)]
    got = dec.forward_batch([(n, c, None) for n, c in zip(nxt, bcaches)])
    for n, c, g in zip(nxt, caches, got):
        assert g.shape == (t.vocab,) and _rel(g.numpy(), dec.forward(n, c).numpy()) < 5e-3
    assert [c.length for c in bcaches] == [7, 2, 10]
    with pytest.raises(ValueError):
        dec.forward_batch([([1], bcaches[0], None), ([2], bcaches[0], None)])  # one cache twice
    assert dec.forward_batch([]) == []


def test_backend_generate_batch(torch_ops):
    """generate_batch (one engine step for several requests in one pass) picks the tokens that
    generate_step picks for each request alone, runs each prompt once and then one position
    per request per step."""
    from ccut_b200.backend import GenericBackend

    m = torch_ops
    t = make_tiny(26)
    dec = _build(m, t)
    prompts = [[4, 8, 15, 16, 23, 42], [7, 7, 7], [1, 2, 3, 4, 5, 6, 7, 8, 9, 10]]
    solo = GenericBackend(dec, max_seqs=1, max_len=32)
    want = []
    for p in prompts:
        ids = list(p)
        for _ in range(3):
            ids.append(solo.generate_step(ids, {"temperature": 0.0}))
        want.append(ids)
    be = GenericBackend(dec, max_seqs=3, max_len=32, prefill_chunk=4)
    seqs = [list(p) for p in prompts]
    for step in range(3):
        before = be.tokens_run
        toks = be.generate_batch([(s, {"temperature": 0.0}) for s in seqs])
        for s, tok in zip(seqs, toks):
            s.append(tok)
        assert be.tokens_run - before == (sum(map(len, prompts)) if step == 0 else 3)
    assert seqs == want
    with pytest.raises(ValueError):
        be.generate_batch([([1], {}), ([2], {}), ([3], {}), ([4], {})])  # more than max_seqs


def test_temperature_topk_constraints_like_reference():
    """The property the reference's own test checks (tests/test_blocks.py,
    test_temperature_topk_constraints): with top_k=5, top_p=0.9 and min_p=0.05 at most five
    tokens keep probability and every row sums to one."""
    from ccut_b200.sampling import temperature_topk

    lg = np.random.default_rng(6).standard_normal((3, 100)).astype(np.float32)
    p = temperature_topk(lg, 1.0, top_k=5, top_p=0.9, min_p=0.05)
    assert ((p > 0).sum(axis=1) <= 5).all()
    np.testing.assert_allclose(p.sum(axis=1), 1.0, atol=1e-5)


class _TorchProj:
    """A projection object ([out, in] weight, fp32 out), as ``quant.QuantLinear`` is one."""

    def __init__(self, w):
        self.w = torch.from_numpy(np.ascontiguousarray(w, np.float32))
        self.out_features, self.in_features = self.w.shape

    def __call__(self, x):
        return x.float() @ self.w.T


@pytest.mark.parametrize("which", ["all", "kv_only"])
def test_decoder_with_projection_objects(torch_ops, which):
    """Projections given as objects (fp32 outputs, as the quantized ones give): all four, or
    k / v only next to bf16 q / o weights (the mixed q / k / v path)."""
    m = torch_ops
    t = make_tiny(27, kv_heads=2, qk_norm="head")
    layers = []
    for i, w in enumerate(t.attn):
        wq, wk, wv, wo = w.wq, _TorchProj(w.wk), _TorchProj(w.wv), w.wo
        if which == "all":
            wq, wo = _TorchProj(w.wq), _TorchProj(w.wo)
        layers.append(m.DecoderLayer(w.ln1, wq, wk, wv, wo, w.ln2, _TorchMoe(t, i), w.q_norm, w.k_norm,
                                     heads=t.heads, kv_heads=t.kv_heads, head_dim=t.head_dim, device="cpu"))
    inv, attn = m.rope_table(t.head_dim, t.theta)
    dec = m.MoeDecoder(t.embed, layers, t.final_norm, t.lm_head, inv_freq=inv, attention_factor=attn, eps=t.eps,
                       device="cpu")
    cache, ocache = dec.new_cache(16), omodel.KvCache()
    rng = np.random.default_rng(4)
    pos = 0
    for n in (6, 1, 2):
        toks = rng.integers(0, t.vocab, n)
        got = dec.forward(toks, cache, all_logits=True)
        ref, _ = omodel.model_forward(toks, t.embed, t.attn, t.dense_ffns(), t.final_norm, t.lm_head, t.spec(),
                                      ocache, pos, bf16_acts=True)
        assert _rel(got.numpy(), ref) < 1e-2
        pos += n
    with pytest.raises(ValueError):  # a projection object of the wrong shape
        w = t.attn[0]
        m.DecoderLayer(w.ln1, _TorchProj(w.wk), w.wk, w.wv, w.wo, w.ln2, None, heads=t.heads, kv_heads=t.kv_heads,
                       head_dim=t.head_dim, device="cpu")


def _attend_pool(q, pool, layer, slots, starts, softcap):
    """Torch stand-in of the pooled attention: row b over its slot's positions <= starts[b] + i."""
    outs = []
    for b in range(q.shape[0]):
        slot, st = int(slots[b]), int(starts[b])
        outs.append(_attend(q[b:b + 1], pool.k[slot, layer], pool.v[slot, layer], st, softcap)[0])
    return torch.stack(outs)


def test_backend_pooled_caches_match(torch_ops, monkeypatch):
    """Caches in one KvPool (a decode step of several requests is one attention call per layer):
    the same tokens as separate caches, the decode steps through the pooled call with every
    request at once, slots reused after eviction, and two views of one slot refused."""
    from ccut_b200.backend import GenericBackend

    m = torch_ops
    calls = []

    def pooled(*a):
        calls.append(a[0].shape[0])
        return _attend_pool(*a)

    monkeypatch.setattr(m, "_attend_pool", pooled)
    t = make_tiny(28, kv_heads=2, qk_norm="head")
    dec = _build(m, t)
    prompts = [[4, 8, 15, 16], [23, 42], [7, 1, 7, 1, 7, 1]]
    ref = GenericBackend(dec, max_seqs=3, max_len=32)
    be = GenericBackend(dec, max_seqs=3, max_len=32, pool=True)
    a, b = [list(p) for p in prompts], [list(p) for p in prompts]
    for _ in range(3):
        for s, tok in zip(a, ref.generate_batch([(s, {"temperature": 0.0}) for s in a])):
            s.append(tok)
        for s, tok in zip(b, be.generate_batch([(s, {"temperature": 0.0}) for s in b])):
            s.append(tok)
    assert a == b
    assert calls and set(calls) == {3}
    assert sorted(s.cache.slot for s in be._seqs) == [0, 1, 2]
    np.testing.assert_allclose(be.logits_for(b[0]).numpy(), ref.logits_for(a[0]).numpy(), rtol=5e-3, atol=5e-3)
    be.logits_for([9, 9, 9])  # a new request takes the least recently used slot
    assert sorted(s.cache.slot for s in be._seqs) == [0, 1, 2]
    with pytest.raises(ValueError):
        dec.forward_batch([([1], be._pool.cache(1), None), ([2], be._pool.cache(1), None)])
    with pytest.raises(ValueError):
        be._pool.cache(3)


MLA_VARIANTS = [{}, {"kv_norm": False}, {"q_rank": 128, "scale": 0.09}]


@pytest.mark.parametrize("extra", MLA_VARIANTS)
def test_mla_decoder_host_logic_matches_oracle(torch_ops, extra):
    """MLA layers (DeepSeek-V2 / V3 latent attention) in MoeDecoder: a 5-token prefill, single
    steps, a 2-token chunk and a recomputed last position against the oracle's MLA decoder
    (bf16 at the same points); the cache holds one [c, k_pe] row per position, no values."""
    m = torch_ops
    t = make_tiny(41, mla={**MLA_TINY, **extra}, norm_topk_prob=bool(extra))
    dec = _build_mla(m, t)
    cache = dec.new_cache(32)
    assert cache.v is None and tuple(cache.k.shape) == (t.layers, 1, 32, 576)
    spec, ocache, ffns = t.spec(), omodel.KvCache(), t.dense_ffns()
    rng = np.random.default_rng(4)
    pos = 0
    for n in (5, 1, 1, 2):
        toks = rng.integers(0, t.vocab, n)
        got = dec.forward(toks, cache, all_logits=True)
        ref, _ = omodel.model_forward(toks, t.embed, t.attn, ffns, t.final_norm, t.lm_head, spec, ocache, pos,
                                      bf16_acts=True)
        assert got.shape == (n, t.vocab) and _rel(got.numpy(), ref) < 5e-3
        pos += n
        assert cache.length == pos
        # the cached latent rows are the oracle's c and rotated k_pe, in bf16
        np.testing.assert_allclose(cache.k[0, 0, :pos, :512].float().numpy(), ocache.k[0][0], rtol=1e-2, atol=1e-2)
        np.testing.assert_allclose(cache.k[0, 0, :pos, 512:].float().numpy(), ocache.v[0][0], rtol=1e-2, atol=1e-2)
        last = dec.forward(toks[-1:], cache, start_pos=pos - 1)
        assert _rel(last.numpy(), ref[-1]) < 5e-3


def test_mla_decoder_batch_and_backend(torch_ops, monkeypatch):
    """forward_batch over MLA caches equals the sequences run alone; the backend's prefix reuse
    runs on MLA caches; with pooled latent caches a decode step of several requests is one
    pooled attention call per layer and generates the same tokens."""
    from ccut_b200.backend import GenericBackend

    m = torch_ops
    calls = []

    def pooled(*a):
        calls.append(a[0].shape[0])
        return _mla_pool(*a)

    monkeypatch.setattr(m, "_mla_attend_pool", pooled)
    t = make_tiny(42, mla=MLA_TINY)
    dec = _build_mla(m, t)
    rng = np.random.default_rng(9)
    prompts = [rng.integers(0, t.vocab, n) for n in (4, 1, 7)]
    singles = [dec.forward(p, dec.new_cache(16), all_logits=True) for p in prompts]
    got = dec.forward_batch([(p, dec.new_cache(16), None) for p in prompts], all_logits=True)
    for g, s in zip(got, singles):
        assert _rel(g.numpy(), s.numpy()) < 5e-3
    be = GenericBackend(dec, max_seqs=2, max_len=32)
    prompt = [7, 3, 11, 5]
    ids = list(prompt)
    for _ in range(3):
        ids.append(be.generate_step(ids, {"temperature": 0.0}))
    assert be.tokens_run == 4 + 2
    full = dec.forward(ids, dec.new_cache(32))
    assert _rel(be.logits_for(ids).numpy(), full.numpy()) < 2e-2
    ref = GenericBackend(dec, max_seqs=3, max_len=32)
    bp = GenericBackend(dec, max_seqs=3, max_len=32, pool=True)
    assert bp._pool.v is None and tuple(bp._pool.k.shape) == (3, t.layers, 1, 32, 576)
    a = [[int(x) for x in p] for p in prompts]
    b = [list(s) for s in a]
    for _ in range(3):
        for s, tok in zip(a, ref.generate_batch([(s, {"temperature": 0.0}) for s in a])):
            s.append(tok)
        for s, tok in zip(b, bp.generate_batch([(s, {"temperature": 0.0}) for s in b])):
            s.append(tok)
    assert a == b
    assert calls and set(calls) == {3} and len(calls) == 2 * t.layers  # two decode steps after the prefill


def test_mla_decoder_checks(torch_ops):
    m = torch_ops
    t = make_tiny(43, mla=MLA_TINY)
    w = t.attn[0]
    kw = dict(heads=w.heads, qk_nope_head_dim=w.d_nope, qk_rope_head_dim=w.d_rope, v_head_dim=w.d_v, device="cpu")
    args = (w.ln1, w.wq, w.wkv_a, w.wkv_b, w.wo, w.ln2, None, w.kv_norm)
    with pytest.raises(NotImplementedError):
        m.MlaDecoderLayer(*args, **{**kw, "kv_lora_rank": 256})
    with pytest.raises(NotImplementedError):
        m.MlaDecoderLayer(*args, **{**kw, "qk_rope_head_dim": 32})
    with pytest.raises(ValueError):
        m.MlaDecoderLayer(w.ln1, w.wq, w.wkv_a, w.wkv_b.T, w.wo, w.ln2, None, **kw)  # kv_b_proj transposed
    with pytest.raises(ValueError):
        m.MlaDecoderLayer(w.ln1, w.wq, w.wkv_a.T, w.wkv_b, w.wo, w.ln2, None, **kw)
    with pytest.raises(ValueError):
        m.MlaDecoderLayer(*args, **{**kw, "v_head_dim": w.d_v + 1})
    with pytest.raises(ValueError):
        m.MlaDecoderLayer(w.ln1, w.wq, w.wkv_a, w.wkv_b, w.wo, w.ln2, None, np.ones(3), **kw)
    with pytest.raises(ValueError):
        m.MlaDecoderLayer(*args, q_a=np.ones((128, t.hidden)), **kw)  # q_a without its norm
    with pytest.raises(ValueError):
        m.MlaDecoderLayer(*args, softmax_scale=0.0, **kw)
    dec = _build_mla(m, t)
    pool = dec.new_pool(2, 16)
    assert pool.v is None and pool.cache(1).v is None and tuple(pool.cache(1).k.shape) == (t.layers, 1, 16, 576)
    inv, _ = m.rope_table(64, t.theta)
    with pytest.raises(NotImplementedError):
        m.MoeDecoder(t.embed, dec.layers, t.final_norm, t.lm_head, inv_freq=inv, softcap=30.0, device="cpu")
    with pytest.raises(ValueError):
        m.MoeDecoder(t.embed, dec.layers, t.final_norm, t.lm_head, inv_freq=np.ones(64), device="cpu")
    g = make_tiny(44, head_dim=64)
    gqa = _build(m, g).layers[0]
    with pytest.raises(ValueError):  # one cache layout per model
        m.MoeDecoder(t.embed, [dec.layers[0], gqa], t.final_norm, t.lm_head, inv_freq=inv, device="cpu")
