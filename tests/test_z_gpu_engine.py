"""The decoder stack and the engine backend on the GPU (``ccut_b200.model``,
``ccut_b200.backend``) against the oracle's decoder (``oracle.model``, pinned to the
reference's own layer forward, ``ccut/models/generic.py:304-447``).

The oracle runs with bf16 at the points where the GPU path stores bf16 and with the
dequantized experts of the same AWQ / FP8 layers.  Its MoE blocks take the expert ids and
weights that the GPU chose for the same call (recorded by ``_Recorded``), after checking that
they are the oracle's own choice except where the oracle's k-th and (k+1)-th router logits lie
within ``NEAR_TIE`` (the two sides' inputs differ by bf16 roundings, so a near tie may break
either way, and a different expert changes that token's output outright).  Tolerance: max over
positions of ``max|logits - ref| / max|ref|`` <= ``LOGITS_TOL``; the MoE layers alone are held to
1e-2 by the kernel tests.  The caches are much longer than the positions in use, so the
attention kernel clips every kv split to the causal range.
"""

from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch

from ccut_b200 import dense
from ccut_b200.backend import GenericBackend
from ccut_b200.checkpoint import load_decoder, load_decoder_weights
from ccut_b200.model import DecoderLayer, MlaDecoderLayer, MoeDecoder, rope_table
from oracle import inputs, moe, routing
from oracle import model as omodel
from tests.ckpt_helpers import write_decoder_checkpoint
from tests.deepseek_helpers import DS_CASES, oracle_decoder, write_deepseek_checkpoint
from tests.gpu_helpers import gpu_layer
from tests.model_helpers import MLA_TINY, make_tiny, quantized_attention, quantized_layers

pytestmark = pytest.mark.gpu

LOGITS_TOL = 3e-2
NEAR_TIE = 5e-3


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from ccut_b200 import build
    build.build()


def _rel_rows(a, b) -> float:
    a, b = np.atleast_2d(np.asarray(a, np.float64)), np.atleast_2d(np.asarray(b, np.float64))
    return float((np.abs(a - b).max(axis=1) / np.maximum(np.abs(b).max(axis=1), 1e-30)).max())


class _Recorded:
    """A ``MoeLayer`` that keeps the routing of every call (ids int64, weights fp32)."""

    def __init__(self, layer):
        self.layer = layer
        self.routes: list = []

    def forward(self, x, out_dtype=torch.bfloat16):
        out, r = self.layer.forward(x, out_dtype, return_routing=True)
        self.routes.append((r.ids.cpu().numpy().astype(np.int64), r.weights.cpu().numpy()))
        return out

    def workspace_status(self) -> int:
        return self.layer.workspace_status()


def _oracle_moe(ol, top_k: int, mode: str, rec: _Recorded):
    """Oracle MoE block on the GPU's routing of the same call (oldest recorded first)."""

    def f(x):
        ids, w = rec.routes.pop(0)
        assert ids.shape == (x.shape[0], top_k)
        lg = x @ ol.router.T
        _, own = routing.route(lg, top_k, mode)
        s = np.sort(lg, axis=1)[:, ::-1]
        for t in range(x.shape[0]):
            if set(ids[t].tolist()) != set(own[t].tolist()):
                assert s[t, top_k - 1] - s[t, top_k] < NEAR_TIE, f"token {t}: {ids[t]} vs {own[t]}"
        return moe.moe_forward(x, ol.router, top_k, mode, ol.w_lookup, ol.shared_cat(), ids=ids, weights=w)[0]

    return f


def _decoder(t, ffns):
    layers = [DecoderLayer(w.ln1, w.wq, w.wk, w.wv, w.wo, w.ln2, f, w.q_norm, w.k_norm, heads=t.heads,
                           kv_heads=t.kv_heads, head_dim=t.head_dim) for w, f in zip(t.attn, ffns)]
    inv, attn = rope_table(t.head_dim, t.theta)
    return MoeDecoder(t.embed, layers, t.final_norm, t.lm_head, inv_freq=inv, attention_factor=attn, eps=t.eps)


def _moe_model(t, fmt: str, seed: int):
    qlayers = quantized_layers(t, fmt, seed=seed)
    recs = [_Recorded(gpu_layer(ol.lw)) for ol in qlayers]
    offs = [_oracle_moe(ol, t.top_k, t.mode, r) for ol, r in zip(qlayers, recs)]
    return _decoder(t, recs), recs, offs


# fmt, kv_heads, qk_norm, head_dim, model seed, token seed
CASES = [("fp8_b128", 2, "head", 64, 31, 5), ("awq_int4_g128", 1, "flat", 128, 32, 6)]


@pytest.mark.parametrize("fmt, kv_heads, qk_norm, head_dim, seed, tseed", CASES)
def test_decoder_matches_oracle(fmt, kv_heads, qk_norm, head_dim, seed, tseed):
    """A 37-token prefill, four single-token steps and a 20-token chunk through two layers
    (GQA or MQA attention, q / k norm per head or over the projection, a MoE block with a
    shared expert): the logits of every position."""
    t = make_tiny(seed, kv_heads=kv_heads, qk_norm=qk_norm, head_dim=head_dim)
    dec, recs, offs = _moe_model(t, fmt, seed)
    cache = dec.new_cache(1024)
    spec, ocache = t.spec(), omodel.KvCache()
    rng = np.random.default_rng(tseed)
    pos = 0
    for n in (37, 1, 1, 1, 1, 20):
        toks = rng.integers(0, t.vocab, n)
        got = dec.forward(toks, cache, all_logits=True)
        torch.cuda.synchronize()
        assert got.shape == (n, t.vocab) and got.dtype == torch.float32 and cache.length == pos + n
        ref, _ = omodel.model_forward(toks, t.embed, t.attn, offs, t.final_norm, t.lm_head, spec, ocache, pos,
                                      bf16_acts=True)
        err = _rel_rows(got.cpu().numpy(), ref)
        assert err <= LOGITS_TOL, (n, pos, err)
        pos += n
    assert all(not r.routes for r in recs)
    for r in recs:
        assert r.workspace_status() == 0


@pytest.mark.parametrize("fmt, extra, seed", [("awq_int4_g128", {}, 35),
                                              ("fp8_b128", {"q_rank": 128, "kv_norm": False}, 36)])
def test_mla_decoder_matches_oracle(fmt, extra, seed):
    """MLA layers (``MlaDecoderLayer``: latent cache rows, ``ccut_mla_attention`` between the
    ``k_up`` / ``v_up`` GEMMs) with quantized MoE blocks: a 37-token prefill, four single-token
    steps and a 20-token chunk, the logits of every position against the oracle's MLA decoder
    (pinned to the reference's MLA blocks)."""
    t = make_tiny(seed, mla={**MLA_TINY, **extra})
    qlayers = quantized_layers(t, fmt, seed=seed)
    recs = [_Recorded(gpu_layer(ol.lw)) for ol in qlayers]
    offs = [_oracle_moe(ol, t.top_k, t.mode, r) for ol, r in zip(qlayers, recs)]
    layers = [MlaDecoderLayer(w.ln1, w.wq, w.wkv_a, w.wkv_b, w.wo, w.ln2, r, w.kv_norm, heads=w.heads,
                              qk_nope_head_dim=w.d_nope, qk_rope_head_dim=w.d_rope, v_head_dim=w.d_v, q_a=w.wq_a,
                              q_a_norm=w.q_a_norm, softmax_scale=w.scale) for w, r in zip(t.attn, recs)]
    inv, attn = rope_table(t.rope_dim, t.theta)
    dec = MoeDecoder(t.embed, layers, t.final_norm, t.lm_head, inv_freq=inv, attention_factor=attn, eps=t.eps)
    cache = dec.new_cache(512)
    spec, ocache = t.spec(), omodel.KvCache()
    rng = np.random.default_rng(seed + 100)
    pos = 0
    for n in (37, 1, 1, 1, 1, 20):
        toks = rng.integers(0, t.vocab, n)
        got = dec.forward(toks, cache, all_logits=True)
        torch.cuda.synchronize()
        assert got.shape == (n, t.vocab) and cache.length == pos + n
        ref, _ = omodel.model_forward(toks, t.embed, t.attn, offs, t.final_norm, t.lm_head, spec, ocache, pos,
                                      bf16_acts=True)
        err = _rel_rows(got.cpu().numpy(), ref)
        assert err <= LOGITS_TOL, (n, pos, err)
        pos += n
    assert all(not r.routes for r in recs)
    # a batch of two sequences (their MoE tokens together) equals each run alone
    be = GenericBackend(dec, max_seqs=2, max_len=128)
    a, b = [int(x) for x in rng.integers(0, t.vocab, 9)], [int(x) for x in rng.integers(0, t.vocab, 3)]
    for r in recs:
        r.routes.clear()
    got = be.logits_batch([a, b])
    for ids, g in zip((a, b), got):
        alone = dec.forward(ids, dec.new_cache(128))
        assert _rel_rows(g.cpu().numpy(), alone.cpu().numpy()) <= LOGITS_TOL


def test_decoder_with_dense_layer():
    """A dense FFN layer (``DenseFfn``, the expert kernels with one expert) before a MoE layer,
    as in models whose first layers are dense."""
    t = make_tiny(33, kv_heads=2, qk_norm=None)
    qlayers = quantized_layers(t, "fp8_b128", seed=33)
    dl = inputs.make_layer(inputs.scaled_config("cfg1", hidden=t.hidden, inter=256, num_experts=1, top_k=1,
                                                num_shared=0), seed=34)
    de = dl.experts[0]
    dff = dense.DenseFfn("fp8_b128", t.hidden, 256, de.gate, de.up, de.down)
    wg, wu, wd = dl.w_lookup(0)
    rec = _Recorded(gpu_layer(qlayers[1].lw))
    offs = [lambda x: moe.expert_ffn(x, wg, wu, wd), _oracle_moe(qlayers[1], t.top_k, t.mode, rec)]
    dec = _decoder(t, [dff, rec])
    cache, ocache = dec.new_cache(256), omodel.KvCache()
    rng = np.random.default_rng(9)
    pos = 0
    for n in (12, 1, 1):
        toks = rng.integers(0, t.vocab, n)
        got = dec.forward(toks, cache, all_logits=True)
        ref, _ = omodel.model_forward(toks, t.embed, t.attn, offs, t.final_norm, t.lm_head, t.spec(), ocache, pos,
                                      bf16_acts=True)
        assert _rel_rows(got.cpu().numpy(), ref) <= LOGITS_TOL
        pos += n
    assert dff.workspace_status() == 0


def test_backend_generate_step():
    """``generate_step`` as the reference's Engine calls it (the whole id list every step,
    ``ccut/engine.py:305-333``): a 40-token prompt run in 16-token prefill chunks, then six
    greedy steps that each run one new position.  Every step's logits equal a fresh prefill of
    the same ids, the greedy token is their arg-max, and the logits of the final ids at every
    position match the oracle."""
    t = make_tiny(35, kv_heads=2, qk_norm="head")
    dec, recs, offs = _moe_model(t, "fp8_b128", 35)
    be = GenericBackend(dec, max_seqs=2, max_len=512, prefill_chunk=16)
    ids = [int(x) for x in np.random.default_rng(11).integers(0, t.vocab, 40)]
    for step in range(6):
        got = be.logits_for(ids).cpu().numpy()
        fresh = dec.forward(ids, dec.new_cache(512)).cpu().numpy()
        assert _rel_rows(got, fresh) <= LOGITS_TOL, step
        tok = be.generate_step(ids, {"temperature": 0.0})
        assert got[tok] >= got.max() - 1e-3 * np.abs(got).max(), step
        ids.append(tok)
    assert be.tokens_run == 40 + 6 * 2 - 1  # the prompt once, then per step the newest id and a recompute
    top5 = set(np.argsort(-be.logits_for(ids).cpu().numpy())[:5].tolist())
    assert {be.generate_step(ids, {"temperature": 1.0, "top_k": 5}) for _ in range(8)} <= top5
    for r in recs:
        r.routes.clear()
    full = dec.forward(ids, dec.new_cache(512), all_logits=True).cpu().numpy()
    ref, _ = omodel.model_forward(ids, t.embed, t.attn, offs, t.final_norm, t.lm_head, t.spec(), omodel.KvCache(), 0,
                                  bf16_acts=True)
    assert _rel_rows(full, ref) <= LOGITS_TOL


def test_backend_generate_batch():
    """``generate_batch`` (one engine step for several requests in one decoder pass, their MoE
    blocks sharing it): every request's logits against its own fresh prefill on the GPU, the
    prompts run once and then one position per request, and the final sequences' logits at
    every position against the oracle."""
    t = make_tiny(36, kv_heads=2, qk_norm="head")
    dec, recs, offs = _moe_model(t, "awq_int4_g128", 36)
    be = GenericBackend(dec, max_seqs=3, max_len=256, prefill_chunk=32)
    rng = np.random.default_rng(12)
    seqs = [[int(x) for x in rng.integers(0, t.vocab, n)] for n in (21, 5, 40)]
    for step in range(4):
        before = be.tokens_run
        logits = be.logits_batch(seqs)
        assert be.tokens_run - before == (66 if step == 0 else 3)
        for s, lg in zip(seqs, logits):
            fresh = dec.forward(s, dec.new_cache(256)).cpu().numpy()
            assert _rel_rows(lg.cpu().numpy(), fresh) <= LOGITS_TOL, step
        toks = be.generate_batch([(s, {"temperature": 0.0}) for s in seqs])
        for s, lg, tok in zip(seqs, logits, toks):
            g = lg.cpu().numpy()
            assert g[tok] >= g.max() - 1e-3 * np.abs(g).max(), step
            s.append(tok)
    for s in seqs:
        for r in recs:
            r.routes.clear()
        full = dec.forward(s, dec.new_cache(256), all_logits=True).cpu().numpy()
        ref, _ = omodel.model_forward(s, t.embed, t.attn, offs, t.final_norm, t.lm_head, t.spec(), omodel.KvCache(),
                                      0, bf16_acts=True)
        assert _rel_rows(full, ref) <= LOGITS_TOL


@pytest.mark.parametrize("fmt, keep_quantized", [("fp8_b128", False), ("awq_int4_g128", False),
                                                 ("fp8_b128", True), ("awq_int4_g128", True)])
def test_load_decoder_matches_oracle(tmp_path, fmt, keep_quantized):
    """``load_decoder`` of a written checkpoint (quantized attention projections dequantized
    on the device to bf16, or kept quantized and run by ``ccut_quant_linear``; MoE layers 0
    and 2, a dense MLP in layer 1) against the oracle's decoder over the same tensors: a
    25-token prefill and two single-token steps."""
    t = make_tiny(44, kv_heads=2, qk_norm="head", layers=3)
    q = quantized_layers(t, fmt, seed=44)
    mats, attn = quantized_attention(t, fmt, seed=45, bf16=not keep_quantized)
    dl = inputs.make_layer(inputs.scaled_config("cfg1" if fmt == "fp8_b128" else "cfg0", hidden=t.hidden, inter=256,
                                                num_experts=1, top_k=1, num_shared=0), seed=46)
    root = write_decoder_checkpoint(tmp_path / "m", t, fmt, q, mats, dense={1: dl.experts[0]}, dense_inter=256)
    dec = load_decoder(root, quantized_projections=keep_quantized)
    recs = {}
    for i in (0, 2):
        dec.layers[i].ffn = recs[i] = _Recorded(dec.layers[i].ffn)
    wg, wu, wd = dl.w_lookup(0)
    offs = [_oracle_moe(q[0], t.top_k, t.mode, recs[0]), lambda x: moe.expert_ffn(x, wg, wu, wd),
            _oracle_moe(q[2], t.top_k, t.mode, recs[2])]
    tq = dataclasses.replace(t, attn=attn)
    cache, ocache = dec.new_cache(128), omodel.KvCache()
    rng = np.random.default_rng(14)
    pos = 0
    for n in (25, 1, 1):
        toks = rng.integers(0, t.vocab, n)
        got = dec.forward(toks, cache, all_logits=True)
        ref, _ = omodel.model_forward(toks, tq.embed, tq.attn, offs, tq.final_norm, tq.lm_head, tq.spec(), ocache,
                                      pos, bf16_acts=True)
        assert _rel_rows(got.cpu().numpy(), ref) <= LOGITS_TOL, (n, pos)
        pos += n


def _forced_moe(rec: _Recorded, inner):
    """The oracle MoE callable ``inner`` (``omodel.moe_ffn``) on the routing the GPU chose,
    after checking that the GPU's experts are a near-optimal choice under the oracle's own
    selection scores (their sum within ``NEAR_TIE`` of the oracle's)."""
    router, top_k, mode, lookup, shared, kw = inner.args

    def f(x):
        ids, w = rec.routes.pop(0)
        lg = x @ router.T
        _, own = routing.route(lg, top_k, mode, **kw)
        c = 1.0 / (1.0 + np.exp(-lg)) + (kw["bias"] if kw.get("bias") is not None else 0.0)
        for t in range(x.shape[0]):
            if set(ids[t].tolist()) != set(own[t].tolist()):
                assert c[t, own[t]].sum() - c[t, ids[t]].sum() < NEAR_TIE, f"token {t}: {ids[t]} vs {own[t]}"
        return moe.moe_forward(x, router, top_k, mode, lookup, shared, ids=ids, weights=w)[0]

    return f


@pytest.mark.parametrize("case", sorted(DS_CASES))
@pytest.mark.parametrize("keep_quantized", [False, True])
def test_load_deepseek_decoder_matches_oracle(tmp_path, case, keep_quantized):
    """``load_decoder`` of a DeepSeek-V3-style checkpoint (MLA with YaRN and interleaved rope
    channels, a dense first layer, grouped sigmoid routing): a 9-token prefill and three
    single-token steps against the oracle's decoder over the same tensors, which matches
    transformers' DeepseekV3ForCausalLM on the CPU."""
    root = write_deepseek_checkpoint(tmp_path / case, case)
    dec = load_decoder(root, quantized_projections=keep_quantized)
    assert type(dec.layers[0]).__name__ == "MlaDecoderLayer" and dec.layout == ("mla", 1, 576)
    rec = _Recorded(dec.layers[1].ffn)
    dec.layers[1].ffn = rec
    w = load_decoder_weights(root)
    layers, ffns, spec = oracle_decoder(w, "quantized" if keep_quantized else "bf16")
    ffns[1] = _forced_moe(rec, ffns[1])
    cache, ocache = dec.new_cache(256), omodel.KvCache()
    toks = np.random.default_rng(7).integers(0, w["spec"].vocab, 12)
    pos = 0
    for n in (9, 1, 1, 1):
        got = dec.forward(toks[pos: pos + n], cache, all_logits=True)
        torch.cuda.synchronize()
        ref, _ = omodel.model_forward(toks[pos: pos + n], w["embed"], layers, ffns, w["final_norm"], w["lm_head"],
                                      spec, ocache, pos, bf16_acts=True)
        err = _rel_rows(got.cpu().numpy(), ref)
        assert err <= LOGITS_TOL, (case, pos, err)
        pos += n
    assert not rec.routes
