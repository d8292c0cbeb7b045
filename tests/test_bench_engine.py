"""``bench.engine_model`` on the CPU: the synthetic decoders of the engine workloads (config 2's
MLA stack with its dense first layer, pooled or not, and config 3's GQA stack) build with
their real attention shapes and run decode steps through ``GenericBackend``.  The MoE layer
and the dense FFN are stand-ins that check the shapes they are given (the AWQ dense FFN's
down projection over the padded intermediate among them); norms, RoPE and attention are the
torch stand-ins of ``tests/test_model_cpu.py``."""

from __future__ import annotations

import types

import numpy as np
import pytest
import torch

import bench
from tests import test_model_cpu as T


class _Moe:
    def __init__(self, fmt, H, I, E, k, routing, router, experts, shared=None, shared_inter=None, device=None, **kw):
        assert len(experts) == E and tuple(router.shape) == (E, H)
        self.H = H

    def forward(self, x, out_dtype=torch.bfloat16):
        assert x.dtype == torch.bfloat16 and x.shape[1] == self.H
        return (x.float() * 0.01).to(out_dtype)


class _Dense:
    def __init__(self, fmt, H, inter, g, u, d, device=None, **kw):
        ip = -(-inter // 128) * 128
        assert g.qweight.shape == (H, inter // 8) and u.scales.shape == (H // 128, inter)
        assert d.qweight.shape == (ip, H // 8)  # drawn over the padded intermediate
        self.H = H

    def forward(self, x, out_dtype=torch.bfloat16):
        assert x.shape[1] == self.H
        return (x.float() * 0.02).to(out_dtype)


@pytest.mark.parametrize("wl", ["cfg2_engine_decode", "cfg2_engine_decode_pool", "cfg3_engine_decode"])
def test_engine_model_builds_and_decodes(monkeypatch, wl):
    import ccut_b200.dense as dense
    import ccut_b200.layer as layer
    import ccut_b200.model as m
    import ccut_b200.synthetic as synthetic
    from ccut_b200.backend import GenericBackend

    for name, fn in (("rms_norm", T._norm), ("apply_rope", T._rope), ("_attend", T._attend), ("_mla_attend", T._mla),
                     ("_mla_attend_pool", T._mla_pool), ("_attend_pool", T._attend_pool)):
        monkeypatch.setattr(m, name, fn)
    monkeypatch.setattr(layer, "MoeLayer", _Moe)
    monkeypatch.setattr(dense, "DenseFfn", _Dense)
    monkeypatch.setattr(synthetic, "make_layer_device", lambda c, seed=0, device=None: types.SimpleNamespace(
        router=torch.zeros((c.num_experts, c.hidden)), experts=[None] * c.num_experts, shared=[]))
    w = dict(bench.ENGINE_WORKLOADS[wl], layers=2, vocab=1000, prompt=12, batch=3)
    dec = bench.engine_model(w, torch.device("cpu"))
    mla = w.get("attn") == "mla"
    assert dec.layout == (("mla", 1, 576) if mla else ("gqa", w["kv_heads"], w["head_dim"]))
    if mla:
        assert isinstance(dec.layers[0].ffn, _Dense) and isinstance(dec.layers[1].ffn, _Moe)
        assert tuple(dec.layers[0].k_up.shape) == (16, 128, 512) and tuple(dec.layers[0].v_up.shape) == (16, 512, 128)
    be = GenericBackend(dec, max_seqs=3, max_len=32, prefill_chunk=12, pool=w["pool"])
    seqs = [[int(x) for x in np.random.default_rng(i).integers(0, 1000, 12)] for i in range(3)]
    for _ in range(3):
        for s, tok in zip(seqs, be.generate_batch([(s, {"temperature": 0.0}) for s in seqs])):
            assert 0 <= tok < 1000
            s.append(tok)
    assert [len(s) for s in seqs] == [15, 15, 15]
