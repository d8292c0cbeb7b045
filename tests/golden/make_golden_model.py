"""Generate ``tests/golden/model_decode.npz`` by running the reference's generic decoder layer
(only where the reference sources exist; they do not travel to GPU boxes)::

    python tests/golden/make_golden_model.py [--reference PATH_TO_REFERENCE/python]

Each case is a seeded tiny model of ``tests/model_helpers.make_tiny`` (bf16 weights, dense
bf16 experts, one shared expert, one kv head) decoding a seeded token sequence one token at a
time, the way ``ccut/models/generic.py:9-18`` lays out a step: ``EmbedTable`` rows
(``ccut/blocks/heads.py:45-46``), ``model_forward_layer`` (``ccut/models/generic.py:403-447``)
for every layer with an ``AttentionContext`` at the token's position and a per-layer kv store,
``rms_norm`` with the final norm and ``LmHead`` (``ccut/blocks/heads.py:59-60``).  Weights reach
the reference through its ``FakeWeightReader`` as raw bf16 bytes, projections as
``LinearProj`` (``[out, in]``), experts under the keys ``_expert_seg_f32`` reads
(``experts.{e}.{proj}_proj``, ``[in, out]``).

The reference's layer passes q as ``[1, seq, heads, d]`` to blocks that take ``[batch, heads,
seq, d]``; with one token and one kv head that is the same computation, so these are the
cases pinned.  Stored per case: the model's seed and options, the tokens, the reference's
``build_rope`` inverse frequencies, the hidden state after every layer and the logits of
every step.  ``samp*``: the reference's sampling transform ``temperature_topk``
(``ccut/blocks/heads.py:76-126``) of seeded logits under several temperature / top-k / top-p /
min-p settings.
"""

from __future__ import annotations

import argparse
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "tests"))

from model_helpers import make_tiny  # noqa: E402
from oracle import formats  # noqa: E402

# seed, norm_topk_prob, qk_norm, steps
CASES = [(11, False, "flat", 6), (12, True, None, 5)]
# temperature, top_k, top_p, min_p
SAMPLING = [(0.7, 0, 1.0, 0.0), (1.0, 20, 1.0, 0.0), (0.8, 0, 0.9, 0.0), (1.2, 0, 1.0, 0.05),
            (0.9, 40, 0.8, 0.02), (1.0, 0, 0.3, 0.0)]


class _KvStore:
    """The kv block view ``full_attn_forward`` writes and gathers: ``write(k, v)`` appends one
    batch of positions, ``gather()`` returns ``[kv_heads, positions, d]`` k and v."""

    def __init__(self, kv_heads: int, d: int):
        self.kvh, self.d = kv_heads, d
        self.k = np.zeros((0, kv_heads, d), np.float32)
        self.v = np.zeros((0, kv_heads, d), np.float32)

    def write(self, k, v):
        self.k = np.concatenate([self.k, np.asarray(k, np.float32).reshape(-1, self.kvh, self.d)])
        self.v = np.concatenate([self.v, np.asarray(v, np.float32).reshape(-1, self.kvh, self.d)])

    def gather(self):
        return self.k.transpose(1, 0, 2), self.v.transpose(1, 0, 2)


def _raw(a: np.ndarray) -> bytes:
    return formats.bf16_bits_from_f32(np.ascontiguousarray(a, np.float32)).tobytes()


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("CCUT_REFERENCE"),
                    help="the reference's python/ directory (or set CCUT_REFERENCE)")
    args = ap.parse_args(argv)
    if not args.reference:
        ap.error("--reference (or CCUT_REFERENCE) must name the reference\'s python/ directory")
    os.environ.setdefault("NUMBA_CACHE_DIR", tempfile.mkdtemp(prefix="ccut-numba-"))
    sys.dont_write_bytecode = True
    sys.path.insert(0, args.reference)
    from ccut.blocks.heads import EmbedTable, LmHead
    from ccut.blocks.norm import rms_norm
    from ccut.blocks.rope import build_rope
    from ccut.models.generic import AttentionContext, FakeWeightReader, build_linear_projs, model_forward_layer
    from ccut.models.spec import LayerTemplate, ModelSpec, MoeSpec

    out = {}
    for ci, (seed, norm, qk_norm, steps) in enumerate(CASES):
        t = make_tiny(seed, norm_topk_prob=norm, qk_norm=qk_norm)
        H, d = t.hidden, t.head_dim
        spec = ModelSpec(
            architectures=["TinyMoe"], model_type="tiny_moe", hidden_size=H, num_hidden_layers=t.layers,
            vocab_size=t.vocab, tie_word_embeddings=False, rms_norm_eps=t.eps, max_position_embeddings=4096,
            rope_theta=t.theta, rope_scaling=None, num_attention_heads=t.heads, num_key_value_heads=t.kv_heads,
            head_dim=d, layer_templates=[LayerTemplate(i, "full_attn") for i in range(t.layers)],
            moe=MoeSpec(t.num_experts, t.top_k, t.inter, norm, t.shared_inter > 0, t.shared_inter),
        )
        table, shapes, state, pools = {}, {}, {}, {}
        for i in range(t.layers):
            w = t.attn[i]
            dims = {"q_proj": (t.heads * d, H), "k_proj": (t.kv_heads * d, H), "v_proj": (t.kv_heads * d, H),
                    "o_proj": (H, t.heads * d)}
            for n, m in zip(dims, (w.wq, w.wk, w.wv, w.wo)):
                table[(i, f"self_attn.{n}")] = _raw(m)
                shapes[(i, f"self_attn.{n}")] = (*m.shape, "bf16")
            for e, (wg, wu, wd) in enumerate(t.experts[i]):
                for proj, m in (("gate_proj", wg), ("up_proj", wu), ("down_proj", wd)):
                    table[(i, f"experts.{e}.{proj}_proj")] = _raw(m)
            sg, su, sd = t.shared[i]
            sdims = {"gate_proj": (t.shared_inter, H), "up_proj": (t.shared_inter, H), "down_proj": (H, t.shared_inter)}
            for n, m in zip(sdims, (sg.T, su.T, sd.T)):
                table[(i, f"shared_expert.{n}")] = _raw(m)
            state[f"{i}.input_layernorm"] = w.ln1
            state[f"{i}.post_attention_layernorm"] = w.ln2
            if w.q_norm is not None:
                state[f"{i}.q_norm"], state[f"{i}.k_norm"] = w.q_norm, w.k_norm
            state[f"{i}.gate_w"] = t.router[i]
            pools[i] = _KvStore(t.kv_heads, d)
        reader = FakeWeightReader(table, shapes)
        for i in range(t.layers):
            state[f"{i}.projs"] = build_linear_projs(i, reader, None, "self_attn.", dims)
            state[f"{i}.shared"] = build_linear_projs(i, reader, None, "shared_expert.", sdims)
        inv_freq, attn_factor = build_rope(d, t.theta, 4096, None)
        rng = np.random.default_rng(1000 + seed)
        tokens = rng.integers(0, t.vocab, steps).astype(np.int64)
        emb, head = EmbedTable(t.embed), LmHead(t.lm_head)
        hs = np.zeros((steps, t.layers, H), np.float32)
        logits = np.zeros((steps, t.vocab), np.float32)
        for s, tok in enumerate(tokens):
            ctx = AttentionContext(inv_freq, attn_factor, {}, start_pos=s)
            h = emb(np.array([tok]))
            for i in range(t.layers):
                h = model_forward_layer(i, h, reader, spec, None, ctx, pools, state)
                hs[s, i] = h[0]
            logits[s] = head(rms_norm(h, t.final_norm, t.eps))[0]
        out.update({f"m{ci}_seed": np.int64(seed), f"m{ci}_norm": np.bool_(norm),
                    f"m{ci}_qk_norm": np.array(qk_norm or "none"), f"m{ci}_tokens": tokens,
                    f"m{ci}_inv_freq": np.asarray(inv_freq, np.float32), f"m{ci}_attn_factor": np.float32(attn_factor),
                    f"m{ci}_h": hs, f"m{ci}_logits": logits})
    # the sampling transform: temperature_topk (ccut/blocks/heads.py:76-126) on seeded logits
    from ccut.blocks.heads import temperature_topk

    rng = np.random.default_rng(77)
    logits = (rng.standard_normal((6, 256)) * 3).astype(np.float32)
    out["samp_logits"] = logits
    out["samp_params"] = np.array(SAMPLING, np.float64)
    for j, (temp, top_k, top_p, min_p) in enumerate(SAMPLING):
        out[f"samp{j}_probs"] = temperature_topk(logits.copy(), temp, top_k=int(top_k), top_p=top_p,
                                                 min_p=min_p).astype(np.float32)
    np.savez_compressed(HERE / "model_decode.npz", **out)
    print("wrote", HERE / "model_decode.npz")
    return 0


if __name__ == "__main__":
    sys.exit(main())
