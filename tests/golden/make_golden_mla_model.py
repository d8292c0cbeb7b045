"""Generate ``tests/golden/mla_decoder.npz``: tiny MLA decoders run through the reference's own
blocks (only where the reference sources exist; they do not travel to GPU boxes)::

    python tests/golden/make_golden_mla_model.py [--reference PATH_TO_REFERENCE/python]

The reference has MLA blocks (``ccut/blocks/attn_mla.py``) but no layer that calls them, so
the layer here is assembled from them in the order the block module's docstring gives
(``ccut/blocks/attn_mla.py:1-13``), with the MoE branch and the step layout of the generic
decoder (``ccut/models/generic.py:9-18``, ``:403-447``):

- ``h_norm = rms_norm(h, input_layernorm)`` (``ccut/blocks/norm.py``);
- ``q = h_norm @ q_proj^T`` (with a q rank: ``rms_norm(h_norm @ q_a^T, q_a_norm) @ q_b^T``),
  split per head into ``q_nope`` and ``q_pe``;
- ``kv_a = h_norm @ kv_a_proj^T`` split into ``c`` and ``k_pe``; ``q_pe`` / ``k_pe`` rotated
  by ``apply_rope`` at the tokens' absolute positions (``ccut/blocks/rope.py:130-175``, the
  table of ``build_rope``);
- the cache update: ``mla_update_state`` when the case has no ``kv_a_layernorm`` (it appends
  the raw ``c`` and the rotated ``k_pe``), else ``MLAState.append`` of ``rms_norm(c)``;
- ``mla_prefill`` for a chunk of several tokens, ``mla_decode`` for one, with ``k_up`` /
  ``v_up`` the per-head blocks of ``kv_b_proj``; then ``o_proj``;
- ``h += attention``, ``h += moe_forward(rms_norm(h, post_attention_layernorm), ...)``
  through a ``FakeWeightReader`` as in ``make_golden_model.py``.

The schedule is a 4-token prefill, three single-token steps and a 2-token chunk.  Stored per
case: the seed and the MLA sizes, the tokens, the hidden state after every layer and the
logits of every token.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "tests"))
sys.path.insert(0, str(HERE))

from make_golden_model import _raw  # noqa: E402
from model_helpers import MLA_TINY, make_tiny  # noqa: E402
from oracle.model import mla_up_blocks  # noqa: E402

# seed, extra MLA options, norm_topk_prob
CASES = [(31, {"kv_norm": False}, False), (32, {"q_rank": 96, "scale": 0.11}, True)]
CHUNKS = (4, 1, 1, 1, 2)


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
    from ccut.blocks.attn_mla import MLAState, mla_decode, mla_prefill, mla_update_state
    from ccut.blocks.heads import EmbedTable, LmHead
    from ccut.blocks.norm import rms_norm
    from ccut.blocks.rope import apply_rope, build_rope
    from ccut.models.generic import FakeWeightReader, build_linear_projs, moe_forward
    from ccut.models.spec import MoeSpec

    out = {}
    for ci, (seed, extra, norm) in enumerate(CASES):
        mla = {**MLA_TINY, **extra}
        t = make_tiny(seed, norm_topk_prob=norm, mla=mla)
        H, R, dn, dr, dv = t.hidden, mla["rank"], mla["d_nope"], mla["d_rope"], mla["d_v"]
        moe_spec = MoeSpec(t.num_experts, t.top_k, t.inter, norm, t.shared_inter > 0, t.shared_inter)
        table, shapes, shared = {}, {}, {}
        sdims = {"gate_proj": (t.shared_inter, H), "up_proj": (t.shared_inter, H), "down_proj": (H, t.shared_inter)}
        for i in range(t.layers):
            for e, (wg, wu, wd) in enumerate(t.experts[i]):
                for proj, m in (("gate_proj", wg), ("up_proj", wu), ("down_proj", wd)):
                    table[(i, f"experts.{e}.{proj}_proj")] = _raw(m)
            sg, su, sd = t.shared[i]
            for n, m in zip(sdims, (sg.T, su.T, sd.T)):
                table[(i, f"shared_expert.{n}")] = _raw(m)
                shapes[(i, f"shared_expert.{n}")] = (*m.shape, "bf16")
        reader = FakeWeightReader(table, shapes)
        for i in range(t.layers):
            shared[i] = build_linear_projs(i, reader, None, "shared_expert.", sdims)
        inv_freq, attn_factor = build_rope(dr, t.theta, 4096, None)
        states = [MLAState(R, dr, max_tokens=64) for _ in range(t.layers)]
        rng = np.random.default_rng(2000 + seed)
        n_tok = sum(CHUNKS)
        tokens = rng.integers(0, t.vocab, n_tok).astype(np.int64)
        emb, head = EmbedTable(t.embed), LmHead(t.lm_head)
        hs = np.zeros((n_tok, t.layers, H), np.float32)
        logits = np.zeros((n_tok, t.vocab), np.float32)
        pos = 0
        for n in CHUNKS:
            h = emb(tokens[pos: pos + n])
            positions = np.arange(pos, pos + n, dtype=np.int64)[None, :]
            for i in range(t.layers):
                w = t.attn[i]
                x = rms_norm(h, w.ln1, t.eps)
                if w.wq_a is not None:
                    q = rms_norm(x @ w.wq_a.T, w.q_a_norm, t.eps) @ w.wq.T
                else:
                    q = x @ w.wq.T
                q = q.reshape(n, t.heads, dn + dr)
                kv_a = x @ w.wkv_a.T
                q_rot, k_rot = apply_rope(q[:, :, dn:].transpose(1, 0, 2)[None], kv_a[:, R:][None, None], inv_freq,
                                          positions, attn_factor, "none")
                q_rot, k_rot = q_rot[0].transpose(1, 0, 2), k_rot[0, 0]
                if w.kv_norm is None:
                    mla_update_state(states[i], x, w.wkv_a.T, None, k_rot)
                else:
                    states[i].append(rms_norm(kv_a[:, :R], w.kv_norm, t.eps), k_rot)
                k_up, v_up = mla_up_blocks(w.wkv_b, t.heads, dn, dv)
                if n == 1:
                    o = mla_decode(states[i], q[0, :, :dn], q_rot[0], k_up, v_up, w.softmax_scale, pos)[None]
                else:
                    o = mla_prefill(states[i], q[:, :, :dn], q_rot, k_up, v_up, w.softmax_scale, pos)
                h = h + o.reshape(n, t.heads * dv) @ w.wo.T
                h = h + moe_forward(rms_norm(h, w.ln2, t.eps), t.router[i], reader, i, moe_spec, shared[i])
                hs[pos: pos + n, i] = h
            logits[pos: pos + n] = head(rms_norm(h, t.final_norm, t.eps))
            pos += n
        out.update({f"c{ci}_seed": np.int64(seed), f"c{ci}_mla": np.array(json.dumps(mla)),
                    f"c{ci}_norm": np.bool_(norm), f"c{ci}_tokens": tokens,
                    f"c{ci}_inv_freq": np.asarray(inv_freq, np.float32), f"c{ci}_h": hs, f"c{ci}_logits": logits})
    out["chunks"] = np.array(CHUNKS, np.int64)
    np.savez_compressed(HERE / "mla_decoder.npz", **out)
    print("wrote", HERE / "mla_decoder.npz")
    return 0


if __name__ == "__main__":
    sys.exit(main())
