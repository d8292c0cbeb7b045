"""Generate ``tests/golden/attn_norm.npz`` by running the reference's attention and
RMSNorm blocks (only where the reference sources exist; they do not travel to GPU boxes)::

    python tests/golden/make_golden_attn.py [--reference PATH_TO_REFERENCE/python]

Cases (inputs are bf16-representable, stored as bf16 bit patterns, outputs fp32):

``gqa{i}_*``  ``gqa_attention_fast`` (``ccut/blocks/attn_gqa.py:127-153``) with the causal
              mask of ``build_causal_mask`` (``:65-73``) broadcast over batch and heads,
              or no mask; grouped (8 query heads on 2 and on 1 kv heads) and plain heads,
              head dims 64 and 128, one and several query rows.
``rms{i}_*``  ``rms_norm`` (``ccut/blocks/norm.py:14-26``) with and without a weight.
``mla{i}_*``  ``mla_decode`` / ``mla_prefill`` (``ccut/blocks/attn_mla.py:85-167``) over an
              ``MLAState`` latent cache: one decode token, and a causal prefill batch after a
              prefix.
``rope{i}_*`` ``apply_rope`` (``ccut/blocks/rope.py:130-175``) with the inverse frequencies
              and attention factor of ``build_rope``: no scaling (head dim 128, theta 1e6)
              and yarn (head dim 64, factor 4: the attention factor scales q).
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

from oracle import formats  # noqa: E402

GQA_CASES = [
    # batch, heads, kv_heads, seq, start_pos (None: no mask, kv_len = extra), d
    (2, 8, 2, 5, 11, 64),
    (3, 8, 1, 1, 36, 128),
    (1, 2, 2, 3, None, 128),
    (1, 16, 2, 7, 40, 128),
]
RMS_CASES = [(7, 384, True, 1e-6), (3, 256, False, 1e-5)]
# batch, heads, kv_heads, seq, head_dim, theta, rope_scaling, first positions per batch row
ROPE_CASES = [(2, 4, 2, 3, 128, 1e6, None, (5, 100)),
              (1, 2, 1, 5, 64, 1e4, {"type": "yarn", "factor": 4.0}, (4000,))]


def bf16_round(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    bits = formats.bf16_bits_from_f32(x.astype(np.float32))
    return bits, formats.bf16_bits_to_f32(bits)


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
    from ccut.blocks.attn_gqa import build_causal_mask, gqa_attention_fast
    from ccut.blocks.norm import rms_norm
    from ccut.blocks.attn_mla import MLAState, mla_decode, mla_prefill
    from ccut.blocks.rope import apply_rope, build_rope

    rng = np.random.default_rng(2024)
    out = {}
    for i, (b, h, kvh, s, start, d) in enumerate(GQA_CASES):
        kv = (start + s) if start is not None else 40
        qb, q = bf16_round(rng.standard_normal((b, h, s, d)))
        kb, k = bf16_round(rng.standard_normal((b, kvh, kv, d)))
        vb, v = bf16_round(rng.standard_normal((b, kvh, kv, d)))
        mask = None
        if start is not None:
            mask = np.broadcast_to(build_causal_mask(s, start)[None, None], (b, h, s, kv)).copy()
        o = gqa_attention_fast(q, k, v, mask, scale=None)
        out.update({f"gqa{i}_q": qb, f"gqa{i}_k": kb, f"gqa{i}_v": vb, f"gqa{i}_out": o.astype(np.float32),
                    f"gqa{i}_start": np.int64(-1 if start is None else start)})
    for i, (n, dim, with_w, eps) in enumerate(RMS_CASES):
        xb, x = bf16_round(rng.standard_normal((n, dim)) * 3)
        w = formats.bf16_bits_to_f32(formats.bf16_bits_from_f32(rng.uniform(0.5, 1.5, dim).astype(np.float32)))
        y = rms_norm(x, w if with_w else None, eps)
        out.update({f"rms{i}_x": xb, f"rms{i}_w": w if with_w else np.zeros(0, np.float32),
                    f"rms{i}_eps": np.float32(eps), f"rms{i}_y": y.astype(np.float32)})
    for i, (b, h, kvh, s, d, theta, scaling, starts) in enumerate(ROPE_CASES):
        qb, q = bf16_round(rng.standard_normal((b, h, s, d)))
        kb, k = bf16_round(rng.standard_normal((b, kvh, s, d)))
        inv_freq, attn = build_rope(d, theta, 8192, scaling)
        stype = (scaling or {}).get("type", "none")
        pos = np.stack([np.arange(p, p + s) for p in starts]).astype(np.int64)
        qo, ko = apply_rope(q, k, inv_freq, pos, attn, stype)
        out.update({f"rope{i}_q": qb, f"rope{i}_k": kb, f"rope{i}_inv_freq": np.asarray(inv_freq, np.float32),
                    f"rope{i}_attn": np.float32(attn), f"rope{i}_type": np.array(stype), f"rope{i}_pos": pos,
                    f"rope{i}_q_out": qo.astype(np.float32), f"rope{i}_k_out": ko.astype(np.float32)})
    # MLA: rank 64, rope dim 16, nope dim 32, v dim 32, 4 heads
    rank, dr, dn, dv, heads = 64, 16, 32, 32, 4
    for i, (prefix, seq) in enumerate(((19, 1), (11, 6))):
        kv = prefix + seq
        _, c = bf16_round(rng.standard_normal((kv, rank)))
        _, kpe = bf16_round(rng.standard_normal((kv, dr)))
        _, qn = bf16_round(rng.standard_normal((seq, heads, dn)))
        _, qp = bf16_round(rng.standard_normal((seq, heads, dr)))
        _, ku = bf16_round(rng.standard_normal((rank, heads * dn)) * 0.125)
        _, vu = bf16_round(rng.standard_normal((rank, heads * dv)) * 0.125)
        st = MLAState(rank, dr, max_tokens=64)
        st.append(c, kpe)
        scale = 1.0 / np.sqrt(dn + dr)
        if seq == 1:
            o = mla_decode(st, qn[0], qp[0], ku, vu, scale, prefix)[None]
        else:
            o = mla_prefill(st, qn, qp, ku, vu, scale, prefix)
        out.update({f"mla{i}_c": c, f"mla{i}_kpe": kpe, f"mla{i}_qn": qn, f"mla{i}_qp": qp, f"mla{i}_ku": ku,
                    f"mla{i}_vu": vu, f"mla{i}_scale": np.float32(scale), f"mla{i}_start": np.int64(prefix),
                    f"mla{i}_out": np.asarray(o, np.float32)})
    np.savez_compressed(HERE / "attn_norm.npz", **out)
    print("wrote", HERE / "attn_norm.npz")
    return 0


if __name__ == "__main__":
    sys.exit(main())
