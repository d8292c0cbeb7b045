"""Generate ``tests/golden/rope_tables.npz``: the reference's ``build_rope`` tables
(``ccut/blocks/rope.py:88-127``) for the scalings it serves (only where the reference sources
exist; they do not travel to GPU boxes)::

    python tests/golden/make_golden_rope.py [--reference PATH_TO_REFERENCE/python]

Stored per case: head dim, theta, the scaling dict (JSON), ``inv_freq`` and the attention
factor.  The yarn cases cover both sides of its factor-1.5 branch and an explicit
``attention_factor``.
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

# head_dim, rope_theta, max_position, rope_scaling
CASES = [
    (128, 1e6, 131072, {"type": "yarn", "factor": 4.0, "original_max_position_embeddings": 32768}),
    (64, 1e4, 8192, {"type": "yarn", "factor": 1.25, "beta_fast": 16.0, "beta_slow": 2.0}),
    (128, 5e5, 65536, {"type": "yarn", "factor": 8.0, "attention_factor": 1.1}),
    (64, 1e4, 4096, {"type": "dynamic", "factor": 2.0}),
    (128, 1e6, 4096, {"type": "linear", "factor": 2.0}),
]


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
    from ccut.blocks.rope import build_rope

    out = {}
    for i, (d, theta, max_pos, rs) in enumerate(CASES):
        inv, af = build_rope(d, theta, max_pos, dict(rs))
        out[f"r{i}_head_dim"] = np.int64(d)
        out[f"r{i}_theta"] = np.float64(theta)
        out[f"r{i}_scaling"] = np.array(json.dumps(rs))
        out[f"r{i}_inv_freq"] = np.asarray(inv, np.float32)
        out[f"r{i}_attn_factor"] = np.float64(af)
    out["n"] = np.int64(len(CASES))
    np.savez_compressed(HERE / "rope_tables.npz", **out)
    print("wrote", HERE / "rope_tables.npz")
    return 0


if __name__ == "__main__":
    sys.exit(main())
