"""Generate ``tests/golden/routing_wide.npz``: the reference's ``topk_softmax``
(``ccut/blocks/moe.py:71-89``) on router shapes beyond the base fixtures (only where the
reference sources exist)::

    python tests/golden/make_golden_routing.py [--reference PATH_TO_REFERENCE/python]

Cases: 128 experts top-8 with ``norm_topk_prob=True`` (Qwen3-30B-A3B), 256 experts top-16
in both modes (the library's limits), each with rows of exact ties (a constant row, a tied
top block) and a row whose k-th and (k+1)-th logits tie.
"""

from __future__ import annotations

import argparse
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
CASES = [(128, 8, True), (256, 16, False), (256, 16, True)]


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
    from ccut.blocks.moe import topk_softmax

    rng = np.random.default_rng(404)
    out = {}
    for i, (E, k, norm) in enumerate(CASES):
        lg = (rng.standard_normal((48, E)) * 1.5).astype(np.float32)
        lg[3, :] = 0.75                    # all tied
        lg[4, 10:10 + k + 3] = 6.0         # a tied top block wider than k
        lg[5, :] = -1.0
        lg[5, 7:7 + k - 1] = 4.0           # k - 1 clear winners ...
        lg[5, [2, 200 % E]] = 2.0          # ... and a tie for the k-th place
        w, ids = topk_softmax(lg, k, norm)
        out.update({f"c{i}_logits": lg, f"c{i}_ids": np.asarray(ids, np.int64), f"c{i}_w": np.asarray(w, np.float32),
                    f"c{i}_k": np.int64(k), f"c{i}_norm": np.bool_(norm)})
    np.savez_compressed(HERE / "routing_wide.npz", **out)
    print("wrote", HERE / "routing_wide.npz")
    return 0


if __name__ == "__main__":
    sys.exit(main())
