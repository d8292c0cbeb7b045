"""CPU oracle for the quantized MoE expert forward -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the CostCut-Infer (``ccut``) reference algorithm for
the MoE expert path so that the CUDA path in ``ccut_b200`` can be checked against it.
It is never the thing measured or shipped:

* only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
  ``--impl reference`` legs of ``bench.py`` may import it;
* the product package ``ccut_b200`` never imports it and has no CPU fallback.

Modules
-------
``formats``  AWQ int4 group-128 and FP8-e4m3 128x128-block weight formats
             (pack / unpack / dequant), plus the e4m3 decode table.
``routing``  router top-k: softmax-then-top-k, top-k-then-softmax, grouped sigmoid.
``moe``      SwiGLU expert FFN, token grouping, weighted combine, shared experts,
             whole-layer forward.
``inputs``   seeded synthetic layer/activation generator for the benchmark configs.
``attention`` GQA / MLA attention, RMSNorm and RoPE blocks.
``model``    the generic decoder layer (attention block + MoE / dense FFN) and a whole
             decoder step (embedding, layers, final norm, ``lm_head``).

Pinning.  Each function cites the reference file:line it follows (paths relative to the
reference's ``python/`` directory).  ``tests/golden/make_golden.py`` imports the
reference itself (only possible where its sources are present) and writes the golden
fixtures under ``tests/golden/``; ``tests/test_oracle_golden.py`` checks this oracle
against them.  The AWQ-int4-g128 and FP8-block-128 formats and grouped sigmoid routing
have no implementation in the reference: those parts are restatements of the published
formats, pinned only where they coincide with a reference format (uniform zero-point /
scale cases, see ``tests/golden/make_golden.py``) -- "parity partially unpinned".
"""

from oracle import formats, inputs, moe, routing  # noqa: F401

__all__ = ["formats", "inputs", "moe", "routing"]
