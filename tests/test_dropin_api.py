"""The drop-in modules keep the reference's names and argument lists (no GPU needed)."""

from __future__ import annotations

import inspect

import pytest

from ccut_b200 import quant
from ccut_b200.blocks import moe

# parameter names of the reference functions (ccut/blocks/moe.py, ccut/models/generic.py,
# ccut/quant/method.py)
REFERENCE = {
    moe.topk: ["x", "k"],
    moe.topk_softmax: ["logits", "k", "norm_topk_prob"],
    moe.moe_combine: ["x", "expert_ids", "weights", "expert_outputs", "expert_fn", "w_lookup"],
    moe.moe_forward: ["h", "gate_w", "reader", "layer", "moe_spec", "shared_projs"],
    moe.shared_expert_add: ["y", "shared_out", "gate_value"],
    quant.QuantizeMethodBase.apply: ["self", "weight_bytes", "scales", "x"],
    quant.QuantizeMethodBase.create_weights: ["self", "spec"],
    quant.QuantizeMethodBase.process_weights_after_loading: ["self"],
}


@pytest.mark.parametrize("fn", list(REFERENCE), ids=lambda f: f.__qualname__)
def test_signature_matches_reference(fn):
    assert list(inspect.signature(fn).parameters) == REFERENCE[fn]


def test_unknown_format_is_not_implemented():
    with pytest.raises(NotImplementedError):
        quant.make_method("nf4", 128, 128)


def test_tile_multiples_required():
    with pytest.raises(ValueError):
        quant.AwqInt4G128Method(100, 128)
