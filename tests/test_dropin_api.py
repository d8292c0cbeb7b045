"""The drop-in modules keep the reference's names and argument lists (no GPU needed)."""

from __future__ import annotations

import inspect

import pytest

import numpy as np

from ccut_b200 import quant
from ccut_b200.blocks import attn_gqa, attn_mla, moe, norm, rope

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
    # ccut/blocks/attn_gqa.py, ccut/blocks/norm.py (leading parameters; the GPU versions add
    # keyword options after them)
    attn_gqa.build_causal_mask: ["seq_len", "start_pos"],
    attn_gqa.gqa_attention: ["q", "k", "v", "mask", "scale", "softcap"],
    norm.rms_norm: ["x", "weight", "eps"],
    rope.apply_rope: ["q", "k", "inv_freq", "positions", "attention_factor", "scaling_type", "seq_len"],
    # ccut/blocks/attn_mla.py
    attn_mla.mla_update_state: ["state", "x", "kv_a_proj", "kv_a_scale", "q_pe"],
    attn_mla.mla_decode: ["state", "q_nope", "q_pe_rot", "k_up_proj", "v_up_proj", "scale", "start_pos"],
    attn_mla.mla_prefill: ["state", "q_nope", "q_pe_rot", "k_up_proj", "v_up_proj", "scale", "start_pos"],
}
PREFIX = {attn_gqa.gqa_attention_fast: ["q", "k", "v", "mask", "scale"],
          attn_mla.MLAState.__init__: ["self", "kv_lora_rank", "qk_rope_head_dim", "max_tokens"]}


@pytest.mark.parametrize("fn", list(PREFIX), ids=lambda f: f.__qualname__)
def test_signature_prefix_matches_reference(fn):
    names = list(inspect.signature(fn).parameters)
    assert names[:len(PREFIX[fn])] == PREFIX[fn]


def test_causal_mask_detection():
    """The attention drop-in turns the reference's build_causal_mask masks (plain or
    broadcast over batch and heads) into a causal offset and rejects other masks."""
    m = attn_gqa.build_causal_mask(3, 5)
    assert m.shape == (3, 8) and m[0, 5] == 0 and m[0, 6] < -1e29 and m[2, 7] == 0
    assert attn_gqa._causal_start(None, 3, 8) == -1
    assert attn_gqa._causal_start(m, 3, 8) == 5
    assert attn_gqa._causal_start(np.broadcast_to(m[None, None], (2, 4, 3, 8)), 3, 8) == 5
    with pytest.raises(NotImplementedError):
        attn_gqa._causal_start(np.zeros((3, 8), np.float32) - 1.0, 3, 8)
    with pytest.raises(NotImplementedError):  # the same masked count, other positions
        attn_gqa._causal_start(m[:, ::-1].copy(), 3, 8)
    with pytest.raises(ValueError):
        attn_gqa._causal_start(m, 2, 8)


@pytest.mark.parametrize("fn", list(REFERENCE), ids=lambda f: f.__qualname__)
def test_signature_matches_reference(fn):
    assert list(inspect.signature(fn).parameters) == REFERENCE[fn]


def test_unknown_format_is_not_implemented():
    with pytest.raises(NotImplementedError):
        quant.make_method("nf4", 128, 128)


def test_tile_multiples_required():
    with pytest.raises(ValueError):
        quant.AwqInt4G128Method(100, 128)


def test_expert_pipeline_host_side():
    """ccut_b200.experts keeps the reference pipeline's names (ccut/experts/pipeline.py): the
    step signature, the metrics dict, the routing history's prediction rule, and the argument
    checks, which run before any GPU work."""
    import types

    from ccut_b200 import experts

    assert list(inspect.signature(experts.ExpertPipeline.step).parameters) == [
        "self", "layer", "x", "gate_w", "top_k", "norm_topk_prob", "shared_projs", "shared_gate"]
    assert list(inspect.signature(experts.ExpertPipeline.__init__).parameters) == [
        "self", "reader", "num_workers", "speculative_window", "prefetch_steps_ahead", "metrics_enabled"]
    m = experts.PipelineMetrics()
    assert set(m.to_dict()) == {"compute_ns", "prefetch_ns", "overlap_ns", "overlap_ratio", "steps",
                                "spec_accept_rate", "ring_hits", "ring_misses"}
    assert m.overlap_ratio() == 0.0 and m.speculative_accept_rate() == 0.0
    h = experts.RouteHistory(window=3)
    assert h.predict(2) == []
    for s in ([1, 2, 3], [2, 3, 4], [3, 5]):
        h.record(s)
    assert h.predict(2) == [3, 2]
    h.record([9])  # the window drops [1, 2, 3]
    assert h.predict(1) == [3] and 1 not in h.predict(10)
    t = experts.RouteHistory(window=2)
    t.record([7])
    t.record([8])
    assert t.predict(2) == [7, 8]  # a tie keeps the order of first counting
    layer = types.SimpleNamespace(top_k=2, routing="softmax_topk", num_slices=0, router=np.zeros((8, 128), np.float32),
                                  hidden=128, device="cuda")
    pipe = experts.ExpertPipeline({0: layer})
    x, gw = np.zeros((2, 128), np.float32), np.zeros((8, 128), np.float32)
    with pytest.raises(ValueError):
        pipe.step(0, x, gw, top_k=3, norm_topk_prob=False)
    with pytest.raises(ValueError):
        pipe.step(0, x, gw, top_k=2, norm_topk_prob=True)
    with pytest.raises(ValueError):
        pipe.step(0, x, gw, top_k=2, norm_topk_prob=False, shared_projs={"gate_proj": None})
    with pytest.raises(ValueError):
        pipe.step(0, x, np.zeros((4, 128), np.float32), top_k=2, norm_topk_prob=False)
    with pytest.raises(KeyError):
        pipe.step(1, x, gw, top_k=2, norm_topk_prob=False)
    pipe.close()
