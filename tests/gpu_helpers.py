"""Shared helpers of the GPU parity tests (CUDA path vs the CPU oracle)."""

from __future__ import annotations

import numpy as np
import torch

from oracle import formats, inputs, moe, routing

# Output tolerance of the MoE layer: max over token rows of max|y - y_ref| / max|y_ref|.
# bf16 outputs with fp32 accumulation; bf16 output rounding alone is ~2^-9.
TOL = 1e-2


def small_cfg(fmt: str, mode: str = "softmax_topk", *, hidden=256, inter=128, experts=8, top_k=2, shared=0,
              shared_inter=None, **kw) -> inputs.MoeLayerConfig:
    return inputs.MoeLayerConfig(
        f"t_{fmt}", hidden=hidden, inter=inter, num_experts=experts, top_k=top_k, num_shared=shared,
        shared_inter=shared_inter or inter, fmt=fmt, routing=mode, **kw,
    )


def gpu_layer(lw: inputs.LayerWeights, device="cuda", **kw):
    from ccut_b200 import MoeLayer

    c = lw.cfg
    return MoeLayer(
        c.fmt, c.hidden, c.inter, c.num_experts, c.top_k, c.routing, lw.router, lw.experts,
        shared=lw.shared, shared_inter=c.shared_inter, n_group=c.n_group, topk_group=c.topk_group,
        routed_scaling=c.routed_scaling, device=device, **kw,
    )


def x_device(xb: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(xb.view(np.int16)).to(device).view(torch.bfloat16)


def rel_err_rows(y: np.ndarray, ref: np.ndarray) -> float:
    denom = np.maximum(np.abs(ref).max(axis=1), 1e-30)
    return float((np.abs(y - ref).max(axis=1) / denom).max())


def oracle_forward(lw: inputs.LayerWeights, xb: np.ndarray, ids=None, weights=None):
    c = lw.cfg
    xf = formats.bf16_bits_to_f32(xb)
    return moe.moe_forward(xf, lw.router, c.top_k, c.routing, lw.w_lookup, shared=lw.shared_cat(),
                           ids=ids, weights=weights, route_kw=c.route_kw)


def oracle_scores(lw: inputs.LayerWeights, xb: np.ndarray) -> np.ndarray:
    """Per-expert selection scores the oracle ranks (for near-tie detection)."""
    c = lw.cfg
    lg = formats.bf16_bits_to_f32(xb) @ lw.router.T
    if c.routing == "sigmoid_group":
        return 1.0 / (1.0 + np.exp(-lg.astype(np.float64)))
    return lg.astype(np.float64)


def ids_match_except_near_ties(gpu_ids: np.ndarray, ref_ids: np.ndarray, scores: np.ndarray, k: int,
                               rel: float = 1e-5) -> np.ndarray:
    """Rows whose id SETS differ although the k-th / (k+1)-th scores are not near-tied."""
    bad = []
    for t in range(ref_ids.shape[0]):
        if set(gpu_ids[t].tolist()) == set(ref_ids[t].tolist()):
            continue
        s = np.sort(scores[t])[::-1]
        gap = abs(s[k - 1] - s[k]) if k < s.size else np.inf
        if gap > rel * max(abs(s[k - 1]), 1e-12):
            bad.append(t)
    return np.asarray(bad, dtype=np.int64)


__all__ = ["TOL", "small_cfg", "gpu_layer", "x_device", "rel_err_rows", "oracle_forward", "oracle_scores",
           "ids_match_except_near_ties", "routing"]
