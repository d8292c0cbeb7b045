"""MoE expert forward restatement (CPU, test infrastructure only).

``expert_ffn``   SwiGLU FFN of one expert, ``ccut/blocks/moe.py:122-141``
``silu_mul``     ``silu(gate) * up`` in float64, stored fp32, ``ccut/quant/kernels.py:219-231``
``group_tokens`` expert -> token list in first-appearance order,
                 ``ccut/models/generic.py:367-371`` / ``ccut/blocks/moe.py:164-170``
``moe_combine``  weighted scatter-add, ``ccut/blocks/moe.py:144-174``
``moe_forward``  router -> top-k -> experts -> combine -> shared experts,
                 ``ccut/models/generic.py:348-386`` (shared experts as one concatenated
                 SwiGLU MLP, ``ccut/models/generic.py:380-385``; optional scalar gate as in
                 ``ccut/experts/pipeline.py:182-190``)
"""

from __future__ import annotations

from typing import Callable

import numpy as np

from oracle import routing

__all__ = ["silu_mul", "expert_ffn", "group_tokens", "moe_combine", "moe_forward"]


def silu_mul(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """``out = gate / (1 + exp(-gate)) * up`` in float64, rounded to fp32."""
    g = np.asarray(gate, dtype=np.float64)
    u = np.asarray(up, dtype=np.float64)
    with np.errstate(over="ignore"):
        return ((g / (1.0 + np.exp(-g))) * u).astype(np.float32)


def expert_ffn(x: np.ndarray, wg: np.ndarray, wu: np.ndarray, wd: np.ndarray) -> np.ndarray:
    """``down(silu(x @ wg) * (x @ wu))`` with fp32 matmuls; ``wg``/``wu`` [H, I], ``wd`` [I, H]."""
    x = np.asarray(x, dtype=np.float32)
    gate = x @ wg
    up = x @ wu
    return silu_mul(gate, up) @ wd


def group_tokens(ids: np.ndarray) -> dict[int, list[int]]:
    """Expert id -> tokens routed to it, experts in order of first appearance scanning
    ``(t, j)`` row-major, tokens ascending."""
    by_e: dict[int, list[int]] = {}
    T, k = ids.shape
    for t in range(T):
        for j in range(k):
            by_e.setdefault(int(ids[t, j]), []).append(t)
    return by_e


def moe_combine(
    x: np.ndarray,
    ids: np.ndarray,
    weights: np.ndarray,
    w_lookup: Callable[[int], tuple[np.ndarray, np.ndarray, np.ndarray]],
) -> np.ndarray:
    """``y[t] = sum_j w[t, j] * expert_{ids[t, j]}(x[t])`` in fp32, scatter-add order as in
    the reference (experts in first-appearance order, tokens ascending)."""
    x = np.asarray(x, dtype=np.float32)
    T, H = x.shape
    out = np.zeros((T, H), dtype=np.float32)
    for eid, toks in group_tokens(ids).items():
        wg, wu, wd = w_lookup(eid)
        rows = np.asarray(toks, dtype=np.int64)
        y = expert_ffn(x[rows], wg, wu, wd)
        # weight of token t for this expert: first j with ids[t, j] == eid
        jpos = np.argmax(ids[rows] == eid, axis=1)
        w = weights[rows, jpos].astype(np.float32)
        for i, t in enumerate(toks):
            out[t] += w[i] * y[i]
    return out


def moe_forward(
    x: np.ndarray,
    router_w: np.ndarray,
    top_k: int,
    mode: str,
    w_lookup: Callable[[int], tuple[np.ndarray, np.ndarray, np.ndarray]],
    shared: tuple[np.ndarray, np.ndarray, np.ndarray] | None = None,
    shared_gate: float = 1.0,
    ids: np.ndarray | None = None,
    weights: np.ndarray | None = None,
    route_kw: dict | None = None,
) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Whole MoE layer on fp32 activations ``x`` [T, H].

    ``router_w`` fp32 [E, H]; ``w_lookup(e)`` returns dequantized ``(wg, wu, wd)`` in
    [in, out] layout; ``shared`` is the concatenated shared-expert MLP (or None).
    ``ids`` / ``weights`` override the router (used to compare the expert and combine
    stages on exactly the routing another implementation chose).
    Returns ``(out fp32 [T, H], ids int64 [T, k], weights fp32 [T, k])``."""
    x = np.asarray(x, dtype=np.float32)
    if ids is None:
        logits = x @ np.asarray(router_w, dtype=np.float32).T
        weights, ids = routing.route(logits, top_k, mode, **(route_kw or {}))
    out = moe_combine(x, ids, weights, w_lookup)
    if shared is not None:
        sg, su, sd = shared
        s_out = expert_ffn(x, sg, su, sd)
        if shared_gate == 1.0:
            out += s_out
        else:
            out += np.float32(shared_gate) * s_out
    return out, ids, weights
