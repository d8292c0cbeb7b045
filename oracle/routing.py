"""Router top-k restatements (CPU, test infrastructure only).

Modes (the ``mode`` codes the C-ABI uses, ``include/ccut_moe.h``):

0 ``softmax_topk``   softmax over all E experts, then top-k, no renormalisation
                     (``norm_topk_prob=False``, DeepSeek-V2-Lite; ``ccut/blocks/moe.py:80-84``)
1 ``topk_softmax``   top-k of the raw logits, then softmax over the k values
                     (``norm_topk_prob=True``, Qwen3; ``ccut/blocks/moe.py:85-89``)
2 ``sigmoid_group``  DeepSeek-V3 grouped sigmoid routing (no reference implementation;
                     restated from the published model description, parity unpinned)
"""

from __future__ import annotations

import numpy as np

__all__ = ["MODES", "topk", "topk_softmax", "grouped_sigmoid_topk", "route"]

MODES = {"softmax_topk": 0, "topk_softmax": 1, "sigmoid_group": 2}


def topk(x: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    """Per-row top-k, values descending, ties to the lowest column index.

    Follows ``ccut/blocks/moe.py:46-68`` (repeated arg-max with a strict ``>``, so the
    first maximal column wins).  A stable descending sort yields the same selection for
    every row whose values exceed the reference's ``-1e30`` sentinel."""
    x = np.asarray(x)
    order = np.argsort(-x, axis=1, kind="stable")[:, :k]
    vals = np.take_along_axis(x, order, axis=1)
    return vals.astype(x.dtype), order.astype(np.int64)


def topk_softmax(logits: np.ndarray, k: int, norm_topk_prob: bool = True) -> tuple[np.ndarray, np.ndarray]:
    """Routing weights and expert ids, ``ccut/blocks/moe.py:71-89`` (fp32 throughout)."""
    logits = np.asarray(logits, dtype=np.float32)
    if not norm_topk_prob:
        e = np.exp(logits - logits.max(axis=1, keepdims=True))
        p = e / np.maximum(e.sum(axis=1, keepdims=True), np.float32(1e-30))
        vals, idx = topk(p, k)
        return vals.astype(np.float32), idx
    vals, idx = topk(logits, k)
    v = vals - vals.max(axis=1, keepdims=True)
    ex = np.exp(v)
    w = ex / np.maximum(ex.sum(axis=1, keepdims=True), np.float32(1e-30))
    return w.astype(np.float32), idx


def grouped_sigmoid_topk(
    logits: np.ndarray,
    k: int,
    n_group: int,
    topk_group: int,
    routed_scaling: float = 1.0,
    bias: np.ndarray | None = None,
    norm_topk_prob: bool = True,
) -> tuple[np.ndarray, np.ndarray]:
    """DeepSeek-V3 routing (restatement; the reference has only softmax routing).

    1. ``s = sigmoid(logits)`` (fp32); ``c = s + bias`` is the selection score.
    2. Group score = sum of the two largest ``c`` in each of ``n_group`` equal groups.
    3. Keep the ``topk_group`` best groups (ties -> lower group index).
    4. Top-k of ``c`` over the kept groups' experts (ties -> lower expert index).
    5. Weights = ``s`` at the chosen experts, divided by their sum (+1e-20) when
       ``norm_topk_prob``, times ``routed_scaling``.
    Ids are ordered by descending ``c``."""
    logits = np.asarray(logits, dtype=np.float32)
    T, E = logits.shape
    if E % n_group:
        raise ValueError("num_experts must be divisible by n_group")
    s = (1.0 / (1.0 + np.exp(-logits.astype(np.float64)))).astype(np.float32)
    c = s if bias is None else (s + np.asarray(bias, dtype=np.float32)[None, :]).astype(np.float32)
    per = E // n_group
    cg = c.reshape(T, n_group, per)
    top2 = -np.sort(-cg, axis=2)[:, :, :2]
    gscore = top2.sum(axis=2, dtype=np.float32)
    gsel = np.argsort(-gscore, axis=1, kind="stable")[:, :topk_group]
    keep = np.zeros((T, n_group), dtype=bool)
    np.put_along_axis(keep, gsel, True, axis=1)
    masked = np.where(np.repeat(keep, per, axis=1), c, -np.inf).astype(np.float32)
    _, idx = topk(masked, k)
    w = np.take_along_axis(s, idx, axis=1).astype(np.float32)
    if norm_topk_prob:
        w = w / (w.sum(axis=1, keepdims=True, dtype=np.float32) + np.float32(1e-20))
    w = (w * np.float32(routed_scaling)).astype(np.float32)
    return w, idx


def route(logits: np.ndarray, k: int, mode: str, **kw) -> tuple[np.ndarray, np.ndarray]:
    """Dispatch on the routing mode name (see module docstring)."""
    if mode == "softmax_topk":
        return topk_softmax(logits, k, norm_topk_prob=False)
    if mode == "topk_softmax":
        return topk_softmax(logits, k, norm_topk_prob=True)
    if mode == "sigmoid_group":
        return grouped_sigmoid_topk(logits, k, **kw)
    raise ValueError(f"unknown routing mode {mode!r}")
