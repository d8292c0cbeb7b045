"""Next-token sampling for the engine backend, on the device that holds the logits.

``temperature_topk`` restates the reference's probability transform
(``ccut/blocks/heads.py:76-126``) with torch ops: temperature, then top-k (values below the
k-th largest dropped, ties kept), min-p (probabilities below ``min_p * p_max`` dropped), top-p
(over the descending order, the first position whose normalised cumulative sum exceeds
``top_p`` and every later one dropped, unless that first position is the top token, in which
case nothing is dropped, as in the reference), then the softmax with the ``1e-30`` clamp.
Dropped entries are set to ``-1e30`` as in the reference.  ``typical_p`` is not applied (the
engine's sampling call, ``ccut/engine.py:335-352``, does not pass it).

``sample`` picks one token: ``temperature <= 0`` is greedy (arg-max, ties to the lowest
index), which is what ``L1Backend.generate`` does without a sampler
(``ccut/models/backend_transformers.py:96-124``); the reference's ``temperature_topk`` itself leaves
logits unscaled at temperature 0 and samples them.  Otherwise one draw from the transformed
distribution with the backend's seeded ``torch.Generator``.
"""

from __future__ import annotations

import numpy as np
import torch

__all__ = ["temperature_topk", "sample"]

_NEG = -1e30


def temperature_topk(logits, temperature: float, top_k: int = 0, top_p: float = 1.0, min_p: float = 0.0):
    """``logits [rows, vocab]`` -> probabilities ``[rows, vocab]`` float32 (numpy in, numpy out)."""
    was_np = not isinstance(logits, torch.Tensor)
    x = torch.from_numpy(np.array(logits, dtype=np.float32)) if was_np else logits.float().clone()
    if x.dim() != 2:
        raise ValueError("logits must be [rows, vocab]")
    V = x.shape[1]
    if temperature > 0:
        x = x / float(temperature)
    if top_k and 0 < top_k < V:
        thr = torch.topk(x, int(top_k), dim=1).values[:, -1:]
        x = torch.where(x < thr, torch.full_like(x, _NEG), x)
    if min_p and 0 < min_p < 1.0:
        e = torch.exp(x - x.max(dim=1, keepdim=True).values)
        p = e / torch.clamp(e.sum(dim=1, keepdim=True), min=1e-30)
        pmax = p.max(dim=1, keepdim=True).values
        x = torch.where(p >= float(min_p) * pmax, x, torch.full_like(x, _NEG))
    if top_p and 0 < top_p < 1.0:
        sx, order = torch.sort(x, dim=1, descending=True)
        csum = torch.cumsum(torch.exp(sx - sx[:, :1]), dim=1)
        csum = csum / torch.clamp(csum[:, -1:], min=1e-30)
        cond = csum > float(top_p)
        first = torch.argmax(cond.to(torch.int32), dim=1, keepdim=True)  # first True; 0 when none
        rank = torch.arange(V, device=x.device)[None, :]
        drop = (rank >= first) & (first > 0)
        x = x.scatter(1, order, torch.where(drop, torch.full_like(sx, _NEG), sx))
    e = torch.exp(x - x.max(dim=1, keepdim=True).values)
    p = e / torch.clamp(e.sum(dim=1, keepdim=True), min=1e-30)
    return p.numpy() if was_np else p


def sample(logits: torch.Tensor, params: dict | None, generator: torch.Generator | None = None) -> int:
    """One token id from ``logits [vocab]`` under the engine's sampling parameters
    (``temperature`` default 1.0, ``top_k`` 0, ``top_p`` 1.0, ``min_p`` 0.0)."""
    params = params or {}
    temp = float(params.get("temperature", 1.0))
    row = logits.reshape(1, -1)
    if temp <= 0:
        return int(torch.argmax(row[0]).item())
    p = temperature_topk(row, temp, int(params.get("top_k", 0) or 0), float(params.get("top_p", 1.0)),
                         float(params.get("min_p", 0.0) or 0.0))
    return int(torch.multinomial(p[0], 1, generator=generator).item())
