"""Drop-in for ``ccut.experts.pipeline`` (``ExpertPipeline``, ``PipelineMetrics``,
``RouteHistory``) over HBM-resident MoE layers.

The reference's pipeline (``ccut/experts/pipeline.py:87-208``) streams each step's experts
from disk: a speculative stage guesses the next experts from the recent routing, a prefetch
stage reads and dequantizes them into a ring, and the compute stage routes, runs the experts
and adds the shared experts.  Here every expert already sits packed in HBM (``MoeLayer``), so
``step`` is one ``ccut_moe_forward`` call and there is nothing to prefetch or to guess: the
constructor's streaming parameters are accepted and have no effect, and the prefetch and
speculation counters of ``PipelineMetrics`` stay zero.  ``step`` keeps the reference's
arguments, return type and errors; its ``reader`` is the resident layer, a ``{layer:
MoeLayer}`` mapping or an object with ``moe_layer(layer)`` (as for ``blocks.moe.moe_forward``).
"""

from __future__ import annotations

import time
from collections import deque
from dataclasses import dataclass
from typing import Iterable

import torch

from ccut_b200.blocks.moe import _resolve_layer, _x_bf16

__all__ = ["PipelineMetrics", "RouteHistory", "ExpertPipeline"]


@dataclass
class PipelineMetrics:
    """The reference's step counters (``ccut/experts/pipeline.py:34-64``)."""

    compute_ns: int = 0
    prefetch_ns: int = 0
    overlap_ns: int = 0
    steps: int = 0
    speculative_correct: int = 0
    speculative_total: int = 0
    ring_hits: int = 0
    ring_misses: int = 0
    ring_evicted: int = 0

    def overlap_ratio(self) -> float:
        return self.overlap_ns / self.compute_ns if self.compute_ns > 0 else 0.0

    def speculative_accept_rate(self) -> float:
        return self.speculative_correct / self.speculative_total if self.speculative_total > 0 else 0.0

    def to_dict(self) -> dict:
        return {"compute_ns": self.compute_ns, "prefetch_ns": self.prefetch_ns, "overlap_ns": self.overlap_ns,
                "overlap_ratio": round(self.overlap_ratio(), 4), "steps": self.steps,
                "spec_accept_rate": round(self.speculative_accept_rate(), 4), "ring_hits": self.ring_hits,
                "ring_misses": self.ring_misses}


class RouteHistory:
    """The last ``window`` steps' expert sets; ``predict(k)`` returns the ``k`` experts seen in
    the most steps, ties in the order the experts were first counted (the rule of
    ``ccut/experts/pipeline.py:66-85``)."""

    def __init__(self, window: int = 4):
        self.window = window
        self._steps: deque = deque(maxlen=window)

    def record(self, topk_ids: Iterable[int]) -> None:
        self._steps.append({int(e) for e in topk_ids})

    def predict(self, top_k: int) -> list[int]:
        seen: dict[int, int] = {}
        for experts in self._steps:
            for e in experts:
                seen[e] = seen.get(e, 0) + 1
        ranked = sorted(seen, key=lambda e: -seen[e])  # stable: first counted wins a tie
        return ranked[:top_k]


class ExpertPipeline:
    """``step(layer, x, gate_w, top_k, norm_topk_prob, shared_projs, shared_gate)`` over resident
    layers: router, top-k, experts, weighted combine and shared experts in one GPU call."""

    def __init__(self, reader, num_workers: int = 2, speculative_window: int = 4, prefetch_steps_ahead: int = 2,
                 metrics_enabled: bool = True):
        self.reader = reader
        self.num_workers = num_workers
        self.prefetch_steps_ahead = prefetch_steps_ahead
        self.metrics = PipelineMetrics() if metrics_enabled else None
        self.history = RouteHistory(window=speculative_window)

    def step(self, layer: int, x, gate_w, top_k: int = 8, norm_topk_prob: bool = True, shared_projs=None,
             shared_gate: float = 1.0):
        """``x [seq, hidden]`` -> fp32 ``[seq, hidden]`` (numpy in, numpy out).  ``gate_w`` must be
        the router the resident layer holds, and ``top_k`` / ``norm_topk_prob`` its routing;
        shared experts are added when ``shared_projs`` is given, scaled by ``shared_gate``."""
        L = _resolve_layer(self.reader, layer)
        if int(top_k) != L.top_k:
            raise ValueError(f"top_k = {top_k} but the resident layer routes top-{L.top_k}")
        if L.routing in ("softmax_topk", "topk_softmax") and bool(norm_topk_prob) != (L.routing == "topk_softmax"):
            raise ValueError(f"norm_topk_prob = {norm_topk_prob} but the resident layer uses {L.routing}")
        has_shared = shared_projs is not None and (not hasattr(shared_projs, "__contains__")
                                                   or "gate_proj" in shared_projs)
        if has_shared != (L.num_slices > 0):
            raise ValueError("shared experts given / not given, but the resident layer has "
                             f"{L.num_slices} shared slices")
        gw = gate_w if isinstance(gate_w, torch.Tensor) else torch.as_tensor(gate_w, dtype=torch.float32)
        if tuple(gw.shape) != tuple(L.router.shape):
            raise ValueError(f"gate_w must be {tuple(L.router.shape)}, got {tuple(gw.shape)}")
        xt, was_np = _x_bf16(x, L.hidden, L.device)
        t0 = time.monotonic_ns()
        gate0 = L.shared_gate
        L.shared_gate = L.desc.shared_gate = float(shared_gate)
        try:
            out, routing = L.forward(xt, out_dtype=torch.float32, return_routing=True)
            ids = routing.ids.cpu()  # waits for the step
        finally:
            L.shared_gate = L.desc.shared_gate = gate0
        if ids.shape[0]:
            self.history.record(ids[0].tolist())
        if self.metrics is not None:
            self.metrics.compute_ns += time.monotonic_ns() - t0
            self.metrics.steps += 1
        return out.cpu().numpy() if was_np else out

    def close(self) -> None:
        return None
