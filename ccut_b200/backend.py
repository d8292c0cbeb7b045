"""Engine backend over ``MoeDecoder``: the served path of the reference's ``Engine`` reaches the
GPU decoder through it.

``Engine._backend_step`` (``ccut/engine.py:305-333``) calls, for every scheduled request,
``backend.generate_step(prompt[:prefill_consumed] + generated, sampling_params=...)`` and takes
one token id back (errors evict that request).  ``GenericBackend`` answers that call:

* it keeps up to ``max_seqs`` sequence caches (``KvCache``, bf16 k / v in HBM) keyed by the
  token ids they hold.  A call reuses the cache with the longest common prefix of its ids (at
  least one token is always recomputed, for its logits), truncates it there and runs the rest
  as prefill chunks of at most ``prefill_chunk`` tokens.  A request that grows by one token per
  step therefore runs one token per step; chunked prefill runs each new chunk once; a request
  that diverges from a cached one (a shared prompt, a retried step) keeps the shared part.
  With all slots held, the least recently used cache is taken;
* it samples the next token from the last position's logits on the device
  (``ccut_b200.sampling.sample``: greedy at ``temperature <= 0``, else the reference's
  temperature / top-k / min-p / top-p transform and one draw from a seeded generator).

``generate_batch([(input_ids, sampling_params), ...])`` answers a whole engine step at once
(the loop of ``_backend_step`` as one call): the requests' new ids run through one decoder
pass per prefill chunk, so their MoE blocks see all the step's tokens together.

``generate`` and ``forward_step`` give the interface of the reference's fallback backend
(``L1Backend``, ``ccut/models/backend_transformers.py:31-124``), which the engine uses when a
backend has no ``generate_step``: ``forward_step(input_ids, past)`` returns the logits of the
last id and the cache to pass back, ``generate`` loops it with a ``sampling(logits, position)``
callable (greedy by default) and stops at ``eos_token_id``.
"""

from __future__ import annotations

from typing import Any, Callable

import numpy as np
import torch

from ccut_b200.model import KvCache, MoeDecoder
from ccut_b200.sampling import sample

__all__ = ["GenericBackend", "common_prefix"]


def common_prefix(a: list[int], b: list[int]) -> int:
    """Length of the longest common prefix of two id lists."""
    n = min(len(a), len(b))
    if a[:n] == b[:n]:
        return n
    x = np.asarray(a[:n], dtype=np.int64)
    y = np.asarray(b[:n], dtype=np.int64)
    return int(np.argmax(x != y))


class _Seq:
    def __init__(self, cache: KvCache):
        self.cache = cache
        self.ids: list[int] = []


class GenericBackend:
    """``generate_step`` backend for the reference's ``Engine`` over a ``MoeDecoder``."""

    tier = "L0"

    def __init__(self, model: MoeDecoder, max_seqs: int = 4, max_len: int = 4096, prefill_chunk: int = 4096,
                 seed: int = 0, eos_token_id: int | None = None, pool: bool = False):
        """``pool``: keep the sequence caches in one ``KvPool``, so that a decode step of several
        requests (``generate_batch``) runs one attention launch per layer."""
        if max_seqs < 1 or max_len < 1 or prefill_chunk < 1:
            raise ValueError("max_seqs, max_len and prefill_chunk must be positive")
        self.model = model
        self._pool = model.new_pool(max_seqs, max_len) if pool else None
        self.max_seqs, self.max_len, self.prefill_chunk = int(max_seqs), int(max_len), int(prefill_chunk)
        self.eos_token_id = eos_token_id
        self._seqs: list[_Seq] = []  # least recently used first
        self._gen = torch.Generator(device=model.device)
        self._gen.manual_seed(int(seed))
        self.tokens_run = 0  # positions the decoder computed (prefix reuse skips the rest)

    # ---- sequence caches ---------------------------------------------------------------
    def _acquire(self, ids: list[int], taken: list) -> tuple[_Seq, int]:
        """The cache to run ``ids`` in (not one of ``taken``) and how many of its positions stay."""
        best, best_p = None, 0
        for s in self._seqs:
            if any(s is t for t in taken):
                continue
            p = common_prefix(s.ids, ids)
            if p > best_p:
                best, best_p = s, p
        reuse = min(best_p, len(ids) - 1)
        if best is None or reuse == 0:
            reuse = 0
            if len(self._seqs) < self.max_seqs:
                cache = (self._pool.cache(len(self._seqs)) if self._pool is not None
                         else self.model.new_cache(self.max_len))
                best = _Seq(cache)
            else:
                free = [s for s in self._seqs if not any(s is t for t in taken)]
                if not free:
                    raise ValueError(f"a batch of more than max_seqs={self.max_seqs} sequences")
                best = free[0]  # least recently used
        if any(best is s for s in self._seqs):
            self._seqs.remove(best)
        self._seqs.append(best)
        return best, reuse

    def _check(self, input_ids) -> list[int]:
        ids = [int(t) for t in input_ids]
        if not ids:
            raise ValueError("generate_step needs at least one input id")
        if len(ids) > self.max_len:
            raise ValueError(f"{len(ids)} ids exceed the backend's max_len of {self.max_len}")
        return ids

    def logits_batch(self, id_lists) -> list:
        """fp32 logits ``[vocab]`` of the last id of every list, the lists run together: each
        call of the decoder takes the next ``prefill_chunk`` ids (at most) of every list that
        has ids left, so decoding sequences share their MoE passes."""
        lists = [self._check(ids) for ids in id_lists]
        seqs: list[_Seq] = []
        pos: list[int] = []
        for ids in lists:
            seq, reuse = self._acquire(ids, seqs)
            seq.cache.truncate(min(reuse, seq.cache.length))
            seq.ids = ids[: seq.cache.length]
            seqs.append(seq)
            pos.append(reuse)
        out: list = [None] * len(lists)
        while True:
            todo = [j for j in range(len(lists)) if pos[j] < len(lists[j])]
            if not todo:
                return out
            ends = [min(len(lists[j]), pos[j] + self.prefill_chunk) for j in todo]
            logits = self.model.forward_batch(
                [(lists[j][pos[j]: e], seqs[j].cache, pos[j]) for j, e in zip(todo, ends)])
            for j, e, lg in zip(todo, ends, logits):
                self.tokens_run += e - pos[j]
                seqs[j].ids = lists[j][:e]
                pos[j] = e
                if e == len(lists[j]):
                    out[j] = lg

    def logits_for(self, input_ids) -> torch.Tensor:
        """fp32 logits ``[vocab]`` of the last of ``input_ids`` (runs what no cache holds)."""
        return self.logits_batch([input_ids])[0]

    # ---- Engine interface ----------------------------------------------------------------
    def generate_step(self, input_ids, sampling_params: dict | None = None) -> int:
        return sample(self.logits_for(input_ids), sampling_params, self._gen)

    def generate_batch(self, requests) -> list[int]:
        """``requests`` = ``[(input_ids, sampling_params), ...]``, one per scheduled request of an
        engine step (at most ``max_seqs``): the next token of each, from one batched pass."""
        requests = list(requests)
        logits = self.logits_batch([r[0] for r in requests])
        return [sample(lg, r[1], self._gen) for lg, r in zip(logits, requests)]

    # ---- L1Backend interface -------------------------------------------------------------
    def forward_step(self, input_ids, past: Any = None) -> tuple[torch.Tensor, KvCache]:
        """``input_ids`` the whole sequence so far; ``past`` the cache a previous call returned
        (its positions must be a prefix of ``input_ids``) or None.  Returns ``(logits [1, vocab],
        cache)``."""
        ids = [int(t) for t in input_ids]
        if not ids:
            raise ValueError("forward_step needs at least one input id")
        cache = past if past is not None else self.model.new_cache(self.max_len)
        if len(ids) > cache.max_len:
            raise ValueError(f"{len(ids)} ids exceed the cache's max_len of {cache.max_len}")
        start = min(cache.length, len(ids) - 1)
        cache.truncate(start)
        logits = None
        for c0 in range(start, len(ids), self.prefill_chunk):
            c1 = min(len(ids), c0 + self.prefill_chunk)
            logits = self.model.forward(ids[c0:c1], cache, c0)
            self.tokens_run += c1 - c0
        return logits.reshape(1, -1), cache

    def generate(self, token_ids, max_tokens: int, on_token: Callable[[int], None] | None = None,
                 sampling: Callable[[Any, int], int] | None = None) -> list[int]:
        if sampling is None:
            def sampling(logits, pos):
                return int(torch.argmax(logits.reshape(-1)).item())
        past = None
        current = [int(t) for t in token_ids]
        out: list[int] = []
        for _ in range(int(max_tokens)):
            logits, past = self.forward_step(current, past)
            tok = int(sampling(logits, len(out)))
            out.append(tok)
            if on_token is not None:
                on_token(tok)
            current.append(tok)
            if self.eos_token_id is not None and tok == self.eos_token_id:
                break
        return out
