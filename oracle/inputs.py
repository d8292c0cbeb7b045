"""Seeded synthetic layers viewed through the oracle (test infrastructure only).

The tensors themselves come from ``ccut_b200.synthetic`` (the seeded random-init
generator that the benchmark also uses, so the checker and the measured path see the
same inputs).  This module adds the oracle's fp32 dequant of each matrix
(``oracle.formats``) and the expert lookup that ``oracle.moe.moe_forward`` consumes.
"""

from __future__ import annotations

import numpy as np

from ccut_b200.synthetic import (  # noqa: F401  (re-exported)
    CONFIGS,
    AwqMatrix,
    ExpertWeights,
    Fp8ChannelMatrix,
    Fp8Matrix,
    Int4SymMatrix,
    LayerWeights,
    MoeLayerConfig,
    scaled_config,
)
from ccut_b200 import synthetic
from oracle import formats

__all__ = ["CONFIGS", "MoeLayerConfig", "AwqMatrix", "Fp8Matrix", "Fp8ChannelMatrix", "Int4SymMatrix",
           "ExpertWeights", "OracleLayer", "make_layer", "scaled_config", "dequant"]


def dequant(mat) -> np.ndarray:
    """fp32 [K, N] ([in, out], the layout ``expert_ffn`` consumes) of one checkpoint matrix."""
    if isinstance(mat, AwqMatrix):
        return formats.awq_dequant(mat.qweight, mat.qzeros, mat.scales)
    if isinstance(mat, Fp8Matrix):
        return np.ascontiguousarray(formats.fp8_block_dequant(mat.weight, mat.scale).T)
    if isinstance(mat, Fp8ChannelMatrix):
        return np.ascontiguousarray(formats.fp8_channel_dequant(mat.weight, mat.scale).T)
    if isinstance(mat, Int4SymMatrix):
        return np.ascontiguousarray(formats.int4_sym_dequant(mat.weight, mat.scale).T)
    raise TypeError(f"unknown matrix type {type(mat).__name__}")


class OracleLayer:
    """A ``synthetic.LayerWeights`` plus cached oracle dequant lookups."""

    def __init__(self, lw: LayerWeights):
        self.lw = lw
        self._cache: dict = {}

    def __getattr__(self, name):
        return getattr(self.lw, name)

    def w_lookup(self, e: int):
        if e not in self._cache:
            ew = self.lw.experts[e]
            self._cache[e] = (dequant(ew.gate), dequant(ew.up), dequant(ew.down))
        return self._cache[e]

    def shared_cat(self):
        """Shared experts as one concatenated SwiGLU MLP (inter = S * shared_inter)."""
        if not self.lw.shared:
            return None
        if "shared" not in self._cache:
            parts = [(dequant(s.gate), dequant(s.up), dequant(s.down)) for s in self.lw.shared]
            self._cache["shared"] = (
                np.concatenate([p[0] for p in parts], axis=1),
                np.concatenate([p[1] for p in parts], axis=1),
                np.concatenate([p[2] for p in parts], axis=0),
            )
        return self._cache["shared"]


def make_layer(cfg, seed: int = 0) -> OracleLayer:
    return OracleLayer(synthetic.make_layer(cfg, seed))
