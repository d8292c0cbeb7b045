"""RoPE inverse-frequency tables (host side, numpy; no torch).

``rope_table`` follows the reference's ``build_rope`` (``ccut/blocks/rope.py:88-127``) for no
scaling and ``linear`` scaling; ``yarn_rope_table`` / ``yarn_mscale`` are YaRN as the MLA
models' configs (DeepSeek-V2 / V3) define it.  ``ccut_b200.model`` re-exports all three.
"""

from __future__ import annotations

import math

import numpy as np

__all__ = ["rope_table", "yarn_mscale", "yarn_rope_table"]


def rope_table(head_dim: int, rope_theta: float, rope_scaling: dict | None = None) -> tuple[np.ndarray, float]:
    """``(inv_freq [head_dim / 2] float32, attention_factor)`` of the reference's ``build_rope``
    (``ccut/blocks/rope.py:88-127``) for no scaling and ``linear`` scaling, computed with the same
    float32 operations.  Other scalings: pass the table ``build_rope`` returns to ``MoeDecoder``."""
    rs = rope_scaling or {}
    stype = (rs.get("type") or "none").casefold()
    factor = float(rs.get("factor", 1.0))
    inv = 1.0 / (rope_theta ** (np.arange(0, head_dim, 2, dtype=np.float32) / head_dim))
    if stype == "none" or factor <= 1.0:
        return inv.astype(np.float32), 1.0
    if stype == "linear":
        return (inv / factor).astype(np.float32), 1.0
    raise NotImplementedError(f"rope scaling {stype!r}: pass inv_freq and attention_factor from build_rope")


def yarn_mscale(factor: float, mscale: float = 1.0) -> float:
    """YaRN's attention temperature ``0.1 * mscale * ln(factor) + 1`` (1 for ``factor <= 1``)."""
    return 1.0 if factor <= 1.0 else 0.1 * float(mscale) * math.log(factor) + 1.0


def yarn_rope_table(dim: int, rope_theta: float, rope_scaling: dict,
                    max_position_embeddings: int | None = None) -> tuple[np.ndarray, float]:
    """``(inv_freq [dim / 2] float32, cos / sin factor)`` of YaRN as DeepSeek-V2 / V3 configs
    use it (Peng et al. 2023, "YaRN: Efficient Context Window Extension of Large Language
    Models"): the rotation dims whose wavelength fits ``beta_fast`` rotations in the original
    context keep their frequency, those below ``beta_slow`` rotations are divided by ``factor``,
    and a linear ramp over the dims between (bounds rounded outwards) mixes the two; the
    factor is ``attention_factor`` if given, else ``yarn_mscale(factor, mscale) /
    yarn_mscale(factor, mscale_all_dim)`` when both keys are set, else ``yarn_mscale(factor)``.
    (The reference's own ``build_rope`` has a different yarn formula; it serves no MLA model.)"""
    rs = dict(rope_scaling)
    orig = int(rs["original_max_position_embeddings"])
    factor = rs.get("factor")
    factor = float(factor) if factor is not None else float(max_position_embeddings) / orig
    beta_fast, beta_slow = float(rs.get("beta_fast") or 32.0), float(rs.get("beta_slow") or 1.0)
    base = float(rope_theta)

    def corr_dim(rotations: float) -> float:
        return dim * math.log(orig / (rotations * 2 * math.pi)) / (2 * math.log(base))

    low = max(math.floor(corr_dim(beta_fast)), 0)
    high = min(math.ceil(corr_dim(beta_slow)), dim - 1)
    if low == high:
        high += 0.001
    ramp = np.clip((np.arange(dim // 2, dtype=np.float32) - np.float32(low)) / np.float32(high - low), 0, 1)
    keep = (1 - ramp).astype(np.float32)  # 1: the original frequency
    pos_freqs = np.float32(base) ** (np.arange(0, dim, 2, dtype=np.float32) / np.float32(dim))
    inv = (1.0 / (np.float32(factor) * pos_freqs)) * (1 - keep) + (1.0 / pos_freqs) * keep
    af = rs.get("attention_factor")
    if af is None:
        m, m_all = rs.get("mscale"), rs.get("mscale_all_dim")
        af = yarn_mscale(factor, m) / yarn_mscale(factor, m_all) if m and m_all else yarn_mscale(factor)
    return inv.astype(np.float32), float(af)
