"""RoPE inverse-frequency tables (host side, numpy; no torch).

``rope_table`` follows the reference's ``build_rope`` (``ccut/blocks/rope.py:88-127``) for no
scaling and ``linear`` scaling; ``yarn_rope_table`` / ``yarn_mscale`` are YaRN as the MLA
models' configs (DeepSeek-V2 / V3) define it.  ``ccut_b200.model`` re-exports all three.
"""

from __future__ import annotations

import math

import numpy as np

__all__ = ["rope_table", "yarn_mscale", "yarn_rope_table"]


def _reference_yarn(dim: int, base: float, factor: float, beta_fast: float, beta_slow: float,
                    attention_factor) -> tuple[np.ndarray, float]:
    """The reference's own yarn table (``_yarn_get_scaled_factors``, ``ccut/blocks/rope.py:42-85``,
    with its correction range ``:30-39``), which differs from published YaRN: the frequencies
    are divided by ``factor / (0.1 factor ln(factor) + 1)`` (by ``factor`` when ``factor <=
    1.5``) with a smoothstep weight over the wavelengths between ``base ** (1 / high)`` and
    ``base ** (1 / low)``, ``low = floor(base sqrt(beta_fast / (1 - exp(-beta_fast / dim)))) /
    0.1`` and ``high = ceil(base sqrt(beta_slow / (1 - exp(-beta_slow / dim)))) / 32``; the
    attention factor is ``attention_factor`` or ``0.1 factor ln(factor) + 1``.  Same float32
    operations, so the table is the reference's."""
    mscale = 0.1 * factor * math.log(factor) + 1.0
    af = float(attention_factor) if attention_factor is not None else mscale
    div = factor / mscale if factor > 1.5 else factor
    low = math.floor(base * (beta_fast / (1 - math.exp(-beta_fast / dim))) ** 0.5) / 0.1
    high = math.ceil(base * (beta_slow / (1 - math.exp(-beta_slow / dim))) ** 0.5) / 32.0
    idx = np.arange(0, dim, 2, dtype=np.float32) / dim
    inv = 1.0 / (base ** idx)
    wave = base ** idx
    lo_w = base ** (1.0 / high) if high > 0 else 0.0
    hi_w = base ** (1.0 / low) if low > 0 else float("inf")
    t = np.clip((wave - lo_w) / (hi_w - lo_w + 1e-12), 0.0, 1.0)
    w = t * t * (3.0 - 2.0 * t)
    return (inv * (1.0 - w) + inv / div * w).astype(np.float32), af


def rope_table(head_dim: int, rope_theta: float, rope_scaling: dict | None = None) -> tuple[np.ndarray, float]:
    """``(inv_freq [head_dim / 2] float32, attention_factor)`` of the reference's ``build_rope``
    (``ccut/blocks/rope.py:88-127``), computed with the same float32 operations: no scaling,
    ``linear`` (frequencies divided by ``factor``), ``dynamic`` (the plain table: the reference
    scales nothing at apply time either) and the reference's own ``yarn`` (``_reference_yarn``).
    The reference's layer forward passes no scaling type to ``apply_rope``, so the attention
    factor is returned but not applied there; ``MoeDecoder``'s default ``scaling_type="none"``
    does the same.  Other kinds raise ``ValueError``, as ``build_rope`` does."""
    rs = rope_scaling or {}
    stype = (rs.get("type") or rs.get("rope_type") or "none").casefold()
    factor = float(rs.get("factor", 1.0) or 1.0)
    inv = 1.0 / (rope_theta ** (np.arange(0, head_dim, 2, dtype=np.float32) / head_dim))
    if stype in ("none", "default") or factor <= 1.0:
        return inv.astype(np.float32), 1.0
    if stype == "linear":
        return (inv / factor).astype(np.float32), 1.0
    if stype == "dynamic":
        return inv.astype(np.float32), 1.0
    if stype == "yarn":
        return _reference_yarn(head_dim, float(rope_theta), factor, float(rs.get("beta_fast", 32.0)),
                               float(rs.get("beta_slow", 1.0)), rs.get("attention_factor"))
    raise ValueError(f"unsupported rope_scaling type {stype!r} (none / linear / dynamic / yarn)")


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
