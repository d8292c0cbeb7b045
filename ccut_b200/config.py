"""The reference's ``[experts]`` and ``[quant]`` settings (``ccut/config.py:91-108``,
``engine.toml:26-42``) read for this path.

- ``[quant]``: ``quantization = "auto"`` takes the format from the checkpoint's
  ``quantization_config`` (AWQ int4 g128 or FP8 e4m3 128 x 128 blocks); the online
  quantization shorthands (``fp8_per_token``, ``mxfp8``, ...) are formats this path does not
  run.  ``fp8_compute_mode = "w8a16"`` is what the kernels do (weights dequantized, activations
  in 16 bits); ``w8a8`` is refused.  ``kv_cache_dtype``: ``auto`` / ``bf16`` (the decoder's
  caches are bf16); ``fp8`` is refused.  ``quant_ignore`` applies to online quantization only.
- ``[experts]``: the reference streams experts from disk (``expert_residency = "zero"`` or
  ``"page_cache_only"``, a ring of ``expert_ring_slots``); here every expert is packed into HBM
  once, so these settings are checked against the reference's allowed values and have no
  further effect.

Unsupported values raise ``NotImplementedError`` and out-of-range ones ``ValueError``, as the
reference's config validation and quant registry do.
"""

from __future__ import annotations

from ccut_b200.checkpoint import quant_format

__all__ = ["quant_settings", "expert_settings", "resolve"]

_ONLINE = ("fp8_per_token", "int8_per_channel_weight_only", "mxfp8", "nvfp4_per_token", "int8_per_token", "bf16")


def _section(app_config, name: str) -> dict:
    if app_config is None:
        return {}
    sec = app_config.get(name, {}) if hasattr(app_config, "get") else getattr(app_config, name, {})
    return dict(sec or {})


def quant_settings(app_config, checkpoint_config: dict) -> dict:
    """``{"format", "fp8_compute_mode", "kv_cache_dtype"}`` for a ``[quant]`` section and the
    checkpoint's ``config.json``."""
    q = _section(app_config, "quant")
    quantization = str(q.get("quantization", "auto"))
    if quantization in _ONLINE:
        raise NotImplementedError(f"online quantization {quantization!r}: this path runs the checkpoint's own AWQ "
                                  "int4 g128 / FP8 e4m3 128x128 weights (quantization = \"auto\")")
    if quantization != "auto":
        raise ValueError(f"[quant] quantization = {quantization!r} is not one of auto, {', '.join(_ONLINE)}")
    mode = str(q.get("fp8_compute_mode", "w8a16"))
    if mode == "w8a8":
        raise NotImplementedError("fp8_compute_mode = \"w8a8\": the kernels dequantize the weights and keep 16-bit "
                                  "activations (w8a16)")
    if mode != "w8a16":
        raise ValueError(f"[quant] fp8_compute_mode = {mode!r} is not one of w8a16, w8a8")
    kv = str(q.get("kv_cache_dtype", "auto"))
    if kv == "fp8":
        raise NotImplementedError("kv_cache_dtype = \"fp8\": the decoder's kv caches are bf16")
    if kv not in ("auto", "bf16"):
        raise ValueError(f"[quant] kv_cache_dtype = {kv!r} is not one of auto, bf16, fp8")
    return {"format": quant_format(checkpoint_config), "fp8_compute_mode": "w8a16", "kv_cache_dtype": "bf16"}


def expert_settings(app_config) -> dict:
    """The ``[experts]`` section checked against the reference's allowed values; the experts
    are resident in HBM whatever it says."""
    e = _section(app_config, "experts")
    residency = str(e.get("expert_residency", "zero"))
    if residency not in ("zero", "page_cache_only"):
        raise ValueError(f"[experts] expert_residency = {residency!r} is not one of zero, page_cache_only")
    slots = int(e.get("expert_ring_slots", 2))
    if not 1 <= slots <= 8:
        raise ValueError(f"[experts] expert_ring_slots = {slots} is outside [1, 8]")
    return {"residency": "hbm", "expert_residency": residency, "expert_ring_slots": slots}


def resolve(app_config, checkpoint_config: dict) -> dict:
    """Both sections, merged."""
    return {**expert_settings(app_config), **quant_settings(app_config, checkpoint_config)}
