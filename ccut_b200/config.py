"""The reference's ``[experts]`` and ``[quant]`` settings (``ccut/config.py:91-108``,
``engine.toml:26-42``) read for this path.

- ``[quant]``: ``quantization = "auto"`` takes the format from the checkpoint's
  ``quantization_config`` (AWQ int4 g128, FP8 e4m3 128 x 128 blocks or per channel, signed
  int4); the online quantization shorthands (``fp8_per_token``, ``mxfp8``, ...) are formats
  this path does not run.  ``fp8_compute_mode``: ``w8a16`` is what the kernels do (exact
  weight codes, activations in 16 bits); ``w8a8`` is accepted and computed the same way, as
  the reference computes it (its ``_w8a8`` dequantizes the weights and multiplies the
  unquantized activations, ``ccut/quant/method.py:131-139``).  ``kv_cache_dtype``: ``auto`` /
  ``bf16`` (the decoder's caches are bf16); ``fp8`` is refused.  ``quant_ignore`` applies to
  online quantization only.
- ``[experts]``: the reference streams experts from disk (``expert_residency = "zero"`` or
  ``"page_cache_only"``, a ring of ``expert_ring_slots``); here every expert is packed into HBM
  once.  ``expert_residency`` takes this path's own value ``"hbm"`` (the default) besides the
  reference's two, which are checked and then run resident as well.  ``expert_parallel_size``
  (new, default 1) splits each layer's routed experts over that many GPUs, one process per
  GPU (``ccut_b200.ep``); it must equal the ``torch.distributed`` world size.
- ``cross_validate`` keeps the reference's rule that ``tensor_parallel_size`` and
  ``pipeline_parallel_size`` are 1 (``ccut/config.py:466-470``) and admits expert parallelism.

Unsupported values raise ``NotImplementedError`` and out-of-range ones ``ValueError``, as the
reference's config validation and quant registry do.
"""

from __future__ import annotations

from ccut_b200.checkpoint import quant_format

__all__ = ["quant_settings", "expert_settings", "cross_validate", "resolve"]

_RESIDENCY = ("hbm", "zero", "page_cache_only")

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
    if mode not in ("w8a16", "w8a8"):
        raise ValueError(f"[quant] fp8_compute_mode = {mode!r} is not one of w8a16, w8a8")
    kv = str(q.get("kv_cache_dtype", "auto"))
    if kv == "fp8":
        raise NotImplementedError("kv_cache_dtype = \"fp8\": the decoder's kv caches are bf16")
    if kv not in ("auto", "bf16"):
        raise ValueError(f"[quant] kv_cache_dtype = {kv!r} is not one of auto, bf16, fp8")
    return {"format": quant_format(checkpoint_config), "fp8_compute_mode": mode, "kv_cache_dtype": "bf16"}


def expert_settings(app_config) -> dict:
    """The ``[experts]`` section checked against the allowed values; the experts are resident
    in HBM whatever it says."""
    e = _section(app_config, "experts")
    residency = str(e.get("expert_residency", "hbm"))
    if residency not in _RESIDENCY:
        raise ValueError(f"[experts] expert_residency = {residency!r} is not one of {', '.join(_RESIDENCY)}")
    slots = int(e.get("expert_ring_slots", 2))
    if not 1 <= slots <= 8:
        raise ValueError(f"[experts] expert_ring_slots = {slots} is outside [1, 8]")
    ep = e.get("expert_parallel_size", 1)
    if isinstance(ep, bool) or not isinstance(ep, int) or ep < 1:
        raise ValueError(f"[experts] expert_parallel_size = {ep!r} must be an integer >= 1")
    return {"residency": "hbm", "expert_residency": residency, "expert_ring_slots": slots,
            "expert_parallel_size": ep}


def cross_validate(app_config, world_size: int | None = None, num_experts: int | None = None) -> dict:
    """Cross-field checks (``ccut/config.py:466-484`` for the reference's own): tensor and
    pipeline parallelism stay 1 as in the reference; expert parallelism may be above 1, equal to
    the process group's ``world_size`` when one is given, and at most ``num_experts`` (every rank
    owns at least one routed expert).  Raises ``ValueError``; returns the ``[experts]`` settings."""
    eng = _section(app_config, "engine")
    for key in ("tensor_parallel_size", "pipeline_parallel_size"):
        v = eng.get(key, 1)
        if v != 1:
            raise ValueError(f"[engine] {key} = {v!r}: only expert parallelism splits a layer over GPUs here "
                             "(tensor and pipeline parallel sizes must be 1, as in the reference)")
    ex = expert_settings(app_config)
    ep = ex["expert_parallel_size"]
    if world_size is not None and ep != world_size:
        raise ValueError(f"[experts] expert_parallel_size = {ep} but the process group has {world_size} ranks")
    if num_experts is not None and ep > num_experts:
        raise ValueError(f"[experts] expert_parallel_size = {ep} exceeds the layer's {num_experts} routed experts")
    return ex


def resolve(app_config, checkpoint_config: dict) -> dict:
    """Both sections, merged, after the cross-field checks."""
    cross_validate(app_config)
    return {**expert_settings(app_config), **quant_settings(app_config, checkpoint_config)}
