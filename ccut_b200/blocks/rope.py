"""Drop-in for ``ccut.blocks.rope.apply_rope`` on the GPU (``ccut_apply_rope``).

``apply_rope(q, k, inv_freq, positions, attention_factor=1.0, scaling_type="none",
seq_len=0)`` rotates q ``[batch, heads, seq, d]`` and k ``[batch, kv_heads, seq, d]`` by
``positions [batch, seq] * inv_freq`` (half rotation), q first scaled by
``attention_factor`` for the ``yarn`` / ``linear`` scalings, and returns ``(q_rot, k_rot)``
float32 (``ccut/blocks/rope.py:130-175``).  ``inv_freq`` is the host table of the
reference's ``build_rope``.  numpy in gives numpy out, torch tensors in give tensors out.
"""

from __future__ import annotations

import numpy as np
import torch

from ccut_b200 import _lib
from ccut_b200.layer import _ptr, _stream

__all__ = ["apply_rope"]


def _rotate(x: torch.Tensor, inv_freq: torch.Tensor, pos: torch.Tensor, scale: float) -> torch.Tensor:
    b, h, s, d = x.shape
    out = torch.empty((b, h, s, d), dtype=torch.float32, device=x.device)
    xd = _lib.OUT_BF16 if x.dtype == torch.bfloat16 else _lib.OUT_F32
    with torch.cuda.device(x.device):
        _lib.call("ccut_apply_rope", _ptr(x), xd, b, h, s, d, _ptr(inv_freq), _ptr(pos), float(scale), _ptr(out),
                  _lib.OUT_F32, _stream())
    return out


def apply_rope(q, k, inv_freq, positions, attention_factor: float = 1.0, scaling_type: str = "none",
               seq_len: int = 0):
    was_np = not isinstance(q, torch.Tensor)
    dev = q.device if isinstance(q, torch.Tensor) and q.is_cuda else torch.device("cuda")

    def up(a):
        t = a if isinstance(a, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
        if t.dtype not in (torch.bfloat16, torch.float32):
            t = t.float()
        return t.to(dev).contiguous()

    qt, kt = up(q), up(k)
    if qt.dim() != 4 or kt.dim() != 4 or qt.shape[-1] % 2 or kt.shape[-1] != qt.shape[-1]:
        raise ValueError("q and k must be [batch, heads, seq, d] with the same even d")
    b, _, s, d = qt.shape
    if kt.shape[0] != b or kt.shape[2] != s:
        raise ValueError("q and k must share batch and seq")
    ft = (inv_freq if isinstance(inv_freq, torch.Tensor) else torch.from_numpy(np.asarray(inv_freq, np.float32)))
    ft = ft.to(device=dev, dtype=torch.float32).contiguous()
    if ft.numel() != d // 2:
        raise ValueError(f"inv_freq has {ft.numel()} entries for head dim {d}")
    pt = positions if isinstance(positions, torch.Tensor) else torch.from_numpy(np.asarray(positions))
    pt = pt.to(device=dev, dtype=torch.int32).reshape(b, s).contiguous()
    qs = float(attention_factor) if scaling_type in ("yarn", "linear") and attention_factor != 1.0 else 1.0
    qo, ko = _rotate(qt, ft, pt, qs), _rotate(kt, ft, pt, 1.0)
    return (qo.cpu().numpy(), ko.cpu().numpy()) if was_np else (qo, ko)
