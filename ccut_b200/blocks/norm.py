"""Drop-in for ``ccut.blocks.norm.rms_norm`` on the GPU (``ccut_rms_norm``).

``rms_norm(x, weight, eps)``: ``y = x * (mean(x^2) + eps)^-1/2 * weight`` per row in fp32
(``ccut/blocks/norm.py:14-26``).  numpy in gives numpy float32 out; torch tensors in give
tensors out (bf16 in -> bf16 out, otherwise float32).  ``weight`` may be None.
"""

from __future__ import annotations

import numpy as np
import torch

from ccut_b200 import _lib
from ccut_b200.layer import _ptr, _stream

__all__ = ["rms_norm"]


def rms_norm(x, weight=None, eps: float = 1e-6):
    was_np = not isinstance(x, torch.Tensor)
    dev = x.device if isinstance(x, torch.Tensor) and x.is_cuda else torch.device("cuda")
    xt = (x if isinstance(x, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)))
    if xt.dtype not in (torch.bfloat16, torch.float32):
        xt = xt.float()
    xt = xt.to(dev).contiguous()
    shape = xt.shape
    dim = shape[-1]
    rows = xt.numel() // dim if dim else 0
    wt = None
    if weight is not None:
        wt = (weight if isinstance(weight, torch.Tensor) else torch.from_numpy(np.asarray(weight, np.float32)))
        wt = wt.to(device=dev, dtype=torch.float32).contiguous()
        if wt.numel() != dim:
            raise ValueError(f"weight has {wt.numel()} elements for rows of {dim}")
    out_dtype = torch.bfloat16 if (not was_np and xt.dtype == torch.bfloat16) else torch.float32
    out = torch.empty(shape, dtype=out_dtype, device=dev)
    xd = _lib.OUT_BF16 if xt.dtype == torch.bfloat16 else _lib.OUT_F32
    od = _lib.OUT_BF16 if out_dtype == torch.bfloat16 else _lib.OUT_F32
    with torch.cuda.device(dev):
        _lib.call("ccut_rms_norm", _ptr(xt), xd, _ptr(wt), rows, dim, float(eps), _ptr(out), od, _stream())
    return out.cpu().numpy() if was_np else out
