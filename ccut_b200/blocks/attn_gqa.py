"""Drop-ins for ``ccut.blocks.attn_gqa`` on the GPU (``ccut_gqa_attention``).

Same names, argument order and meaning as the reference: ``q [batch, heads, seq, d]``,
``k`` / ``v`` ``[batch, kv_heads, kv_len, d]``, output ``[batch, heads, seq, d]`` float32;
numpy in gives numpy out, torch tensors in give torch tensors out.  The differences:

- q, k and v enter the kernel as bf16 (the reference attends over fp32 arrays; a bf16 KV
  cache is the GPU's layout), scores and softmax stay fp32;
- ``mask`` may be None or the causal mask of ``build_causal_mask`` (broadcast over batch and
  heads or not); other additive masks raise ``NotImplementedError``.  ``start_pos`` gives
  the causal offset directly instead of a mask;
- head dims 64 and 128.

Reference: ``ccut/blocks/attn_gqa.py:65-73`` (build_causal_mask), ``:127-153``
(gqa_attention_fast, the function the attention layer calls at
``ccut/models/generic.py:343``), ``:76-124`` (gqa_attention: the same semantics with a
``softcap``; the reference's own per-token version of it fails on every input, its
``np.dot(q, k)`` misses a transpose).
"""

from __future__ import annotations

import numpy as np
import torch

from ccut_b200 import _lib
from ccut_b200.layer import _ptr, _stream

__all__ = ["build_causal_mask", "gqa_attention", "gqa_attention_fast"]


def build_causal_mask(seq_len: int, start_pos: int) -> np.ndarray:
    """[seq_len, start_pos + seq_len] float32: 0 where query i sees kv position j
    (j <= start_pos + i), -1e30 elsewhere."""
    q_idx = np.arange(start_pos, start_pos + seq_len)[:, None]
    kv_idx = np.arange(start_pos + seq_len)[None, :]
    m = np.zeros((seq_len, start_pos + seq_len), dtype=np.float32)
    m[kv_idx > q_idx] = -1e30
    return m


def _causal_start(mask, seq: int, kv_len: int) -> int:
    """-1 for no mask; the causal offset of a build_causal_mask mask; else NotImplementedError."""
    if mask is None:
        return -1
    m = mask.detach().float().cpu().numpy() if isinstance(mask, torch.Tensor) else np.asarray(mask, np.float32)
    if m.shape[-2:] != (seq, kv_len):
        raise ValueError(f"mask shape {m.shape} does not end in (seq, kv_len) = {(seq, kv_len)}")
    start = kv_len - seq
    ref = build_causal_mask(seq, start) if start >= 0 else None
    m2 = m.reshape(-1, seq, kv_len)
    if ref is None or not all(np.array_equal(mi <= -1e29, ref <= -1e29) and np.all(mi[ref > -1e29] == 0) for mi in m2):
        raise NotImplementedError("only causal masks (build_causal_mask) are supported on the GPU path")
    return start


def gqa_attention_fast(q, k, v, mask=None, scale=None, softcap=None, start_pos: int | None = None):
    was_np = not isinstance(q, torch.Tensor)
    dev = q.device if isinstance(q, torch.Tensor) and q.is_cuda else torch.device("cuda")

    def up(a):
        t = a if isinstance(a, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
        return t.to(device=dev, dtype=torch.bfloat16).contiguous()

    qt, kt, vt = up(q), up(k), up(v)
    if qt.dim() != 4 or kt.dim() != 4 or vt.dim() != 4:
        raise ValueError("q, k and v must be [batch, heads, seq, d]")
    b, h, s, d = qt.shape
    kvh, L = kt.shape[1], kt.shape[2]
    if tuple(kt.shape) != (b, kvh, L, d) or tuple(vt.shape) != tuple(kt.shape):
        raise ValueError(f"k / v shapes {tuple(kt.shape)} / {tuple(vt.shape)} do not match q {tuple(qt.shape)}")
    if h % kvh:
        raise ValueError(f"heads ({h}) must be a multiple of kv_heads ({kvh})")
    if d not in (64, 128):
        raise NotImplementedError(f"head dim {d} (have 64, 128)")
    causal = int(start_pos) if start_pos is not None else _causal_start(mask, s, L)
    out = torch.empty((b, h, s, d), dtype=torch.float32, device=dev)
    lib = _lib.load()
    nbytes = lib.ccut_gqa_attention_workspace_bytes(b, h, kvh, s, L, d)
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _lib.call("ccut_gqa_attention", _ptr(qt), _ptr(kt), _ptr(vt), b, h, kvh, s, L, d, causal,
                  float(scale or 0.0), float(softcap or 0.0), _ptr(out), _lib.OUT_F32, _ptr(ws), ws.numel(), _stream())
    return out.cpu().numpy() if was_np else out


def gqa_attention(q, k, v, mask=None, scale=None, softcap=None):
    """``gqa_attention``'s interface (with ``softcap``); computed as ``gqa_attention_fast``."""
    return gqa_attention_fast(q, k, v, mask, scale, softcap)
