"""Drop-ins for ``ccut.blocks.attn_mla`` on the GPU (``ccut_mla_attention``).

Same names, argument order and meaning as the reference (``ccut/blocks/attn_mla.py:27-167``):
``MLAState(kv_lora_rank, qk_rope_head_dim, max_tokens)`` holds one sequence's latent cache,
``mla_update_state`` projects and appends, ``mla_decode`` attends one token's heads over every
cached position, ``mla_prefill`` a batch of tokens causally (query ``s`` sees
``min(start_pos + s + 1, n)`` positions).  numpy in gives numpy out, torch tensors in give
tensors out.  The differences:

- the cache is bf16 in HBM, one 576-element row per position (the latent ``c`` then ``k_pe``),
  where the reference keeps fp32 arrays; ``bytes()`` counts the bf16 bytes;
- the attention runs in the latent space: ``q_nope`` of every head is folded through its
  ``k_up`` block first (``q_nope k_up_h^T``, a batched GEMM), the kernel computes
  ``softmax(q . kv^T * scale) @ c`` per head over the shared latent rows, and the result is
  unfolded through ``v_up_h`` (a batched GEMM); this is the reference's computation regrouped
  (``(c k_up_h) . q_nope = (q_nope k_up_h^T) . c`` and ``probs @ (c v_up_h) = (probs @ c) v_up_h``);
- ``kv_lora_rank`` 512 and ``qk_rope_head_dim`` 64 (DeepSeek-V2 / V3); other sizes raise
  ``NotImplementedError``.
"""

from __future__ import annotations

import numpy as np
import torch

from ccut_b200 import _lib
from ccut_b200.layer import _ptr, _stream

__all__ = ["MLAState", "mla_update_state", "mla_decode", "mla_prefill"]

_RANK, _ROPE = 512, 64


def _f32(a, dev) -> torch.Tensor:
    t = a if isinstance(a, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
    return t.to(device=dev, dtype=torch.float32)


class MLAState:
    """One sequence's MLA cache: ``kv`` bf16 ``[max_tokens, kv_lora_rank + qk_rope_head_dim]``
    on the device (``c`` then ``k_pe`` per position), ``n`` positions valid."""

    def __init__(self, kv_lora_rank: int, qk_rope_head_dim: int, max_tokens: int = 32768, device="cuda"):
        if (kv_lora_rank, qk_rope_head_dim) != (_RANK, _ROPE):
            raise NotImplementedError(f"MLA with kv_lora_rank {kv_lora_rank} / qk_rope_head_dim {qk_rope_head_dim}"
                                      f" (have {_RANK} / {_ROPE})")
        self.kv_lora_rank, self.qk_rope_head_dim = kv_lora_rank, qk_rope_head_dim
        self.device = torch.device(device)
        self.kv = torch.zeros((int(max_tokens), _RANK + _ROPE), dtype=torch.bfloat16, device=self.device)
        self.n = 0

    @property
    def c(self) -> torch.Tensor:
        return self.kv[: self.n, :_RANK]

    @property
    def k_pe(self) -> torch.Tensor:
        return self.kv[: self.n, _RANK:]

    def append(self, c, k_pe) -> int:
        """Append ``c [n_new, rank]`` and ``k_pe [n_new, rope]``; returns the first position."""
        ct, kt = _f32(c, self.device), _f32(k_pe, self.device)
        n_new = ct.shape[0]
        if tuple(ct.shape) != (n_new, _RANK) or tuple(kt.shape) != (n_new, _ROPE):
            raise ValueError(f"c must be [n, {_RANK}] and k_pe [n, {_ROPE}], got {tuple(ct.shape)} / {tuple(kt.shape)}")
        if self.n + n_new > self.kv.shape[0]:
            raise MemoryError(f"MLAState holds {self.kv.shape[0]} positions: {self.n} + {n_new} do not fit")
        self.kv[self.n: self.n + n_new, :_RANK] = ct
        self.kv[self.n: self.n + n_new, _RANK:] = kt
        pos = self.n
        self.n += n_new
        return pos

    def reset(self) -> None:
        self.n = 0

    def bytes(self) -> int:
        return (self.kv_lora_rank + self.qk_rope_head_dim) * 2 * self.n


def mla_update_state(state: MLAState, x, kv_a_proj, kv_a_scale, q_pe):
    """``x @ kv_a_proj`` split into ``c`` (the first ``rank`` features); appends ``(c, q_pe)``
    -- the caller passes the rotated ``k_pe`` as ``q_pe``, as in the reference -- and returns
    them (``kv_a_scale`` is unused there too)."""
    was_np = not isinstance(x, torch.Tensor)
    kv_a = _f32(x, state.device) @ _f32(kv_a_proj, state.device)
    c = kv_a[..., : state.kv_lora_rank]
    state.append(c, q_pe)
    if was_np:
        return c.cpu().numpy(), np.asarray(q_pe, dtype=np.float32)
    return c, q_pe


def _latent_attention(q: torch.Tensor, kv: torch.Tensor, causal_start: int, scale: float) -> torch.Tensor:
    """q fp32 [S, H, 576], kv bf16 [n, 576] -> o_lat fp32 [S * H, 512] (``ccut_mla_attention``)."""
    S, H, _ = q.shape
    n = kv.shape[0]
    out = torch.empty((S * H, _RANK), dtype=torch.float32, device=q.device)
    lib = _lib.load()
    nbytes = lib.ccut_mla_attention_workspace_bytes(1, H, S, n)
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=q.device)
    with torch.cuda.device(q.device):
        _lib.call("ccut_mla_attention", _ptr(q), _ptr(kv), 1, H, S, n, _RANK, _ROPE, int(causal_start), float(scale),
                  _ptr(out), _lib.OUT_F32, _ptr(ws), ws.numel(), _stream())
    return out


def _attend(state: MLAState, q_nope: torch.Tensor, q_pe: torch.Tensor, k_up, v_up, scale: float,
            causal_start: int) -> torch.Tensor:
    """q_nope [S, H, d_nope], q_pe [S, H, rope] -> [S, H, d_v] fp32."""
    dev = state.device
    S, H, dn = q_nope.shape
    if q_pe.shape != (S, H, _ROPE):
        raise ValueError(f"q_pe must be [{S}, {H}, {_ROPE}], got {tuple(q_pe.shape)}")
    ku = _f32(k_up, dev)
    vu = _f32(v_up, dev)
    if ku.shape != (_RANK, H * dn) or vu.dim() != 2 or vu.shape[0] != _RANK or vu.shape[1] % H:
        raise ValueError(f"k_up must be [{_RANK}, {H * dn}] and v_up [{_RANK}, {H} * d_v]")
    dv = vu.shape[1] // H
    if not scale > 0:
        raise ValueError("scale must be positive")
    q_lat = torch.einsum("shd,rhd->shr", q_nope, ku.view(_RANK, H, dn))
    q = torch.cat([q_lat, q_pe], dim=-1).contiguous()  # [S, H, 576] fp32
    out = _latent_attention(q, state.kv[: state.n], causal_start, scale)
    return torch.einsum("shr,rhd->shd", out.view(S, H, _RANK), vu.view(_RANK, H, dv))


def mla_decode(state: MLAState, q_nope, q_pe_rot, k_up_proj, v_up_proj, scale: float, start_pos: int):
    """One token: ``q_nope [heads, d_nope]``, ``q_pe_rot [heads, rope]`` over every cached
    position -> ``[heads, d_v]`` float32."""
    was_np = not isinstance(q_nope, torch.Tensor)
    qn, qp = _f32(q_nope, state.device), _f32(q_pe_rot, state.device)
    if qn.dim() != 2 or qp.dim() != 2:
        raise ValueError("q_nope must be [heads, d_nope] and q_pe_rot [heads, rope]")
    o = _attend(state, qn[None], qp[None], k_up_proj, v_up_proj, scale, -1)[0]
    return o.cpu().numpy() if was_np else o


def mla_prefill(state: MLAState, q_nope, q_pe_rot, k_up_proj, v_up_proj, scale: float, start_pos: int):
    """A causal batch: ``q_nope [seq, heads, d_nope]``, ``q_pe_rot [seq, heads, rope]``;
    token ``s`` sees ``min(start_pos + s + 1, n)`` positions -> ``[seq, heads, d_v]`` float32."""
    was_np = not isinstance(q_nope, torch.Tensor)
    qn, qp = _f32(q_nope, state.device), _f32(q_pe_rot, state.device)
    if qn.dim() != 3 or qp.dim() != 3:
        raise ValueError("q_nope must be [seq, heads, d_nope] and q_pe_rot [seq, heads, rope]")
    if start_pos < 0:
        raise ValueError("start_pos must be >= 0")
    o = _attend(state, qn, qp, k_up_proj, v_up_proj, scale, int(start_pos))
    return o.cpu().numpy() if was_np else o
