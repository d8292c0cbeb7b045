"""MLA attention on the GPU (``ccut_mla_attention`` through the ``ccut_b200.blocks.attn_mla``
drop-ins) against the oracle's ``mla_attention`` (pinned to the reference's ``mla_decode`` /
``mla_prefill``, ``ccut/blocks/attn_mla.py:85-167``) at the DeepSeek-V2 / V3 latent sizes
(rank 512, rope 64): decode over every cached position, a causal prefill after a prefix, kv
ranges split over CTAs, 16 and 128 heads.  Inputs are bf16-representable (the cache is bf16);
tolerance 1e-3 of the largest output."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention, formats

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from ccut_b200 import build
    build.build()


def _bf(rng, shape, s=1.0):
    return formats.bf16_bits_to_f32(formats.bf16_bits_from_f32((rng.standard_normal(shape) * s).astype(np.float32)))


def _case(rng, heads, prefix, seq, dn=128, dv=128):
    rank, dr = 512, 64
    kv = prefix + seq
    return dict(c=_bf(rng, (kv, rank)), kpe=_bf(rng, (kv, dr)), qn=_bf(rng, (seq, heads, dn)),
                qp=_bf(rng, (seq, heads, dr)), ku=_bf(rng, (rank, heads * dn), 0.05), vu=_bf(rng, (rank, heads * dv), 0.05),
                scale=float(1.0 / np.sqrt(dn + dr)))


def _close(got, ref, tol=1e-3):
    err = np.abs(np.asarray(got) - ref).max() / np.abs(ref).max()
    assert err <= tol, err


@pytest.mark.parametrize("heads, prefix, seq", [(16, 300, 1), (128, 70, 1), (16, 5, 40), (16, 900, 3), (4, 0, 17)])
def test_mla_matches_oracle(heads, prefix, seq):
    from ccut_b200.blocks import attn_mla

    rng = np.random.default_rng(heads + prefix + seq)
    k = _case(rng, heads, prefix, seq)
    st = attn_mla.MLAState(512, 64, max_tokens=1024)
    st.append(k["c"], k["kpe"])
    assert st.n == prefix + seq and st.bytes() == 576 * 2 * st.n
    ref = attention.mla_attention(k["c"], k["kpe"], k["qn"], k["qp"], k["ku"], k["vu"], k["scale"], prefix)
    if seq == 1:  # decode: every cached position
        got = attn_mla.mla_decode(st, k["qn"][0], k["qp"][0], k["ku"], k["vu"], k["scale"], prefix)
        assert got.shape == (heads, 128)
        _close(got, ref[0])
    got = attn_mla.mla_prefill(st, k["qn"], k["qp"], k["ku"], k["vu"], k["scale"], prefix)
    assert isinstance(got, np.ndarray) and got.shape == (seq, heads, 128)
    _close(got, ref)
    # torch in, torch out
    gt = attn_mla.mla_prefill(st, torch.from_numpy(k["qn"]).cuda(), torch.from_numpy(k["qp"]).cuda(), k["ku"],
                              k["vu"], k["scale"], prefix)
    assert gt.is_cuda
    _close(gt.cpu().numpy(), ref)


def test_mla_edges():
    from ccut_b200 import _lib
    from ccut_b200.blocks import attn_mla
    from ccut_b200.layer import _ptr, _stream

    rng = np.random.default_rng(3)
    k = _case(rng, 16, 30, 2)
    st = attn_mla.MLAState(512, 64, max_tokens=40)
    # no cached positions: zeros (the reference's 1e-30 clamp on an empty sum)
    z = attn_mla.mla_prefill(st, k["qn"], k["qp"], k["ku"], k["vu"], k["scale"], 0)
    assert np.count_nonzero(z) == 0
    st.append(k["c"], k["kpe"])
    with pytest.raises(MemoryError):
        st.append(k["c"][:9], k["kpe"][:9])
    # bf16 latent output straight from the C ABI equals the fp32 one rounded
    q = torch.cat([torch.einsum("shd,rhd->shr", torch.from_numpy(k["qn"]).cuda(),
                                torch.from_numpy(k["ku"]).cuda().view(512, 16, 128)),
                   torch.from_numpy(k["qp"]).cuda()], -1).contiguous()
    kv = st.kv[: st.n]
    o32 = attn_mla._latent_attention(q, kv, 30, k["scale"])
    ob = torch.empty((32, 512), dtype=torch.bfloat16, device="cuda")
    ws = torch.empty(max(_lib.load().ccut_mla_attention_workspace_bytes(1, 16, 2, st.n), 256), dtype=torch.uint8,
                     device="cuda")
    _lib.call("ccut_mla_attention", _ptr(q), _ptr(kv), 1, 16, 2, st.n, 512, 64, 30, k["scale"], _ptr(ob),
              _lib.OUT_BF16, _ptr(ws), ws.numel(), _stream())
    torch.cuda.synchronize()
    np.testing.assert_allclose(ob.float().cpu().numpy(), o32.cpu().numpy(), rtol=1e-2, atol=1e-2)
    with pytest.raises(NotImplementedError):
        attn_mla.MLAState(64, 16)
    with pytest.raises(NotImplementedError):  # the C ABI rejects other latent sizes
        _lib.call("ccut_mla_attention", _ptr(q), _ptr(kv), 1, 16, 2, st.n, 256, 64, 30, k["scale"], _ptr(ob),
                  _lib.OUT_BF16, _ptr(ws), ws.numel(), _stream())
    with pytest.raises(ValueError):
        attn_mla.mla_prefill(st, k["qn"], k["qp"], k["ku"], k["vu"], 0.0, 0)
