"""The C ABI's argument checks and size queries on the CPU (no GPU needed): every call here
returns before it touches a device, with the error code the header documents
(``include/ccut_moe.h``), which ``_lib.check`` maps to the reference's exception classes."""

from __future__ import annotations

import ctypes as C

import pytest

from ccut_b200 import _lib

FAKE = C.c_void_p(4096)  # a non-null device pointer that the checked calls never use
NULL = None


@pytest.fixture(scope="module")
def lib():
    from ccut_b200 import build

    build.build()  # nvcc cross-compiles here; no GPU is needed to load the library
    return _lib.load()


def _rp(mode=_lib.ROUTE_SOFTMAX_TOPK, k=2, n_group=1, topk_group=1):
    return _lib.RouteParams(mode, k, n_group, topk_group, 1.0, None)


def test_packed_sizes(lib):
    """Packed block bytes (AWQ 8512, FP8 16400 per 128 x 128 tile) and the cfg0 per-expert total
    (4,494,336 bytes, the algorithmic count of one DeepSeek-V2-Lite AWQ expert)."""
    assert lib.ccut_packed_matrix_bytes(_lib.FMT_AWQ_INT4_G128, 128, 128) == 8512
    assert lib.ccut_packed_matrix_bytes(_lib.FMT_FP8_E4M3_B128, 128, 128) == 16400
    awq = _lib.FMT_AWQ_INT4_G128
    assert lib.ccut_w13_bytes(awq, 2048, 1408) + lib.ccut_w2_bytes(awq, 2048, 1408) == 4_494_336
    assert lib.ccut_packed_matrix_bytes(awq, 100, 128) == 0
    assert lib.ccut_packed_matrix_bytes(7, 128, 128) == 0


def test_route_and_topk_checks(lib):
    ids = wts = FAKE
    assert lib.ccut_moe_topk(FAKE, 4, 8, None, ids, wts, NULL) == _lib.ERR_INVALID
    assert lib.ccut_moe_topk(FAKE, 4, 8, C.byref(_rp(k=0)), ids, wts, NULL) == _lib.ERR_INVALID
    assert lib.ccut_moe_topk(FAKE, 4, 8, C.byref(_rp(k=9)), ids, wts, NULL) == _lib.ERR_INVALID  # k > E
    assert lib.ccut_moe_topk(FAKE, 4, 8, C.byref(_rp(k=17)), ids, wts, NULL) == _lib.ERR_INVALID
    assert lib.ccut_moe_topk(FAKE, 4, 512, C.byref(_rp()), ids, wts, NULL) == _lib.ERR_UNSUPPORTED
    assert lib.ccut_moe_topk(FAKE, 4, 8, C.byref(_rp(mode=7)), ids, wts, NULL) == _lib.ERR_UNSUPPORTED
    sig = _lib.ROUTE_SIGMOID_GROUP
    assert lib.ccut_moe_topk(FAKE, 4, 12, C.byref(_rp(sig, 2, 8, 4)), ids, wts, NULL) == _lib.ERR_INVALID  # 12 % 8
    assert lib.ccut_moe_topk(FAKE, 4, 16, C.byref(_rp(sig, 2, 8, 9)), ids, wts, NULL) == _lib.ERR_INVALID
    assert lib.ccut_moe_topk(FAKE, 4, 16, C.byref(_rp(sig, 8, 8, 2)), ids, wts, NULL) == _lib.ERR_INVALID  # 2*2 < 8
    assert lib.ccut_moe_topk(FAKE, -1, 8, C.byref(_rp()), ids, wts, NULL) == _lib.ERR_INVALID
    assert lib.ccut_moe_topk(NULL, 0, 8, C.byref(_rp()), NULL, NULL, NULL) == _lib.OK  # no tokens: no work
    assert lib.ccut_moe_topk(NULL, 3, 8, C.byref(_rp()), ids, wts, NULL) == _lib.ERR_INVALID
    assert lib.ccut_moe_route(FAKE, FAKE, 4, 100, 8, C.byref(_rp()), ids, wts, NULL, FAKE, 1 << 20,
                              NULL) == _lib.ERR_INVALID  # H % 128
    assert lib.ccut_moe_route(NULL, NULL, 0, 128, 8, C.byref(_rp()), NULL, NULL, NULL, NULL, 0, NULL) == _lib.OK


def test_permute_and_combine_checks(lib):
    out4 = [FAKE] * 4
    assert lib.ccut_moe_permute(FAKE, FAKE, 4, 0, 8, 0, 1.0, *out4, FAKE, 1 << 20, NULL) == _lib.ERR_INVALID
    assert lib.ccut_moe_permute(FAKE, FAKE, 4, 2, 0, 0, 1.0, *out4, FAKE, 1 << 20, NULL) == _lib.ERR_INVALID
    assert lib.ccut_moe_permute(FAKE, FAKE, 4, 2, 300, 0, 1.0, *out4, FAKE, 1 << 20, NULL) == _lib.ERR_INVALID
    assert lib.ccut_moe_permute(FAKE, FAKE, 4, 2, 8, 0, 1.0, NULL, *out4[1:], FAKE, 1 << 20,
                                NULL) == _lib.ERR_INVALID
    need = lib.ccut_permute_workspace_bytes(8)
    assert need > 0
    assert lib.ccut_moe_permute(FAKE, FAKE, 4, 2, 8, 0, 1.0, *out4, FAKE, need - 1, NULL) == _lib.ERR_WORKSPACE
    assert lib.ccut_moe_combine(FAKE, FAKE, 4, 2, 130, 0, FAKE, _lib.OUT_BF16, NULL) == _lib.ERR_INVALID  # H % 4
    assert lib.ccut_moe_combine(FAKE, FAKE, 4, 2, 128, 33, FAKE, _lib.OUT_BF16, NULL) == _lib.ERR_UNSUPPORTED
    assert lib.ccut_moe_combine(FAKE, FAKE, 4, 2, 128, 0, FAKE, 5, NULL) == _lib.ERR_INVALID
    assert lib.ccut_moe_combine(FAKE, FAKE, 4, 0, 128, 0, FAKE, _lib.OUT_BF16, NULL) == _lib.ERR_INVALID
    assert lib.ccut_moe_combine(NULL, NULL, 0, 2, 128, 0, NULL, _lib.OUT_F32, NULL) == _lib.OK


def test_layer_and_linear_checks(lib):
    fmt = _lib.FMT_FP8_E4M3_B128
    bad = _lib.MoeLayerDesc(9, _lib.KERNEL_AUTO, 256, 128, 8, 0, 1.0, FAKE, FAKE, FAKE, FAKE, FAKE)
    assert lib.ccut_moe_forward_workspace_bytes(C.byref(bad), 4, 2) == 0
    rag = _lib.MoeLayerDesc(fmt, _lib.KERNEL_AUTO, 200, 128, 8, 0, 1.0, FAKE, FAKE, FAKE, FAKE, FAKE)
    assert lib.ccut_moe_forward_workspace_bytes(C.byref(rag), 4, 2) == 0
    assert lib.ccut_moe_forward(C.byref(bad), C.byref(_rp()), FAKE, 4, FAKE, _lib.OUT_BF16, NULL, NULL, FAKE,
                                1 << 20, NULL) == _lib.ERR_UNSUPPORTED
    assert lib.ccut_moe_forward(C.byref(rag), C.byref(_rp()), FAKE, 4, FAKE, _lib.OUT_BF16, NULL, NULL, FAKE,
                                1 << 20, NULL) == _lib.ERR_INVALID
    assert lib.ccut_quant_linear(9, _lib.LAYOUT_ROWS, FAKE, 128, 128, FAKE, 4, FAKE, FAKE, 1 << 20,
                                 NULL) == _lib.ERR_UNSUPPORTED
    assert lib.ccut_quant_linear(fmt, 9, FAKE, 128, 128, FAKE, 4, FAKE, FAKE, 1 << 20, NULL) == _lib.ERR_UNSUPPORTED
    assert lib.ccut_quant_linear(fmt, _lib.LAYOUT_ROWS, FAKE, 100, 128, FAKE, 4, FAKE, FAKE, 1 << 20,
                                 NULL) == _lib.ERR_INVALID
    assert lib.ccut_quant_linear(fmt, _lib.LAYOUT_ROWS, NULL, 128, 128, NULL, 0, NULL, NULL, 0, NULL) == _lib.OK
    need = lib.ccut_quant_linear_workspace_bytes(fmt, 4, 128)
    assert lib.ccut_quant_linear(fmt, _lib.LAYOUT_ROWS, FAKE, 128, 128, FAKE, 4, FAKE, FAKE, need - 1,
                                 NULL) == _lib.ERR_WORKSPACE


def test_attention_norm_rope_checks(lib):
    bf, f32 = _lib.OUT_BF16, _lib.OUT_F32
    gqa = lib.ccut_gqa_attention
    assert gqa(FAKE, FAKE, FAKE, 1, 8, 2, 1, 64, 96, -1, 0.0, 0.0, FAKE, bf, FAKE, 256, NULL) == _lib.ERR_UNSUPPORTED
    assert gqa(FAKE, FAKE, FAKE, 1, 3, 2, 1, 64, 64, -1, 0.0, 0.0, FAKE, bf, FAKE, 256, NULL) == _lib.ERR_INVALID
    assert gqa(FAKE, FAKE, FAKE, 1, 8, 2, 1, 64, 64, -1, 0.0, 0.0, FAKE, 4, FAKE, 256, NULL) == _lib.ERR_INVALID
    assert gqa(NULL, NULL, NULL, 0, 8, 2, 1, 64, 64, -1, 0.0, 0.0, NULL, bf, NULL, 0, NULL) == _lib.OK
    assert gqa(NULL, FAKE, FAKE, 1, 8, 2, 1, 64, 64, -1, 0.0, 0.0, FAKE, bf, FAKE, 256, NULL) == _lib.ERR_INVALID
    need = lib.ccut_gqa_attention_workspace_bytes(1, 8, 2, 1, 4096, 128)
    assert need > 256  # split over the kv range
    assert gqa(FAKE, FAKE, FAKE, 1, 8, 2, 1, 4096, 128, -1, 0.0, 0.0, FAKE, bf, FAKE, need - 1,
               NULL) == _lib.ERR_WORKSPACE
    assert lib.ccut_gqa_attention_workspace_bytes(1, 8, 3, 1, 64, 64) == 0
    mla = lib.ccut_mla_attention
    assert mla(FAKE, FAKE, 1, 16, 1, 64, 256, 64, -1, 0.1, FAKE, f32, FAKE, 256, NULL) == _lib.ERR_UNSUPPORTED
    assert mla(FAKE, FAKE, 1, 16, 1, 64, 512, 32, -1, 0.1, FAKE, f32, FAKE, 256, NULL) == _lib.ERR_UNSUPPORTED
    assert mla(FAKE, FAKE, 1, 16, 1, 64, 512, 64, -1, 0.0, FAKE, f32, FAKE, 256, NULL) == _lib.ERR_INVALID
    assert mla(FAKE, FAKE, 1, 0, 1, 64, 512, 64, -1, 0.1, FAKE, f32, FAKE, 256, NULL) == _lib.ERR_INVALID
    assert mla(FAKE, FAKE, 1, 16, 1, 64, 512, 64, -1, 0.1, FAKE, 3, FAKE, 256, NULL) == _lib.ERR_INVALID
    assert mla(C.c_void_p(4104), FAKE, 1, 16, 1, 64, 512, 64, -1, 0.1, FAKE, f32, FAKE, 256,
               NULL) == _lib.ERR_INVALID  # q not 16-byte aligned
    assert mla(NULL, NULL, 1, 16, 0, 64, 512, 64, -1, 0.1, NULL, f32, NULL, 0, NULL) == _lib.OK
    need = lib.ccut_mla_attention_workspace_bytes(1, 16, 1, 4096)
    assert need == 256 + 64 * 16 * (512 + 2) * 4  # 64 kv splits of one 16-row CTA
    assert mla(FAKE, FAKE, 1, 16, 1, 4096, 512, 64, -1, 0.1, FAKE, f32, FAKE, need - 1,
               NULL) == _lib.ERR_WORKSPACE
    assert lib.ccut_mla_attention_workspace_bytes(1, 0, 1, 64) == 0
    assert lib.ccut_rms_norm(FAKE, f32, NULL, 4, 0, 1e-6, FAKE, f32, NULL) == _lib.ERR_INVALID
    assert lib.ccut_rms_norm(FAKE, f32, NULL, 4, 64, -1.0, FAKE, f32, NULL) == _lib.ERR_INVALID
    assert lib.ccut_rms_norm(FAKE, 3, NULL, 4, 64, 1e-6, FAKE, f32, NULL) == _lib.ERR_INVALID
    assert lib.ccut_rms_norm(NULL, f32, NULL, 0, 64, 1e-6, NULL, f32, NULL) == _lib.OK
    assert lib.ccut_rms_norm(NULL, f32, NULL, 4, 64, 1e-6, FAKE, f32, NULL) == _lib.ERR_INVALID
    rope = lib.ccut_apply_rope
    assert rope(FAKE, bf, 1, 4, 2, 63, FAKE, FAKE, 1.0, FAKE, f32, NULL) == _lib.ERR_INVALID  # odd head dim
    assert rope(FAKE, 7, 1, 4, 2, 64, FAKE, FAKE, 1.0, FAKE, f32, NULL) == _lib.ERR_INVALID
    assert rope(NULL, bf, 1, 4, 0, 64, NULL, NULL, 1.0, NULL, f32, NULL) == _lib.OK
    assert rope(FAKE, bf, 1, 4, 2, 64, NULL, FAKE, 1.0, FAKE, f32, NULL) == _lib.ERR_INVALID


def test_error_strings_and_status(lib):
    for code in range(7):
        assert lib.ccut_strerror(code).decode()
    assert lib.ccut_workspace_status(NULL, NULL) == _lib.ERR_INVALID
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_WORKSPACE)
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.ERR_UNSUPPORTED)
    with pytest.raises(TimeoutError):
        _lib.check(_lib.ERR_TIMEOUT)
    _lib.check(_lib.OK)


def test_static_permute_checks(lib):
    """The allocation-free permutation refuses more experts than its fixed scratch holds and
    bad shapes before it looks up that scratch."""
    out4 = [FAKE] * 4
    assert lib.ccut_moe_permute_static(FAKE, FAKE, 4, 2, 257, 0, 1.0, *out4, NULL) == _lib.ERR_UNSUPPORTED
    assert lib.ccut_moe_permute_static(FAKE, FAKE, 4, 0, 8, 0, 1.0, *out4, NULL) == _lib.ERR_INVALID
    assert lib.ccut_moe_permute_static(FAKE, FAKE, -1, 2, 8, 0, 1.0, *out4, NULL) == _lib.ERR_INVALID
    assert lib.ccut_moe_permute_static(NULL, NULL, 4, 2, 8, 0, 1.0, *out4, NULL) == _lib.ERR_INVALID
    assert lib.ccut_moe_permute_static(FAKE, FAKE, 4, 2, 8, 0, 1.0, NULL, *out4[1:], NULL) == _lib.ERR_INVALID


def test_pool_attention_checks(lib):
    bf = _lib.OUT_BF16
    pool = lib.ccut_gqa_attention_pool
    stride = 2 * 300 * 64

    def call(*, q=FAKE, slots=FAKE, batch=3, heads=8, kvh=2, seq=1, L=300, d=64, stride=stride, n=4, out_dtype=bf,
             ws=1 << 20):
        return pool(q, FAKE, FAKE, slots, FAKE, batch, heads, kvh, seq, L, d, stride, n, 0.0, 0.0, FAKE, out_dtype,
                    FAKE, ws, NULL)

    assert call(d=96) == _lib.ERR_UNSUPPORTED
    assert call(heads=3) == _lib.ERR_INVALID
    assert call(stride=stride - 8) == _lib.ERR_INVALID  # slots would overlap
    assert call(stride=stride + 4) == _lib.ERR_INVALID  # slots not 16-byte aligned
    assert call(n=-1) == _lib.ERR_INVALID
    assert call(out_dtype=9) == _lib.ERR_INVALID
    assert call(batch=0) == _lib.OK
    assert call(slots=NULL) == _lib.ERR_INVALID
    assert call(q=NULL) == _lib.ERR_INVALID
    need = lib.ccut_gqa_attention_workspace_bytes(3, 8, 2, 1, 300, 64)
    if need > 256:
        assert call(ws=need - 1) == _lib.ERR_WORKSPACE


def test_mla_pool_attention_checks(lib):
    f32 = _lib.OUT_F32
    pool = lib.ccut_mla_attention_pool
    stride = 300 * 576

    def call(*, q=FAKE, kv=FAKE, slots=FAKE, batch=3, heads=16, seq=1, L=300, rank=512, rope=64, stride=stride, n=4,
             scale=0.1, out_dtype=f32, ws=1 << 24):
        return pool(q, kv, slots, FAKE, batch, heads, seq, L, rank, rope, stride, n, scale, FAKE, out_dtype, FAKE, ws,
                    NULL)

    assert call(rank=256) == _lib.ERR_UNSUPPORTED
    assert call(rope=32) == _lib.ERR_UNSUPPORTED
    assert call(heads=0) == _lib.ERR_INVALID
    assert call(scale=0.0) == _lib.ERR_INVALID
    assert call(stride=stride - 8) == _lib.ERR_INVALID  # slots would overlap
    assert call(stride=stride + 4) == _lib.ERR_INVALID  # slots not 16-byte aligned
    assert call(n=-1) == _lib.ERR_INVALID
    assert call(out_dtype=9) == _lib.ERR_INVALID
    assert call(batch=0) == _lib.OK
    assert call(slots=NULL) == _lib.ERR_INVALID
    assert call(kv=NULL) == _lib.ERR_INVALID
    assert call(q=C.c_void_p(4104)) == _lib.ERR_INVALID  # q not 16-byte aligned
    need = lib.ccut_mla_attention_workspace_bytes(3, 16, 1, 300)
    assert need > 256
    assert call(ws=need - 1) == _lib.ERR_WORKSPACE


def test_expert_parallel_checks(lib):
    """The routed-rows exchange's size queries and argument checks, before any NCCL call."""
    nb = lib.ccut_moe_ep_exchange_workspace_bytes(2, 64, 256, 6)
    assert nb > 2 * 64 * 256 * 2  # at least the send rows
    assert lib.ccut_moe_ep_exchange_workspace_bytes(0, 64, 256, 6) == 0
    assert lib.ccut_moe_ep_exchange_workspace_bytes(65, 64, 256, 6) == 0  # at most 64 ranks
    assert lib.ccut_moe_ep_exchange_workspace_bytes(2, 64, 100, 6) == 0  # rows of 16-byte lanes
    assert lib.ccut_moe_ep_exchange_workspace_bytes(2, 64, 256, 17) == 0
    n = C.c_int(0)
    # no handle
    assert lib.ccut_moe_ep_dispatch(NULL, FAKE, FAKE, FAKE, 4, 4, 256, 2, 8, FAKE, FAKE, FAKE, 8, C.byref(n), FAKE,
                                    nb, NULL) == _lib.ERR_INVALID
    assert lib.ccut_moe_ep_combine(NULL, FAKE, 4, 4, 256, 2, FAKE, FAKE, nb, NULL) == _lib.ERR_INVALID
    layer = _lib.MoeLayerDesc(_lib.FMT_FP8_E4M3_B128, 0, 256, 128, 4, 0, 1.0, FAKE.value, FAKE.value, None, None,
                              FAKE.value)
    assert lib.ccut_moe_ep_forward_workspace_bytes(C.byref(layer), 8, 2, 64, 2) > 0
    assert lib.ccut_moe_ep_forward_workspace_bytes(C.byref(layer), 2, 2, 64, 2) == 0  # fewer global than local
    assert lib.ccut_moe_ep_forward(NULL, C.byref(layer), 0, 8, C.byref(_rp()), FAKE, 4, 4, FAKE, 0, FAKE, 1 << 30,
                                   NULL) == _lib.ERR_INVALID


def test_wait_expiry_checks(lib):
    assert lib.ccut_debug_wait_expiry(NULL, 1000, NULL) == _lib.ERR_INVALID
    assert lib.ccut_debug_wait_expiry(FAKE, -1, NULL) == _lib.ERR_INVALID
    assert lib.ccut_debug_wait_expiry(FAKE, 1 << 40, NULL) == _lib.ERR_INVALID  # above the kernels' own budget


def test_router_scratch_sizes(lib):
    """From 256 tokens on, the router scratch also holds the exact three-way bf16 split of the
    router (3 x E x H x 2 bytes); the expert-parallel workspace, sized once for T_cap tokens per
    rank, never shrinks as T_cap grows, so every smaller batch fits in it."""
    E, H = 128, 2048
    small = lib.ccut_route_workspace_bytes(255, E, H)
    big = lib.ccut_route_workspace_bytes(256, E, H)
    assert big - small >= 3 * E * H * 2
    layer = _lib.MoeLayerDesc(_lib.FMT_AWQ_INT4_G128, _lib.KERNEL_AUTO, H, 768, 16, 0, 1.0, FAKE, FAKE, FAKE, FAKE,
                              FAKE)
    sizes = [lib.ccut_moe_ep_forward_workspace_bytes(C.byref(layer), E, 8, t, 8) for t in range(1, 1200, 7)]
    assert all(s > 0 for s in sizes)
    assert all(b >= a for a, b in zip(sizes, sizes[1:]))
