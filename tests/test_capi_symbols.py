"""The C-ABI library loads and exports every symbol ``include/ccut_moe.h`` declares.

No compute call is made (this runs without a GPU)."""

from __future__ import annotations

import ctypes
import re

import pytest

from ccut_b200 import _lib, build

HEADER = build.INCLUDE / "ccut_moe.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"^CCUT_API\s+[\w\s\*]+?\b(ccut_\w+)\(", text, flags=re.M)


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert len(syms) >= 20
    for s in ("ccut_moe_route", "ccut_moe_permute", "ccut_moe_expert_ffn_w4a16", "ccut_moe_expert_ffn_fp8b128",
              "ccut_moe_combine", "ccut_moe_forward", "ccut_quant_linear", "ccut_pack_matrix"):
        assert s in syms


def test_library_exports_every_declared_symbol(lib):
    for s in declared_symbols():
        assert hasattr(lib, s), f"{s} missing from {_lib.LIB_PATH}"


def test_binding_table_matches_header():
    assert set(declared_symbols()) == set(_lib.SIGNATURES)


def test_host_only_calls(lib):
    # pure host arithmetic: no device work
    assert lib.ccut_abi_version() == 1
    assert lib.ccut_strerror(_lib.ERR_TIMEOUT) == b"bounded device wait expired"
    assert lib.ccut_packed_matrix_bytes(_lib.FMT_AWQ_INT4_G128, 2048, 1408) == 16 * 11 * 8512
    assert lib.ccut_packed_matrix_bytes(_lib.FMT_FP8_E4M3_B128, 1408, 2048) == 16 * 11 * 16400
    assert lib.ccut_packed_matrix_bytes(_lib.FMT_AWQ_INT4_G128, 100, 128) == 0
    assert lib.ccut_w13_bytes(_lib.FMT_FP8_E4M3_B128, 2048, 1408) == 2 * 11 * 16 * 16400


def test_argument_errors_map_to_reference_exceptions(lib):
    rp = _lib.RouteParams(0, 0, 1, 1, 1.0, None)  # top_k = 0 is invalid
    with pytest.raises(ValueError):
        _lib.call("ccut_moe_topk", ctypes.c_void_p(0), 4, 64, ctypes.byref(rp), None, None, None)
    rp = _lib.RouteParams(7, 2, 1, 1, 1.0, None)  # unknown mode
    with pytest.raises(NotImplementedError):
        _lib.call("ccut_moe_topk", ctypes.c_void_p(0), 4, 64, ctypes.byref(rp), None, None, None)
    with pytest.raises(NotImplementedError):
        _lib.call("ccut_pack_matrix", 9, 0, None, None, None, 128, 128, 0, None, 1, 0, None)
