"""The C-ABI library loads without a GPU and exports every declared entry point (CPU)."""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "h3b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"H3B200_API\s+[\w\s\*]+?\b(h3b200_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "h3b200_fused_gated_mlp" in syms and "h3b200_quantize_int8_rowwise" in syms
    assert len(syms) >= 15


def test_library_exports_all_declared_symbols():
    from h3b200 import _lib

    if not os.path.exists(_lib.LIB_PATH):
        pytest.fail("libh3b200.so is not built (run __graft_entry__.build())")
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert missing == []
    # the ctypes signature table covers exactly the declared API
    assert sorted(_lib.SIGNATURES) == declared_symbols()


def test_version_and_error_without_gpu():
    from h3b200 import _lib

    lib = _lib.load()
    assert b"sm_100a" in lib.h3b200_version()
    # contract checks run on the host before any CUDA call
    rc = lib.h3b200_quantize_int8_rowwise(None, 4, 16, 8, 0, None, None, None)
    assert rc == _lib.ERR_INVALID
    assert b"bad shape" in lib.h3b200_last_error()
    rc = lib.h3b200_fused_gated_mlp(None, 64, None, None, None, None, None, None, 64, None, 64, 8, 64, 256, 2,
                                    None, 0, None)
    assert rc == _lib.ERR_UNSUPPORTED
    assert lib.h3b200_fused_gated_mlp_workspace_bytes(100, 3072, 12288) > 100 * 12288 * 3
