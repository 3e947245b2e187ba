"""C-ABI library checks that need no GPU: it loads and exports every symbol
include/wgkv.h declares (no compute calls)."""
import ctypes
import os

import pytest

from wgkv._lib import HEADER, LIB_PATH, parse_header


def test_header_parses():
    decls = parse_header()
    assert "wgkv_paged_decode" in decls
    assert len(decls) >= 4


def test_library_exports_every_declared_symbol():
    if not os.path.exists(LIB_PATH):
        pytest.skip("libwgkv.so not built")
    lib = ctypes.CDLL(LIB_PATH)
    missing = [n for n in parse_header() if not hasattr(lib, n)]
    assert not missing, missing


def test_version_without_gpu():
    if not os.path.exists(LIB_PATH):
        pytest.skip("libwgkv.so not built")
    from wgkv import lib
    assert lib.wgkv_version() >= 1
