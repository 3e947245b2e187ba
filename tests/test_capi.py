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


def test_every_entry_point_the_host_layer_calls_is_declared_and_exported():
    """A function the Python layer calls but the header does not declare would be built with hidden
    visibility (the library compiles with -fvisibility=hidden) and fail only on a GPU box."""
    import ctypes
    import glob
    import os
    import re
    import wgkv
    from wgkv._lib import LIB_PATH, parse_header
    pkg = os.path.dirname(os.path.abspath(wgkv.__file__))
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    used = set()
    for f in (glob.glob(os.path.join(pkg, "*.py")) + glob.glob(os.path.join(repo, "tests", "*.py")) +
              [os.path.join(repo, "bench.py"), os.path.join(repo, "__graft_entry__.py")]):
        used |= set(re.findall(r"lib\.(wgkv_\w+)", open(f).read()))
    declared = parse_header()
    assert used, "no entry points found"
    assert not (used - set(declared)), sorted(used - set(declared))
    lib = ctypes.CDLL(LIB_PATH)
    missing = [n for n in used if not hasattr(lib, n)]
    assert not missing, missing


def test_decode_argument_checks_run_before_any_device_work():
    """Both decode entry points refuse an unsupported head_dim with WGKV_EINVAL before they enqueue
    anything, so the check needs no GPU (the pointers are never dereferenced)."""
    if not os.path.exists(LIB_PATH):
        pytest.skip("libwgkv.so not built")
    from wgkv import lib
    fake = 4096  # non-null, 16-byte aligned, never touched
    for hd in (96, 32, 256):
        assert lib.wgkv_paged_decode_noalloc(fake, fake, fake, 8, 16, fake, fake, 1, 1, 8, 2, hd, 1.0, fake, fake,
                                             None) == -1
        assert lib.wgkv_paged_decode(fake, fake, fake, 8, 16, fake, fake, 1, 1, 8, 2, hd, 1.0, fake, fake, 1 << 20,
                                     fake, None) == -1
    # a missing output is refused before the size check of the static scratch
    assert lib.wgkv_paged_decode_noalloc(fake, fake, fake, 8, 16, fake, fake, 1, 4096, 128, 8, 128, 1.0, None, fake,
                                         None) == -1
