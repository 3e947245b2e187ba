"""Host-side logic that needs no GPU: sizing functions of the C ABI, argument validation (bad
arguments are refused before any CUDA call), and the graph runner's ring bookkeeping."""
import ctypes
from types import SimpleNamespace

import pytest

from wgkv._lib import lib
from wgkv.graph import graph_variant
from wgkv.pool import WgkvPool, advance_host_ring

EINVAL, ENOSPC = -1, -3


def _pool(**kw):
    p = WgkvPool()
    p.layers, p.batch, p.kv_heads, p.head_dim = kw.get("layers", 2), kw.get("batch", 3), kw.get("kv_heads", 4), 128
    p.window, p.page = kw.get("window", 64), 16
    p.max_blocks_per_head, p.max_tokens_per_head = kw.get("max_blocks", 100), kw.get("max_blocks", 100) * 16
    p.total_blocks = 10000
    return p


def test_quest_table_stride():
    # ring pages + the budget's pages (+1 spare), capped by the head's global pages
    assert lib.wgkv_quest_table_stride(64, 16, 144, 100) == 4 + (144 + 15) // 16 + 1
    assert lib.wgkv_quest_table_stride(64, 16, 10 ** 6, 100) == 4 + 96
    assert lib.wgkv_quest_table_stride(64, 16, 0, 100) == 4 + 1


def test_workspace_sizes():
    p = _pool()
    BH = 3 * 4
    assert lib.wgkv_quest_workspace_size(ctypes.addressof(p)) == BH * 100 * 2 + 256
    win, hq = 32, 16
    R = win * hq // 4
    r256 = lambda x: (x + 255) // 256 * 256  # noqa: E731
    splits = -(-(-(-1600 // 128)) // 32)  # row statistics per (head, row): one per 32-tile key split
    assert lib.wgkv_snapkv_workspace_size(ctypes.addressof(p), win, hq) == \
        r256(BH * R * 8 * splits) + 2 * r256(BH * 1600 * 4) + r256(2 * BH * 8) + 2 * r256(2 * BH * 4) + \
        r256(2 * BH * ((1600 + 31) // 32 + 32) * 4)  # + keep bits per position (+ a chunk's slack)
    assert lib.wgkv_argmax_workspace_size(2, 128256) == 2 * (((128256 + 4095) // 4096) * 8 + 4) + 256


def test_entry_points_refuse_bad_arguments_without_a_gpu():
    p = _pool()
    pr = ctypes.addressof(p)
    # no pool bounds / free list / ring state attached: refused up front
    assert lib.wgkv_quest_select(pr, 0, 10, 1, 0, 16, 144, 1, 1, 100, 1, 1 << 20, None) == EINVAL
    assert lib.wgkv_snapkv_evict(pr, 1, 32, 16, 0.1, 0.3, 5, 1, 1 << 20, None) == EINVAL
    assert lib.wgkv_ring_advance(pr, None) == EINVAL
    assert lib.wgkv_promote(pr, -1, None) == EINVAL  # device ring position without ring_state
    # skinny GEMM: more than 8 rows, k not a multiple of 8, paired with an odd n
    assert lib.wgkv_skinny_gemm(16, 8, 9, 16, 8, 8, 16, 8, 0, None, 0, None, 0.0, 0, None) == EINVAL
    assert lib.wgkv_skinny_gemm(16, 8, 1, 16, 8, 12, 16, 8, 0, None, 0, None, 0.0, 0, None) == EINVAL
    assert lib.wgkv_skinny_gemm(16, 8, 1, 16, 7, 8, 16, 8, 0, None, 0, None, 0.0, 1, None) == EINVAL
    assert lib.wgkv_rms_norm(16, 8, 16, 1, 12, 1e-5, 16, 8, None) == EINVAL
    assert lib.wgkv_argmax(16, 8, 0, 8, 16, 1, 16, 1 << 20, None) == EINVAL
    assert lib.wgkv_argmax(16, 8, 1, 8, 16, 1, 16, 0, None) == ENOSPC


@pytest.mark.parametrize("W,defer", [(8, False), (8, True)])
def test_graph_variant_and_host_ring(W, defer):
    """The host ring copy follows decode_wrapper (:1408-1413); the rescoring variant comes up once per
    window of steps with deferred gating, on the step that writes slot window - 1."""
    c = SimpleNamespace(local_length=3, local_ptr=0)
    seen = []
    for _ in range(3 * W):
        seen.append(graph_variant(c.local_length, c.local_ptr, W, defer))
        advance_host_ring(c, W)
    assert (c.local_length, c.local_ptr) == (W, (3 * W - (W - 3)) % W)
    refresh = [i for i, v in enumerate(seen) if v == "refresh"]
    if not defer:
        assert refresh == []
    else:
        assert refresh == [W - 1 - 3, 2 * W - 1 - 3, 3 * W - 1 - 3]
