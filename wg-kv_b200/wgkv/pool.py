"""Device-resident paged KV pool (the state the reference hangs on its cache).

The reference's ``prefill_wrapper`` (src/modeling_layers.py:1196-1288)
attaches ``block_table``, ``block_pool_k/v``, ``local_is_global``,
``global_lengths``, ``local_region_starts``, ``local_ptr``,
``local_length``, ``next_free_block`` and ``total_blocks`` to the HF
cache object.  :func:`init_pool` attaches the same attribute names (with a
batch axis on the per-head tensors) plus a ``wgkv_pool`` ctypes struct that
the C ABI consumes.  ``next_free_block`` lives on the device (a 1-element
int32 tensor) so page allocation never syncs the host.
"""
from __future__ import annotations

import ctypes

import torch

from .runtime import err_word


class WgkvPool(ctypes.Structure):
    """Mirror of ``wgkv_pool`` in include/wgkv.h."""
    _fields_ = [
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("block_table", ctypes.c_void_p),
        ("global_lengths", ctypes.c_void_p),
        ("local_is_global", ctypes.c_void_p),
        ("local_pre_key", ctypes.c_void_p),
        ("next_free_block", ctypes.c_void_p),
        ("err", ctypes.c_void_p),
        ("total_blocks", ctypes.c_int64),
        ("layers", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("window", ctypes.c_int32),
        ("page", ctypes.c_int32),
        ("max_blocks_per_head", ctypes.c_int32),
        ("max_tokens_per_head", ctypes.c_int32),
        ("ring_state", ctypes.c_void_p),
        ("quest_min", ctypes.c_void_p),
        ("quest_max", ctypes.c_void_p),
        ("free_ids", ctypes.c_void_p),
        ("free_count", ctypes.c_void_p),
    ]


def init_pool(cache, *, layers, batch, kv_heads, head_dim, window, page, max_total_tokens, max_tokens_per_head,
              device, dtype=torch.bfloat16, defer=False, quest=False, snapkv_window=None, q_heads=None):
    """Allocate the pool on ``cache`` (any attribute holder), as prefill_wrapper does at layer 0."""
    assert window % page == 0, "local_window_size must be a multiple of block_size"
    local_pages = window // page
    total_local = layers * batch * kv_heads * local_pages
    total_blocks = (max_total_tokens + page - 1) // page
    max_blocks_per_head = (max_tokens_per_head + page - 1) // page
    assert total_blocks > total_local, "max_total_tokens leaves no room for global pages"
    assert max_blocks_per_head >= local_pages
    sentinel = total_blocks - 1
    dev = torch.device(device)
    cache.block_table = torch.full((layers, batch, kv_heads, max_blocks_per_head), sentinel, dtype=torch.int32,
                                   device=dev)
    cache.block_table[..., :local_pages] = torch.arange(total_local, dtype=torch.int32, device=dev).view(
        layers, batch, kv_heads, local_pages)
    cache.block_pool_k = torch.empty(total_blocks * page, head_dim, dtype=dtype, device=dev)
    cache.block_pool_v = torch.empty(total_blocks * page, head_dim, dtype=dtype, device=dev)
    cache.local_is_global = torch.zeros(layers, batch, kv_heads, window, dtype=torch.uint8, device=dev)
    cache.global_lengths = torch.zeros(layers, batch, kv_heads, dtype=torch.int32, device=dev)
    cache.local_pre_key = (torch.empty(layers, batch, kv_heads, window, head_dim, dtype=dtype, device=dev)
                           if defer else None)
    cache.next_free_block = torch.full((1,), total_local, dtype=torch.int32, device=dev)
    cache.local_region_starts = (torch.arange(layers * batch * kv_heads, dtype=torch.int64, device=dev)
                                 .view(layers, batch, kv_heads) * window)
    cache.local_ptr = 0
    cache.local_length = 0
    cache.total_blocks = total_blocks
    cache.wgkv_batch = batch
    cache.cache_seqlens = torch.zeros(batch, kv_heads, dtype=torch.int32, device=dev)
    # device copy of (local_length, local_ptr), used when a decode step runs as a CUDA graph
    cache.ring_state = torch.zeros(2, dtype=torch.int32, device=dev)
    cache.wgkv_device_ring = False
    if snapkv_window:  # SnapKV state (modeling_layers.py:1249-1262), a batch axis on the query window
        cache.snapkv_query_buffer = torch.zeros(layers, batch, snapkv_window, q_heads, head_dim, dtype=dtype,
                                                device=dev)
        cache.snapkv_query_length = 0
        cache.snapkv_query_ptr = 0
        cache.snapkv_evict_count = 0
        cache.free_block_ids = torch.zeros(total_blocks, dtype=torch.int32, device=dev)
        cache.free_block_count = torch.zeros(1, dtype=torch.int32, device=dev)
    if quest:  # per-page key bounds for QUEST selection (modeling_layers.py:1232-1240)
        cache.quest_block_key_min = torch.zeros(total_blocks, head_dim, dtype=dtype, device=dev)
        cache.quest_block_key_max = torch.zeros(total_blocks, head_dim, dtype=dtype, device=dev)
    s = WgkvPool()
    s.k = cache.block_pool_k.data_ptr()
    s.v = cache.block_pool_v.data_ptr()
    s.block_table = cache.block_table.data_ptr()
    s.global_lengths = cache.global_lengths.data_ptr()
    s.local_is_global = cache.local_is_global.data_ptr()
    s.local_pre_key = cache.local_pre_key.data_ptr() if defer else None
    s.next_free_block = cache.next_free_block.data_ptr()
    s.err = err_word(dev).data_ptr()
    s.total_blocks = total_blocks
    s.layers, s.batch, s.kv_heads, s.head_dim = layers, batch, kv_heads, head_dim
    s.window, s.page = window, page
    s.max_blocks_per_head, s.max_tokens_per_head = max_blocks_per_head, max_tokens_per_head
    s.ring_state = cache.ring_state.data_ptr()
    s.quest_min = cache.quest_block_key_min.data_ptr() if quest else None
    s.quest_max = cache.quest_block_key_max.data_ptr() if quest else None
    s.free_ids = cache.free_block_ids.data_ptr() if snapkv_window else None
    s.free_count = cache.free_block_count.data_ptr() if snapkv_window else None
    cache.wgkv_pool = s
    cache.gated_kv_initialized = True
    return cache


def pool_ref(cache) -> int:
    return ctypes.addressof(cache.wgkv_pool)


RING_ON_DEVICE = -1  # WGKV_RING_ON_DEVICE


def ring_to_device(cache):
    """Copy the host ring position (local_length, local_ptr) into ``cache.ring_state``."""
    cache.ring_state.copy_(torch.tensor([cache.local_length, cache.local_ptr], dtype=torch.int32))


def advance_host_ring(cache, window):
    """The host-side update decode_wrapper makes after the last layer (:1408-1413)."""
    if cache.local_length < window:
        cache.local_length += 1
    else:
        cache.local_ptr = (cache.local_ptr + 1) % window
