"""Ragged paged decode attention -- the reference's decode kernel surface.

Drop-in for ``flash_attn_with_kvcache_wrapper_triton_handle`` /
``flash_attn_with_kvcache_wrapper_triton`` (src/modeling_layers.py:1007-1140)
and the batched ``flash_attn_with_kvcache_wrapper`` (:766-811), backed by
``wgkv_paged_decode`` in libwgkv.so.  Unlike the reference handle, building
the handle does no host sync and no host-side schedule: the split over
ragged heads is computed on the device.
"""
from __future__ import annotations

import torch

from ._lib import check, lib
from .runtime import err_word, require_cuda, stream_ptr, workspace


def _validate(q, k_cache, v_cache, cache_seqlens, block_table):
    for t, n in ((q, "q"), (k_cache, "k_cache"), (v_cache, "v_cache"), (cache_seqlens, "cache_seqlens"),
                 (block_table, "block_table")):
        require_cuda(t, n)
    if q.dtype != torch.bfloat16 or k_cache.dtype != torch.bfloat16 or v_cache.dtype != torch.bfloat16:
        # same exception type as the reference (:1021-1022)
        raise TypeError("This kernel only supports BF16 inputs for q, k_cache, and v_cache.")
    B, q_len, Hq, D = q.shape
    assert q_len == 1
    assert cache_seqlens.dim() == 2 and cache_seqlens.shape[0] == B
    Hk = cache_seqlens.shape[1]
    assert Hq % Hk == 0
    assert block_table.dim() == 3 and block_table.shape[:2] == (B, Hk)
    assert k_cache.dim() == 3 and k_cache.shape == v_cache.shape and k_cache.shape[2] == D
    return B, Hq, Hk, D


def paged_decode(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale, out=None):
    """out (B, 1, Hq, D) bf16 = GQA softmax attention of q over each (b, kv-head)'s pages."""
    B, Hq, Hk, D = _validate(q, k_cache, v_cache, cache_seqlens, block_table)
    q = q.contiguous()
    if not k_cache.is_contiguous() or not v_cache.is_contiguous():
        raise ValueError("k_cache / v_cache must be contiguous (num_pages, page_size, head_dim)")
    sl = cache_seqlens.to(torch.int32).contiguous()
    bt = block_table.to(torch.int32)
    if bt.stride(2) != 1 or bt.stride(0) != bt.shape[1] * bt.stride(1):
        bt = bt.contiguous()
    if out is None:
        out = torch.empty_like(q)
    dev = q.device
    nbytes = int(lib.wgkv_paged_decode_workspace_size(B, Hq, Hk, D))
    ws = workspace(dev, "paged_decode", nbytes, zero_prefix=((B * Hk * 4 + 255) // 256) * 256)
    st = lib.wgkv_paged_decode(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[0],
                               k_cache.shape[1], sl.data_ptr(), bt.data_ptr(), bt.stride(1), B, Hq, Hk, D,
                               float(softmax_scale), out.data_ptr(), ws.data_ptr(), ws.numel(),
                               err_word(dev).data_ptr(), stream_ptr(dev))
    check(st, "wgkv_paged_decode")
    return out


def flash_attn_with_kvcache_wrapper_triton_handle(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale,
                                                  num_splits=None, block_n=None, num_warps=None, num_stages=None):
    """Returns a zero-argument callable that launches the decode kernel.

    Signature of modeling_layers.py:1007-1018 (the tuning knobs are accepted
    and ignored: the split is derived on the device from the SM count).
    Accepts batch > 1.  Inputs are captured by reference, so the handle may be
    called repeatedly (e.g. timed, or captured in a CUDA graph)."""
    _validate(q, k_cache, v_cache, cache_seqlens, block_table)
    out = torch.empty_like(q)
    sl = cache_seqlens.to(torch.int32).contiguous()
    bt = block_table.to(torch.int32)

    def handle():
        return paged_decode(q, k_cache, v_cache, sl, bt, softmax_scale, out=out)

    return handle


def flash_attn_with_kvcache_wrapper_triton(*args, **kwargs):
    return flash_attn_with_kvcache_wrapper_triton_handle(*args, **kwargs)()


def flash_attn_with_kvcache_wrapper(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale):
    """Batched decode API of modeling_layers.py:766-811."""
    return paged_decode(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale)


def flash_attn_with_kvcache_wrapper_handle(*args, **kwargs):
    return lambda: flash_attn_with_kvcache_wrapper(*args, **kwargs)
