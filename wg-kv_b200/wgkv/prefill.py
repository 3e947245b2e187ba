"""Block-sparse prefill attention: the ``sparse_attn_func`` surface.

Drop-in for ``vllm.vllm_flash_attn.sparse_attn_func`` as the reference calls
it (src/modeling_layers.py:1366-1374, ``sparse_attn_func_wrapper`` :448-449),
backed by ``wgkv_sparse_prefill``.
"""
from __future__ import annotations

import torch

from ._lib import check, lib
from .runtime import err_word, require_cuda, stream_ptr, workspace


def sparse_attn_func(q, k, v, block_count, block_offset, column_count, column_index, softmax_scale=None,
                     causal=True, return_softmax_lse=False, out=None):
    """q (B, L, Hq, D), k/v (B, L, Hk, D) bf16 -> (B, L, Hq, D) bf16.

    ``block_count`` (1, 1, R) / ``block_offset`` (1, 1, R, P+1) describe the
    local band shared by all heads; ``column_count`` (B, Hk, R) /
    ``column_index`` (B, Hk, 1, Gmax) the admitted columns per KV head."""
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        require_cuda(t, n)
        if t.dtype != torch.bfloat16:
            raise TypeError("sparse_attn_func supports bf16 q/k/v")
    if not causal:
        raise NotImplementedError("the vertical-slash prefill path is causal")
    if return_softmax_lse:
        raise NotImplementedError("return_softmax_lse is not used by the WG-KV path")
    B, L, Hq, D = q.shape
    Hk = k.shape[2]
    assert k.shape == (B, L, Hk, D) and v.shape == k.shape and Hq % Hk == 0
    if softmax_scale is None:
        softmax_scale = D ** -0.5

    def lastdim(t):
        return t if t.stride(-1) == 1 else t.contiguous()

    q, k, v = lastdim(q), lastdim(k), lastdim(v)
    R = (L + 63) // 64
    bc = block_count.reshape(-1).to(torch.int32).contiguous()
    bo = block_offset.reshape(R, -1).to(torch.int32).contiguous()
    cc = column_count.to(torch.int32).contiguous()
    ci = column_index.to(torch.int32)
    assert ci.dim() == 4 and ci.shape[:3] == (B, Hk, 1)
    if ci.numel() == 0:  # Gmax == 0: no admitted columns anywhere, column_count is all zero
        ci = torch.zeros(B, Hk, 1, 1, dtype=torch.int32, device=q.device)
    if ci.stride(3) != 1 or ci.stride(0) != Hk * ci.stride(1):
        ci = ci.contiguous()
    if out is None:
        out = torch.empty(B, L, Hq, D, dtype=q.dtype, device=q.device)
    cap = ci.shape[3]
    if _tc_eligible(q, k, v, out) and B * Hk * cap < 2 ** 31:
        # compact the admitted columns into contiguous rows, then read them as plain TMA tiles
        ws = workspace(q.device, "columns", 2 * B * Hk * cap * D * 2)
        ck = ws[:B * Hk * cap * D * 2].view(torch.bfloat16).view(B * Hk * cap, D)
        cv = ws[B * Hk * cap * D * 2:2 * B * Hk * cap * D * 2].view(torch.bfloat16).view(B * Hk * cap, D)
        st = lib.wgkv_gather_columns(k.data_ptr(), k.stride(0), k.stride(1), k.stride(2), v.data_ptr(), v.stride(0),
                                     v.stride(1), v.stride(2), B, Hk, D, L, cc.data_ptr(), ci.data_ptr(), ci.stride(1),
                                     cap, ck.data_ptr(), cv.data_ptr(), stream_ptr(q.device))
        check(st, "wgkv_gather_columns")
        base = (torch.arange(B * Hk, dtype=torch.int32, device=q.device) * cap).view(B, Hk, 1)
        return sparse_attn_func_pooled(q, k, v, block_count, block_offset, cc, ci, ck, cv, base, 0, 1,
                                       softmax_scale=softmax_scale, out=out)
    st = lib.wgkv_sparse_prefill(q.data_ptr(), q.stride(0), q.stride(1), q.stride(2), k.data_ptr(), k.stride(0),
                                 k.stride(1), k.stride(2), v.data_ptr(), v.stride(0), v.stride(1), v.stride(2), B, L,
                                 Hq, Hk, D, bc.data_ptr(), bo.data_ptr(), bo.stride(0), cc.data_ptr(), ci.data_ptr(),
                                 ci.stride(1), float(softmax_scale), out.data_ptr(), out.stride(0), out.stride(1),
                                 out.stride(2), err_word(q.device).data_ptr(), stream_ptr(q.device))
    check(st, "wgkv_sparse_prefill")
    return out


def _tc_eligible(q, k, v, out):
    """Shapes the tensor-core kernel takes (mirrors the check in sparse_prefill_tc.cu)."""
    B, L, Hq, D = q.shape
    Hk = k.shape[2]
    if (Hq // Hk) % 2 or D not in (64, 128):
        return False
    for t in (q, k, v):
        if t.stride(2) != D or t.stride(1) % 8 or (B > 1 and t.stride(0) != L * t.stride(1)) or t.data_ptr() % 16:
            return False
    return out.data_ptr() % 16 == 0 and all(x % 8 == 0 for x in out.stride()[:3])


def sparse_attn_func_wrapper(*args, **kwargs):
    return sparse_attn_func(*args, **kwargs)


def sparse_attn_func_pooled(q, k, v, block_count, block_offset, column_count, column_index, pool_k, pool_v,
                            block_table, table_first, page_size, softmax_scale=None, out=None):
    """``sparse_attn_func`` whose admitted-column keys are read from the paged pool.

    Valid right after the admission compaction of the same mask: the admitted
    tokens of (b, h) sit in token order in contiguous pool rows starting at
    ``block_table[b, h, table_first] * page_size``.  ``block_table`` is the
    layer's (B, Hk, maxb) table.  Same result as :func:`sparse_attn_func`."""
    for t, n in ((q, "q"), (k, "k"), (v, "v"), (pool_k, "pool_k"), (block_table, "block_table")):
        require_cuda(t, n)
    B, L, Hq, D = q.shape
    Hk = k.shape[2]
    if softmax_scale is None:
        softmax_scale = D ** -0.5
    R = (L + 63) // 64
    bc = block_count.reshape(-1).to(torch.int32).contiguous()
    bo = block_offset.reshape(R, -1).to(torch.int32).contiguous()
    cc = column_count.to(torch.int32).contiguous()
    ci = column_index.to(torch.int32)
    if ci.numel() == 0:
        ci = torch.zeros(B, Hk, 1, 1, dtype=torch.int32, device=q.device)
    if ci.stride(3) != 1 or ci.stride(0) != Hk * ci.stride(1):
        ci = ci.contiguous()
    assert block_table.dim() == 3 and block_table.stride(2) == 1 and block_table.stride(0) == Hk * block_table.stride(1)
    assert pool_k.is_contiguous() and pool_v.is_contiguous() and pool_k.shape[-1] == D
    if out is None:
        out = torch.empty(B, L, Hq, D, dtype=q.dtype, device=q.device)
    st = lib.wgkv_sparse_prefill_pooled(q.data_ptr(), q.stride(0), q.stride(1), q.stride(2), k.data_ptr(),
                                        k.stride(0), k.stride(1), k.stride(2), v.data_ptr(), v.stride(0),
                                        v.stride(1), v.stride(2), B, L, Hq, Hk, D, bc.data_ptr(), bo.data_ptr(),
                                        bo.stride(0), cc.data_ptr(), ci.data_ptr(), ci.stride(1),
                                        float(softmax_scale), out.data_ptr(), out.stride(0), out.stride(1),
                                        out.stride(2), pool_k.data_ptr(), pool_v.data_ptr(),
                                        pool_k.numel() // D, block_table.data_ptr(), block_table.stride(1),
                                        int(table_first), int(page_size), err_word(q.device).data_ptr(),
                                        stream_ptr(q.device))
    check(st, "wgkv_sparse_prefill_pooled")
    return out
