"""Vertical-slash sparse indices (generate_sparse_indices, src/modeling_layers.py:385-409)."""
from __future__ import annotations

import torch

from ._lib import check, lib
from .runtime import require_cuda, stream_ptr, workspace


def sparse_indices_into(g_mask, local_window_size, seq_len, block_size=64, column_index=None, max_count=None):
    """Device-only variant (no host sync): returns block_count (1,1,R), block_offset (1,1,R,P+1),
    column_count (B,Hk,R) and column_index (B,Hk,1,cap) with cap >= seq_len.  ``max_count``
    (int32 (1,) tensor, zeroed by the caller) receives Gmax."""
    require_cuda(g_mask, "g_mask")
    if g_mask.dtype == torch.bool:
        g_mask = g_mask.view(torch.uint8)
    B, Hk, L = g_mask.shape
    assert L == seq_len
    assert local_window_size % block_size == 0  # as the reference asserts (:394)
    dev = g_mask.device
    R = (L + block_size - 1) // block_size
    P = min(local_window_size // block_size, R)
    bc = torch.empty(1, 1, R, dtype=torch.int32, device=dev)
    bo = torch.empty(1, 1, R, P + 1, dtype=torch.int32, device=dev)
    cc = torch.empty(B, Hk, R, dtype=torch.int32, device=dev)
    if column_index is None:
        column_index = torch.zeros(B, Hk, 1, L, dtype=torch.int32, device=dev)
    assert column_index.shape[:3] == (B, Hk, 1) and column_index.shape[3] >= L and column_index.stride(3) == 1
    assert column_index.stride(0) == Hk * column_index.stride(1)
    nbytes = int(lib.wgkv_sparse_indices_workspace_size(B, Hk, L))
    ws = workspace(dev, "sparse_indices", nbytes)
    st = lib.wgkv_sparse_indices(g_mask.data_ptr(), g_mask.stride(0), g_mask.stride(1), g_mask.stride(2), B, Hk, L,
                                 local_window_size, block_size, bc.data_ptr(), bo.data_ptr(), cc.data_ptr(),
                                 column_index.data_ptr(), column_index.stride(1),
                                 max_count.data_ptr() if max_count is not None else None, ws.data_ptr(),
                                 ws.numel(), stream_ptr(dev))
    check(st, "wgkv_sparse_indices")
    return bc, bo, cc, column_index


def generate_sparse_indices(g_mask, local_window_size, batch_size, num_kv_heads, seq_len, device=None,
                            block_size=64):
    """Same signature and outputs as the reference (:385-409), including the
    (B, Hk, 1, Gmax) shape of column_index -- which, as in the reference
    (``.item()`` at :369), needs one host sync to learn Gmax."""
    assert g_mask.shape == (batch_size, num_kv_heads, seq_len)
    mc = torch.zeros(1, dtype=torch.int32, device=g_mask.device)
    bc, bo, cc, ci = sparse_indices_into(g_mask, local_window_size, seq_len, block_size, max_count=mc)
    gmax = int(mc.item())
    return bc, bo, cc, ci[..., :gmax].contiguous()
