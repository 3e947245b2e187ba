"""The two attention kernels as registered torch operators (``torch.ops.wgkv.*``).

``paged_decode`` and ``sparse_attn_func`` are plain Python calls over the C ABI.  Registering
them with ``torch.library`` makes them visible to torch's dispatcher: a caller that traces a
model (FakeTensor / meta shape propagation, ``torch.export``, ``torch.compile`` of the code
around the attention) sees one opaque operator with a known output shape instead of a ctypes
call it cannot trace.  The real implementation is CUDA only; there is no CPU kernel, so a CPU
tensor raises ``NotImplementedError`` from the dispatcher.

* ``torch.ops.wgkv.paged_decode(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale)``
  -- the decode kernel slot (src/modeling_layers.py:1007-1140, batched :766-811).
* ``torch.ops.wgkv.sparse_attn(q, k, v, block_count, block_offset, column_count, column_index,
  softmax_scale)`` -- the prefill kernel slot (``sparse_attn_func`` as called at
  src/modeling_layers.py:1366-1374), causal, without the log-sum-exp output.
"""
from __future__ import annotations

import torch

from .decode import paged_decode as _paged_decode
from .prefill import sparse_attn_func as _sparse_attn_func


@torch.library.custom_op("wgkv::paged_decode", mutates_args=(), device_types="cuda")
def paged_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, cache_seqlens: torch.Tensor,
                 block_table: torch.Tensor, softmax_scale: float) -> torch.Tensor:
    return _paged_decode(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale)


@paged_decode.register_fake
def _(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale):
    torch._check(q.dim() == 4 and q.shape[1] == 1, lambda: "q must be (B, 1, Hq, D)")
    torch._check(q.dtype == torch.bfloat16, lambda: "paged_decode supports bf16 inputs")
    torch._check(cache_seqlens.dim() == 2 and block_table.dim() == 3, lambda: "(B, Hk) lengths, (B, Hk, maxb) table")
    torch._check(q.shape[2] % cache_seqlens.shape[1] == 0, lambda: "Hq must be a multiple of Hk")
    return torch.empty(q.shape, dtype=q.dtype, device=q.device)


@torch.library.custom_op("wgkv::sparse_attn", mutates_args=(), device_types="cuda")
def sparse_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, block_count: torch.Tensor,
                block_offset: torch.Tensor, column_count: torch.Tensor, column_index: torch.Tensor,
                softmax_scale: float) -> torch.Tensor:
    return _sparse_attn_func(q, k, v, block_count, block_offset, column_count, column_index,
                             softmax_scale=softmax_scale)


@sparse_attn.register_fake
def _(q, k, v, block_count, block_offset, column_count, column_index, softmax_scale):
    torch._check(q.dim() == 4 and k.dim() == 4 and k.shape == v.shape, lambda: "q (B, L, Hq, D), k/v (B, L, Hk, D)")
    torch._check(q.dtype == torch.bfloat16, lambda: "sparse_attn supports bf16 inputs")
    torch._check(q.shape[2] % k.shape[2] == 0, lambda: "Hq must be a multiple of Hk")
    return torch.empty(q.shape, dtype=q.dtype, device=q.device)
