"""wgkv -- B200-native (sm_100a) WG-KV KV-admission hot path.

Host-side mirror of the reference's operator surface (EMCLab-Sinica/WG-KV,
src/modeling_layers.py) over the C ABI of libwgkv.so (include/wgkv.h).
"""
from ._lib import lib  # noqa: F401
from .decode import (  # noqa: F401
    flash_attn_with_kvcache_wrapper,
    flash_attn_with_kvcache_wrapper_handle,
    flash_attn_with_kvcache_wrapper_triton,
    flash_attn_with_kvcache_wrapper_triton_handle,
    paged_decode,
)
from .gate import GatingPredictor, GatingRMSNorm, load_gate_checkpoint  # noqa: F401
from .graph import DecodeGraph  # noqa: F401
from .indices import generate_sparse_indices, sparse_indices_into  # noqa: F401
from .layers import (  # noqa: F401
    decode_wrapper,
    migrate_local_kv_to_global,
    prefill_wrapper,
    quest_select_blocks,
    refresh_local_is_global,
    self_attn_forward_patch,
    self_attn_decode_fused,
    snapkv_evict,
    snapkv_record_queries,
    self_attn_forward_patch_inference,
)
from .pool import RING_ON_DEVICE, WgkvPool, advance_host_ring, init_pool, ring_to_device  # noqa: F401
from .prefill import sparse_attn_func, sparse_attn_func_pooled, sparse_attn_func_wrapper  # noqa: F401
from . import ops  # noqa: F401  (torch.ops.wgkv.paged_decode, torch.ops.wgkv.sparse_attn)
from .runtime import check_errors  # noqa: F401
from .tp import KVHeadParallelAttention, shard_gate, shard_o_proj  # noqa: F401


def attach(attn, config=None):
    """Install the WG-KV operator slots on an attention module, as
    LlamaAttention.__init__ does (src/modeling_llama.py:240-250), pointing at
    the CUDA implementations.  ``attn`` needs ``layer_idx``, ``head_dim``,
    ``scaling`` and ``g_predictors`` (a :class:`GatingPredictor`)."""
    if config is not None:
        attn.config = config
    attn.self_attn_forward_patch = self_attn_forward_patch
    attn.self_attn_decode_fused = self_attn_decode_fused
    attn.prefill_wrapper = prefill_wrapper
    attn.decode_wrapper = decode_wrapper
    attn.prefill_kernel = sparse_attn_func_wrapper
    attn.decode_kernel_handle = flash_attn_with_kvcache_wrapper_triton_handle
    attn.decode_kernel_executor = lambda func: func()
    return attn
