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
from .runtime import check_errors  # noqa: F401
