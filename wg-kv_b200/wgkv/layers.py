"""The WG-KV attention patch on the CUDA kernels: reference-named drop-ins.

Mirrors the operator surface the patched Llama/Qwen3 attention layers call
(src/modeling_llama.py:240-250, :273-287; src/modeling_layers.py):

* ``self_attn_forward_patch(self, gating_mode, attention_mask, past_key_value,
  input_shape, query_states, pre_key, key_states, value_states)`` (:1534)
* ``self_attn_forward_patch_inference`` (:1452), ``prefill_wrapper`` (:1183),
  ``decode_wrapper`` (:1379), ``migrate_local_kv_to_global`` (:674),
  ``refresh_local_is_global`` (:1169), ``quest_select_blocks`` (:452),
  ``snapkv_record_queries`` / ``snapkv_evict`` (:579, :595)
* ``self_attn_decode_fused``: the decode step fed by raw q/k/v projection rows
  (q/k norm + RoPE fused into the gate launch)

``self`` is the attention module (``layer_idx``, ``config``, ``head_dim``,
``scaling``, ``g_predictors`` and the kernel slots); ``past_key_value`` is any
attribute holder (the HF cache object), which gets the pool attributes of
:func:`wgkv.pool.init_pool`.  Differences from the reference, all on the
host side: batch > 1 is accepted (the pool has a batch axis); no step
synchronises the host (page allocation, compaction and the decode schedule
run on the device; SnapKV keeps the reference's one host read of the cached
total to decide on eviction); capacity violations are reported through the
device error word (``wgkv.check_errors()``), not an immediate assert.  With
``past_key_value.wgkv_device_ring`` set the ring position is read on the
device, so a whole decode step can be captured (``wgkv.DecodeGraph``).
"""
from __future__ import annotations

import torch

from ._lib import check, lib
from .indices import sparse_indices_into
from .pool import RING_ON_DEVICE, init_pool, pool_ref
from .prefill import sparse_attn_func, sparse_attn_func_pooled, sparse_attn_func_wrapper
from .runtime import stream_ptr, workspace


def _cfg(self):
    return self.config


def _maybe_init(self, past_key_value, batch_size, key_states):
    c = _cfg(self)
    if not getattr(past_key_value, "gated_kv_initialized", False):
        assert self.layer_idx == 0, "the pool is created by layer 0's prefill"
        init_pool(past_key_value, layers=c.num_hidden_layers, batch=batch_size, kv_heads=c.num_key_value_heads,
                  head_dim=self.head_dim, window=c.local_window_size, page=c.block_size,
                  max_total_tokens=c.max_total_tokens, max_tokens_per_head=c.max_tokens_per_head,
                  device=key_states.device, dtype=key_states.dtype, defer=bool(getattr(c, "g_defer", False)),
                  quest=bool(getattr(c, "use_quest", False)),
                  snapkv_window=c.snapkv_window_size if getattr(c, "snapkv_enabled", False) else None,
                  q_heads=getattr(c, "num_attention_heads", None))
    elif self.layer_idx == 0:
        raise AssertionError("prefill on an initialised cache (the reference asserts the same, :1197)")


def _device_ring(cache):
    """True while decode steps take the ring position from ``cache.ring_state`` (graph capture)."""
    return getattr(cache, "wgkv_device_ring", False)


def _promote_now(cache, W):
    return _device_ring(cache) or cache.local_length == W


def _s4(t):
    return (t.data_ptr(), t.stride(0), t.stride(1), t.stride(2)) if t is not None else (None, 0, 0, 0)


def prefill_wrapper(self, past_key_value, query_states, pre_key, key_states, value_states, batch_size, q_seq_len,
                    device, g_mask, local_blocks_per_head):
    """Ring fill + admission compaction + sparse indices + sparse prefill (:1183-1376).

    q (B, Hq, L, D), pre_key/key/value (B, Hk, L, D), g_mask (B, Hk, L) bool/uint8.
    Returns (B, L, Hq, D)."""
    c = _cfg(self)
    _maybe_init(self, past_key_value, batch_size, key_states)
    if g_mask.dtype == torch.bool:
        g_mask = g_mask.view(torch.uint8)
    W = c.local_window_size
    L = q_seq_len
    defer = past_key_value.local_pre_key is not None
    nbytes = int(lib.wgkv_prefill_admit_workspace_size(batch_size, c.num_key_value_heads, max(L - W, 0)))
    ws = workspace(device, "prefill_admit", nbytes)
    st = lib.wgkv_prefill_admit(pool_ref(past_key_value), self.layer_idx, L, *_s4(key_states), *_s4(value_states),
                                *_s4(pre_key if defer else None), *_s4(g_mask), ws.data_ptr(), ws.numel(),
                                stream_ptr(device))
    check(st, "wgkv_prefill_admit")
    past_key_value.local_length = min(L, W)
    bc, bo, cc, ci = sparse_indices_into(g_mask, W, L, 64)
    if self.prefill_kernel in (sparse_attn_func_wrapper, sparse_attn_func):
        # fast path: the admitted columns were just packed into contiguous pool pages
        return sparse_attn_func_pooled(query_states.transpose(1, 2), key_states.transpose(1, 2),
                                       value_states.transpose(1, 2), bc, bo, cc, ci, past_key_value.block_pool_k,
                                       past_key_value.block_pool_v, past_key_value.block_table[self.layer_idx],
                                       W // c.block_size, c.block_size, softmax_scale=self.scaling)
    return self.prefill_kernel(query_states.transpose(1, 2), key_states.transpose(1, 2),
                               value_states.transpose(1, 2), bc, bo, cc, ci, softmax_scale=self.scaling,
                               causal=True, return_softmax_lse=False)


def migrate_local_kv_to_global(self, past_key_value, device, local_blocks_per_head):
    """Lazy promotion of every (layer, b, h) ring slot at local_ptr (:674-763), one launch.

    With the device ring (``wgkv_device_ring``) the slot, and whether the ring is full yet, are
    read on the device, so the launch is made on every step."""
    ptr = RING_ON_DEVICE if _device_ring(past_key_value) else int(past_key_value.local_ptr)
    st = lib.wgkv_promote(pool_ref(past_key_value), ptr, stream_ptr(device))
    check(st, "wgkv_promote")


def refresh_local_is_global(self, past_key_value, device):
    """Deferred gating: re-score this layer's whole ring (:1169-1180)."""
    c = _cfg(self)
    l = self.layer_idx
    B, Hk, W, D = past_key_value.wgkv_batch, c.num_key_value_heads, c.local_window_size, self.head_dim
    n_ring = c.num_hidden_layers * B * Hk * W
    ring_k = past_key_value.block_pool_k[:n_ring].view(c.num_hidden_layers, B, Hk, W, D)[l]
    ring_v = past_key_value.block_pool_v[:n_ring].view(c.num_hidden_layers, B, Hk, W, D)[l]
    self.g_predictors.admit(past_key_value.local_pre_key[l], ring_k, ring_v, c.g_threshold,
                            past_key_value.local_is_global[l])


def decode_wrapper(self, past_key_value, query_states, pre_key, key_states, value_states, device, g_mask,
                   local_blocks_per_head, appended=False):
    """Ring append + (deferred) admission + ragged paged attention for one token (:1379-1449).

    ``g_mask`` (B, Hk, 1): the new token's admission bit, or None when it was
    already written into ``local_is_global`` by the fused gate (or deferred)."""
    c = _cfg(self)
    W = c.local_window_size
    l = self.layer_idx
    if past_key_value.local_length < W:
        insert_pos = past_key_value.local_length
        cur = past_key_value.local_length + 1
    else:
        insert_pos = past_key_value.local_ptr
        cur = W
    defer = past_key_value.local_pre_key is not None
    dr = _device_ring(past_key_value)
    if not appended:
        _append(self, past_key_value, l, RING_ON_DEVICE if dr else insert_pos, cur, pre_key, key_states,
                value_states, defer, device)
    if g_mask is not None:
        if dr:
            raise NotImplementedError("a precomputed g_mask needs the host ring position (no device ring)")
        past_key_value.local_is_global[l, :, :, insert_pos] = g_mask[:, :, 0].to(torch.uint8)
    elif defer and insert_pos == W - 1:
        refresh_local_is_global(self, past_key_value, device)
    if l == c.num_hidden_layers - 1:
        if dr:
            check(lib.wgkv_ring_advance(pool_ref(past_key_value), stream_ptr(device)), "wgkv_ring_advance")
        if past_key_value.local_length < W:
            past_key_value.local_length = cur
        else:
            past_key_value.local_ptr = (past_key_value.local_ptr + 1) % W
    T = c.block_size
    k_cache = past_key_value.block_pool_k.view(past_key_value.total_blocks, T, self.head_dim)
    v_cache = past_key_value.block_pool_v.view(past_key_value.total_blocks, T, self.head_dim)
    if getattr(c, "use_quest", False):
        cache_seqlens, block_table = quest_select_blocks(self, query_states, past_key_value, local_blocks_per_head,
                                                         device, RING_ON_DEVICE if dr else cur)
    else:
        cache_seqlens, block_table = past_key_value.cache_seqlens, past_key_value.block_table[l]
    handle = self.decode_kernel_handle(query_states.transpose(1, 2), k_cache, v_cache, cache_seqlens, block_table,
                                       self.scaling)
    return self.decode_kernel_executor(handle)


def quest_select_blocks(self, query_states, past_key_value, local_blocks_per_head, device, local_tokens_total):
    """QUEST page selection (:452-576) on the device (``wgkv_quest_select``), batched.

    query_states (B, Hq, 1, D).  Returns (cache_seqlens (B, Hk) int32, block_table (B, Hk, S) int32):
    the ring pages, the best full global pages by their key-bound score within
    ``config.quest_token_budget`` (ties to the lower position) and the trailing partial page, in
    position order (the reference lists the full pages in score order; attention does not depend on
    it).  ``local_tokens_total`` may be ``RING_ON_DEVICE`` (-1) under graph capture."""
    c = _cfg(self)
    assert c.quest_token_budget is not None
    s = past_key_value.wgkv_pool
    B, Hq, _, D = query_states.shape
    q = query_states[:, :, 0]
    if q.stride(1) != D or q.stride(2) != 1:
        q = q.contiguous()
    stride = int(lib.wgkv_quest_table_stride(s.window, s.page, int(c.quest_token_budget), s.max_blocks_per_head))
    seqlens = torch.empty(B, s.kv_heads, dtype=torch.int32, device=device)
    table = torch.empty(B, s.kv_heads, stride, dtype=torch.int32, device=device)
    ws = workspace(device, "quest", int(lib.wgkv_quest_workspace_size(pool_ref(past_key_value))))
    st = lib.wgkv_quest_select(pool_ref(past_key_value), self.layer_idx, int(local_tokens_total), q.data_ptr(),
                               q.stride(0), Hq, int(c.quest_token_budget), seqlens.data_ptr(), table.data_ptr(),
                               stride, ws.data_ptr(), ws.numel(), stream_ptr(device))
    check(st, "wgkv_quest_select")
    return seqlens, table


def _append(self, past_key_value, l, insert_pos, cur, pre_key, key_states, value_states, defer, device):
    """Ring append + cache_seqlens (wgkv_decode_append)."""
    k1 = key_states[:, :, 0]
    v1 = value_states[:, :, 0]
    p1 = pre_key[:, :, 0] if (defer and pre_key is not None) else None
    st = lib.wgkv_decode_append(pool_ref(past_key_value), l, insert_pos, cur, k1.data_ptr(), k1.stride(0),
                                k1.stride(1), v1.data_ptr(), v1.stride(0), v1.stride(1),
                                p1.data_ptr() if p1 is not None else None, p1.stride(0) if p1 is not None else 0,
                                p1.stride(1) if p1 is not None else 0, past_key_value.cache_seqlens.data_ptr(),
                                stream_ptr(device))
    check(st, "wgkv_decode_append")


def self_attn_forward_patch_inference(self, past_key_value, input_shape, query_states, pre_key, key_states,
                                      value_states, g_scores, g_mask=None):
    """:1452-1509.  Either ``g_scores`` (thresholded here, as the reference
    does) or a precomputed uint8 ``g_mask`` may be given; with neither on a
    decode step the new token's bit is expected in ``local_is_global``
    already (fused gate) or deferred."""
    c = _cfg(self)
    batch_size, q_seq_len = input_shape
    device = query_states.device
    is_prefilling = q_seq_len > 1
    if g_mask is None and g_scores is not None:
        g_mask = (g_scores > c.g_threshold).to(torch.uint8)
    assert c.local_window_size % c.block_size == 0
    local_blocks_per_head = c.local_window_size // c.block_size
    if (not is_prefilling) and self.layer_idx == 0 and _promote_now(past_key_value, c.local_window_size):
        migrate_local_kv_to_global(self, past_key_value, device, local_blocks_per_head)
    if is_prefilling:
        out = self.prefill_wrapper(self, past_key_value, query_states, pre_key, key_states, value_states,
                                   batch_size, q_seq_len, device, g_mask, local_blocks_per_head)
    else:
        out = self.decode_wrapper(self, past_key_value, query_states, pre_key, key_states, value_states, device,
                                  g_mask, local_blocks_per_head)
    _snapkv_after(self, past_key_value, query_states)
    return out


def self_attn_forward_patch(self, gating_mode, attention_mask, past_key_value, input_shape, query_states, pre_key,
                            key_states, value_states):
    """:1534-1629, inference mode (gating_mode 3) only: training and the
    comparison baselines are outside this library.

    Prefill: the gate writes the admission mask (one kernel).  Decode without
    deferral: the gate writes the new token's bit straight into the cache's
    ``local_is_global`` ring slot (after the layer-0 promotion has read the
    old bit), so no scores tensor is materialised."""
    if gating_mode != 3:
        raise NotImplementedError("only WG-KV inference (gating_mode=3) is implemented on the CUDA path")
    assert attention_mask is None
    assert past_key_value is not None
    c = _cfg(self)
    batch_size, q_len = input_shape
    kv_seq_len = key_states.size(2)
    device = query_states.device
    if kv_seq_len > 1:
        B, Hk, L, _ = key_states.shape
        g_mask = torch.empty(B, Hk, L, dtype=torch.uint8, device=device)
        self.g_predictors.admit(pre_key, key_states, value_states, c.g_threshold, g_mask)
        out = self_attn_forward_patch_inference(self, past_key_value, input_shape, query_states, pre_key,
                                                key_states, value_states, None, g_mask=g_mask)
        return out, None, None
    if getattr(c, "g_defer", False):
        out = self_attn_forward_patch_inference(self, past_key_value, input_shape, query_states, pre_key,
                                                key_states, value_states, None)
        return out, None, None
    W = c.local_window_size
    local_blocks_per_head = W // c.block_size
    l = self.layer_idx
    if l == 0 and _promote_now(past_key_value, W):
        migrate_local_kv_to_global(self, past_key_value, device, local_blocks_per_head)
    if _device_ring(past_key_value):
        insert_pos, cur = RING_ON_DEVICE, 0
    elif past_key_value.local_length < W:
        insert_pos, cur = past_key_value.local_length, past_key_value.local_length + 1
    else:
        insert_pos, cur = past_key_value.local_ptr, W
    # one fused launch: gate on the new key -> admission bit in the ring slot, K/V append, cache_seqlens
    self.g_predictors.decode_admit_append(past_key_value, l, insert_pos, cur, pre_key, key_states, value_states,
                                          c.g_threshold)
    out = self.decode_wrapper(self, past_key_value, query_states, pre_key, key_states, value_states, device, None,
                              local_blocks_per_head, appended=True)
    _snapkv_after(self, past_key_value, query_states)
    return out, None, None


def self_attn_decode_fused(self, past_key_value, qkv, q_heads, position, rope_cos, rope_sin, q_norm=None,
                           k_norm=None, qk_eps=1e-6):
    """Decode step of ``self_attn_forward_patch`` (gating_mode 3) fed by the raw q/k/v projection rows.

    The patched layers rotate q/k and keep the pre-RoPE key before calling the patch
    (src/modeling_llama.py:265-287, src/modeling_qwen3.py:236-239); here that prologue runs inside
    the gate + append launch (``wgkv_decode_prologue``): optional q/k RMS norm, RoPE at the device
    position ``position`` (1-element int64) from the (n, D) tables, gate on the pre-RoPE key (or,
    with g_defer, the pre-key store), ring append, lengths.  Then the layer-0 promotion order,
    the deferred rescoring and the paged attention are those of the unfused patch.
    qkv (B, (Hq + 2 Hk) D) bf16 -> attention output (B, 1, Hq, D)."""
    c = _cfg(self)
    W = c.local_window_size
    l = self.layer_idx
    device = qkv.device
    B = qkv.shape[0]
    if l == 0 and _promote_now(past_key_value, W):
        migrate_local_kv_to_global(self, past_key_value, device, W // c.block_size)
    if _device_ring(past_key_value):
        insert_pos, cur = RING_ON_DEVICE, 0
    elif past_key_value.local_length < W:
        insert_pos, cur = past_key_value.local_length, past_key_value.local_length + 1
    else:
        insert_pos, cur = past_key_value.local_ptr, W
    q = torch.empty(B, q_heads, self.head_dim, dtype=qkv.dtype, device=device)
    defer = bool(getattr(c, "g_defer", False))
    self.g_predictors.decode_prologue(past_key_value, l, insert_pos, cur, qkv, q_heads, position, rope_cos,
                                      rope_sin, q, c.g_threshold, q_norm=q_norm, k_norm=k_norm, qk_eps=qk_eps,
                                      gate=not defer)
    return self.decode_wrapper(self, past_key_value, q.view(B, q_heads, 1, self.head_dim), None, None, None,
                               device, None, W // c.block_size, appended=True)


def snapkv_record_queries(self, past_key_value, query_states):
    """:579-592 with a batch axis: keep the last ``snapkv_window_size`` queries of every layer
    (post-RoPE, (B, Hq, L, D)) in ``snapkv_query_buffer``; length / pointer advance at the last layer."""
    c = _cfg(self)
    win = c.snapkv_window_size
    buf = past_key_value.snapkv_query_buffer[self.layer_idx]  # (B, win, Hq, D)
    L = query_states.shape[2]
    if L > 1:
        take = min(win, L)
        buf[:, :take].copy_(query_states[:, :, L - take:].transpose(1, 2))
        if self.layer_idx == c.num_hidden_layers - 1:
            past_key_value.snapkv_query_length = take
            past_key_value.snapkv_query_ptr = take % win
    else:
        buf[:, past_key_value.snapkv_query_ptr].copy_(query_states[:, :, 0])
        if self.layer_idx == c.num_hidden_layers - 1:
            past_key_value.snapkv_query_length = min(win, past_key_value.snapkv_query_length + 1)
            past_key_value.snapkv_query_ptr = (past_key_value.snapkv_query_ptr + 1) % win


def snapkv_evict(self, past_key_value, device, local_blocks_per_head):
    """:595-671 for every layer and head at once (``wgkv_snapkv_evict``)."""
    c = _cfg(self)
    assert past_key_value.snapkv_query_length == c.snapkv_window_size
    nbytes = int(lib.wgkv_snapkv_workspace_size(pool_ref(past_key_value), c.snapkv_window_size,
                                                c.num_attention_heads))
    ws = workspace(device, "snapkv", nbytes)
    st = lib.wgkv_snapkv_evict(pool_ref(past_key_value), past_key_value.snapkv_query_buffer.data_ptr(),
                               c.snapkv_window_size, c.num_attention_heads, float(self.scaling),
                               float(c.snapkv_evict_ratio), int(c.snapkv_kernel_size), ws.data_ptr(), ws.numel(),
                               stream_ptr(device))
    check(st, "wgkv_snapkv_evict")


def _snapkv_after(self, past_key_value, query_states):
    """The SnapKV hook that follows the attention of every layer (:1500-1507): record the queries,
    and after the last layer evict when the global tokens exceed snapkv_max_cached_tokens (one host
    read of the total, as in the reference)."""
    c = _cfg(self)
    if not getattr(c, "snapkv_enabled", False):
        return
    if _device_ring(past_key_value):
        raise NotImplementedError("SnapKV decides on the host; it is not captured in decode graphs")
    snapkv_record_queries(self, past_key_value, query_states)
    if self.layer_idx == c.num_hidden_layers - 1 and \
            int(past_key_value.global_lengths.sum().item()) > c.snapkv_max_cached_tokens:
        past_key_value.snapkv_evict_count += 1
        snapkv_evict(self, past_key_value, query_states.device, c.local_window_size // c.block_size)
