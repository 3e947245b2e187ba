/*
 * wgkv.h -- C ABI of the B200 (sm_100a) WG-KV admission hot path.
 *
 * Every entry point takes plain device pointers, sizes and element strides,
 * plus a CUDA stream passed as `void*` (a cudaStream_t; NULL = legacy default
 * stream).  Nothing here allocates device memory, synchronises the device or
 * reads device data back to the host: capacity violations detected on the
 * device are OR-ed into the caller's device error word `err` (WGKV_ERR_*),
 * which the caller inspects when it chooses to synchronise.  Host-detectable
 * argument errors are returned immediately as a negative status.
 *
 * bf16 tensors are `uint16_t` bit patterns (bfloat16).  The innermost
 * (head_dim) axis must be contiguous; other strides are in elements.
 *
 * Reference interfaces replaced (EMCLab-Sinica/WG-KV, src/modeling_layers.py):
 *   wgkv_gate_scores          GatingPredictor.forward fast path :170-196 + `g_scores > g_threshold` :1465
 *   wgkv_prefill_admit        prefill_wrapper ring fill + compaction :1290-1331
 *   wgkv_promote              migrate_local_kv_to_global :674-763
 *   wgkv_decode_append        decode_wrapper ring append / local_is_global :1390-1413, tables :1429-1436
 *   wgkv_decode_gate_append   self_attn_forward_patch gate on one token :1579 fused with the above
 *   wgkv_refresh_ring         refresh_local_is_global :1169-1180 (deferred gating)
 *   wgkv_sparse_indices       generate_sparse_indices :385-409 (+ generate_block_offset :321-349,
 *                             generate_column_index :352-381)
 *   wgkv_sparse_prefill       sparse_attn_func (vLLM fork) as called at :1366-1374
 *   wgkv_paged_decode         flash_attn_with_kvcache_wrapper_triton_handle + split/reduce kernels :818-1140
 *                             (and the batched flash_attn_with_kvcache_wrapper :766-811)
 */
#ifndef WGKV_H_
#define WGKV_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define WGKV_API __attribute__((visibility("default")))
#else
#define WGKV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status / device error bits ---------------------------------------- */
#define WGKV_OK 0
#define WGKV_EINVAL (-1)      /* bad argument (shape, alignment, unsupported size) */
#define WGKV_ECUDA (-2)       /* a CUDA runtime call failed (launch, attribute query) */
#define WGKV_ENOSPC (-3)      /* caller-provided workspace too small */

#define WGKV_ERR_HEAD_CAPACITY 0x1 /* tokens of a head exceed max_tokens_per_head */
#define WGKV_ERR_POOL_EXHAUSTED 0x2 /* page allocation past total_blocks */
#define WGKV_ERR_TIMEOUT 0x4        /* an mbarrier wait gave up (kernel returned early) */
#define WGKV_ERR_BAD_PAGE 0x8       /* a page id outside [0, total_blocks) was met */

/* Library version and build info. */
WGKV_API int wgkv_version(void);
/* Number of SMs of the current device (cached per device). <0 on error. */
WGKV_API int wgkv_num_sms(void);

/* ---- (a7, a8) ragged paged decode attention ----------------------------- */
/*
 * out[b, 0, hq, :] = softmax(q[b, 0, hq, :] . K_h^T * scale) V_h, h = hq / G,
 * over the first cache_seqlens[b, h] logical tokens of (b, h), whose pages are
 * block_table[b, h, 0 .. ceil(len / page_size)).  Entries past that are never
 * read.  A head of length 0 yields zeros.  Probabilities are rounded to bf16
 * before the PV product and m / l / acc are fp32, as in the reference Triton
 * kernel (modeling_layers.py:916-937).
 *
 *   q, out           (B, 1, Hq, D) contiguous bf16
 *   k_cache, v_cache (num_pages, page_size, D) contiguous bf16
 *   cache_seqlens    (B, Hk) int32, contiguous
 *   block_table      (B, Hk, max_pages) int32, row stride `table_stride` (elements)
 * Constraints: D in {64, 128}; page_size % 16 == 0; Hq % Hk == 0; Hq / Hk <= 16.
 * workspace: wgkv_paged_decode_workspace_size() bytes; its first
 * B*Hk*4 bytes are per-head counters that must be zero before the first call
 * (the kernel leaves them zero again).  Calls sharing a workspace must be
 * stream-ordered.
 */
WGKV_API size_t wgkv_paged_decode_workspace_size(int batch, int num_q_heads, int num_kv_heads, int head_dim);
WGKV_API int wgkv_paged_decode(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, int64_t num_pages,
                      int page_size, const int32_t* cache_seqlens, const int32_t* block_table, int64_t table_stride,
                      int batch, int num_q_heads, int num_kv_heads, int head_dim, float softmax_scale, uint16_t* out,
                      void* workspace, size_t workspace_bytes, int* err, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* WGKV_H_ */
