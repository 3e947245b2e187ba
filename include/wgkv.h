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
 *   wgkv_ring_advance         local_ptr / local_length update in decode_wrapper :1408-1413
 *   wgkv_decode_append        decode_wrapper ring append / local_is_global :1390-1413, tables :1429-1436
 *   wgkv_decode_gate_append   self_attn_forward_patch gate on one token :1579 fused with the above
 *   wgkv_decode_prologue      the same, fused behind q/k norm + RoPE (modeling_llama.py:265-271,
 *                             modeling_qwen3.py:236-239)
 *   (deferred gating)         refresh_local_is_global :1169-1180 is wgkv_gate_scores over the ring rows
 *   wgkv_sparse_indices       generate_sparse_indices :385-409 (+ generate_block_offset :321-349,
 *                             generate_column_index :352-381)
 *   wgkv_sparse_prefill       sparse_attn_func (vLLM fork) as called at :1366-1374
 *   wgkv_quest_select         quest_select_blocks :452-576 (page bounds kept by prefill :1333-1347 and
 *                             promotion :744-761)
 *   wgkv_snapkv_evict         snapkv_evict :595-671 (free list reused by promotion :694-709)
 *   wgkv_paged_decode         flash_attn_with_kvcache_wrapper_triton_handle + split/reduce kernels :818-1140
 *                             (and the batched flash_attn_with_kvcache_wrapper :766-811)
 *   wgkv_oproj_allreduce      self.o_proj(attn_output) (src/modeling_llama.py:286) of a KV-head-sharded
 *                             layer plus the sum over GPUs (the reference has no tensor parallelism)
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
#define WGKV_ERR_BAD_POSITION 0x10  /* a RoPE position outside the caller's tables (clamped) */

/*
 * Failure-path self test (no reference counterpart): one CTA waits on an mbarrier that nothing ever
 * completes, with the bounded wait every pipelined kernel here uses; after the limit (about two
 * seconds) it ORs WGKV_ERR_TIMEOUT into *err and returns.  No fault, no trap: the context stays
 * usable, which is what the tests of the error path check.
 */
WGKV_API int wgkv_selftest_wait_limit(int* err, void* stream);

/* Library version and build info. */
WGKV_API int wgkv_version(void);
/* Number of SMs of the current device (cached per device). <0 on error. */
WGKV_API int wgkv_num_sms(void);

/* ---- paged pool state (shared by the admission entry points) ------------ */
/*
 * Device-resident state that the reference attaches to its DynamicCache in
 * prefill_wrapper (modeling_layers.py:1196-1288), with a batch axis added.
 * Layout (batch 1 reproduces the reference exactly):
 *   k, v             (total_blocks * page, head_dim) bf16 rows; page p = rows [p*page, (p+1)*page)
 *   block_table      (layers, batch, kv_heads, max_blocks_per_head) int32; entries [0, window/page) are
 *                    the ring pages, global pages follow; unused entries hold total_blocks - 1
 *   global_lengths   (layers, batch, kv_heads) int32
 *   local_is_global  (layers, batch, kv_heads, window) uint8
 *   local_pre_key    (layers, batch, kv_heads, window, head_dim) bf16, deferred gating only (else NULL)
 *   next_free_block  device int32 scalar: bump allocator of global pages
 *   err              device int32 error word (WGKV_ERR_* bits)
 *   ring_state       optional device int32[2] = {local_length, local_ptr}: the ring position the
 *                    reference keeps on the host (:1286-1287, :1408-1413).  When set, the decode entry
 *                    points accept WGKV_RING_ON_DEVICE in place of insert_pos / local_ptr and read the
 *                    position here, and wgkv_ring_advance moves it, so that one captured CUDA graph
 *                    replays every decode step.  NULL = positions come from the host only.
 *   quest_min/max    optional (total_blocks, head_dim) bf16: element-wise min / max of the keys of every
 *                    global page (quest_block_key_min / _max, :1232-1240), kept by wgkv_prefill_admit and
 *                    wgkv_promote when set; read by wgkv_quest_select.  NULL = QUEST off.
 *   free_ids/count   optional SnapKV free list (free_block_ids, :1262): device int32[total_blocks] and its
 *                    device length.  wgkv_snapkv_evict appends the pages it empties; wgkv_promote takes
 *                    new pages from the list's tail first (:694-709).  NULL = no free list.
 * The ring slot s of (layer l, batch b, head h) is pool row ((l*batch + b)*kv_heads + h)*window + s.
 */
typedef struct wgkv_pool {
  uint16_t* k;
  uint16_t* v;
  int32_t* block_table;
  int32_t* global_lengths;
  uint8_t* local_is_global;
  uint16_t* local_pre_key;
  int32_t* next_free_block;
  int* err;
  int64_t total_blocks;
  int32_t layers;
  int32_t batch;
  int32_t kv_heads;
  int32_t head_dim;
  int32_t window;
  int32_t page;
  int32_t max_blocks_per_head;
  int32_t max_tokens_per_head;
  int32_t* ring_state;
  uint16_t* quest_min;
  uint16_t* quest_max;
  int32_t* free_ids;
  int32_t* free_count;
} wgkv_pool;

/* insert_pos / local_ptr value that means "read the position from pool->ring_state". */
#define WGKV_RING_ON_DEVICE (-1)

/* `act` flag of the gate entry points: GatingPredictor's conv path (g_fast_path=False). */
#define WGKV_GATE_SILU 0x1
#define WGKV_GATE_CONV 0x2

/* ---- (a1, a2) write gate + admission mask --------------------------------- */
/*
 * scores[b,h,t] = bf16(sigmoid(w2_h . act(W1_h x + b1_h) + b2_h)), mask = scores > threshold,
 * x = concat of the inputs selected by `input_mask` (bit 0 pre_k, bit 1 post_k, bit 2 value, in that
 * order), each optionally RMS-normalised with its row of `norm_w` (3, D) when norm_w != NULL.  Rounds
 * to bf16 where the reference's bf16 tensors do; GEMM accumulation is fp32.  `act` bit 0 picks the
 * activation (0 GELU (erf), 1 SiLU); bit 1 (WGKV_GATE_CONV) picks the reference's default
 * g_fast_path=False numerics (:198-205: each 1x1 conv rounds once, after its bias, and the score is
 * floored at bf16(score_floor) = g_epsilon by torch.clamp before the threshold); without it the
 * einsum fast path (:185-196: products rounded, then the bias added and rounded; score_floor unused).
 * Inputs are (B, Hk, L, D) with element strides (sb, sh, st); unused inputs may be NULL.  w1
 * (Hk, inner, I), b1 (Hk, inner), w2 (Hk, inner), b2 (Hk) bf16.  Either output may be NULL; strides
 * are in elements.
 * Constraints: D in {64, 128}; inner % 8 == 0; I = D * popcount(input_mask) <= 384.
 */
WGKV_API int wgkv_gate_scores(const uint16_t* pre_k, int64_t pk_sb, int64_t pk_sh, int64_t pk_st,
                              const uint16_t* post_k, int64_t k_sb, int64_t k_sh, int64_t k_st,
                              const uint16_t* value, int64_t v_sb, int64_t v_sh, int64_t v_st, int batch,
                              int kv_heads, int seq_len, int head_dim, int input_mask, const uint16_t* w1,
                              const uint16_t* b1, const uint16_t* w2, const uint16_t* b2, const uint16_t* norm_w,
                              float rms_eps, int inner, int act, float score_floor, float threshold,
                              uint16_t* scores, int64_t s_sb, int64_t s_sh, int64_t s_st, uint8_t* mask, int64_t m_sb, int64_t m_sh, int64_t m_st,
                              void* stream);

/* ---- (a3) prefill: ring fill + admission compaction ----------------------- */
/*
 * For every (b, h) of `layer`: the last min(L, window) tokens go to ring slots 0.. (with their mask
 * bits into local_is_global, and pre_k into local_pre_key when the pool has it); the admitted tokens
 * among the first L - window are packed, in token order, into freshly allocated contiguous global
 * pages.  Pages are allocated from next_free_block in (b, h) order, so batch 1 reproduces the
 * reference's page ids.  On a capacity violation nothing of the layer is written and err gets
 * WGKV_ERR_HEAD_CAPACITY / WGKV_ERR_POOL_EXHAUSTED (reference asserts :1313-1321).
 * k, v, pre_k: (B, Hk, L, D) strided; g_mask (B, Hk, L) uint8 strided.
 */
WGKV_API size_t wgkv_prefill_admit_workspace_size(int batch, int kv_heads, int seq_len);
WGKV_API int wgkv_prefill_admit(const wgkv_pool* pool, int layer, int seq_len, const uint16_t* k, int64_t k_sb,
                                int64_t k_sh, int64_t k_st, const uint16_t* v, int64_t v_sb, int64_t v_sh,
                                int64_t v_st, const uint16_t* pre_k, int64_t pk_sb, int64_t pk_sh, int64_t pk_st,
                                const uint8_t* g_mask, int64_t m_sb, int64_t m_sh, int64_t m_st, void* workspace,
                                size_t workspace_bytes, void* stream);

/* ---- (a4) lazy promotion ---------------------------------------------------- */
/*
 * For every (layer, b, h) whose ring slot `local_ptr` is admitted: append that slot's K/V to the
 * head's global pages (a new page from next_free_block when the length is a multiple of `page`,
 * allocated in (layer, b, h) order) and bump global_lengths.  One launch for all layers, as the
 * reference does at layer 0 when the ring is full (:1470-1471).  Capacity violations write nothing
 * and set err; while err holds a capacity error (not yet cleared by the caller) promotions do nothing.
 * Two launches: the allocation pass (one CTA) and the row copies (one CTA per 32 heads).  local_ptr = WGKV_RING_ON_DEVICE: the slot is ring_state[1], and nothing happens while
 * ring_state[0] < window (the reference promotes only once the ring is full, :1470).
 */
WGKV_API int wgkv_promote(const wgkv_pool* pool, int local_ptr, void* stream);

/*
 * Advance pool->ring_state by one decoded token, as decode_wrapper does after the last layer
 * (:1408-1413): local_length += 1 while the ring fills, else local_ptr = (local_ptr + 1) % window.
 * One single-thread launch; requires pool->ring_state.
 */
WGKV_API int wgkv_ring_advance(const wgkv_pool* pool, void* stream);

/* ---- (a5, a6) decode: ring append + attention lengths --------------------- */
/*
 * Writes k_new/v_new (B, Hk, D; strides sb, sh) into ring slot `insert_pos` of `layer`, pre_k_new into
 * local_pre_key when non-NULL, and cache_seqlens[b, h] = cur_local_len + global_lengths[layer, b, h]
 * (modeling_layers.py:1390-1400, :1429-1432).  The admission bit of the new token is written by
 * wgkv_gate_scores straight into local_is_global.  insert_pos = WGKV_RING_ON_DEVICE (pool->ring_state
 * set): insert_pos and cur_local_len are taken from ring_state (cur_local_len is then ignored).
 */
WGKV_API int wgkv_decode_append(const wgkv_pool* pool, int layer, int insert_pos, int cur_local_len,
                                const uint16_t* k_new, int64_t k_sb, int64_t k_sh, const uint16_t* v_new,
                                int64_t v_sb, int64_t v_sh, const uint16_t* pre_k_new, int64_t pk_sb, int64_t pk_sh,
                                int32_t* cache_seqlens, void* stream);

/*
 * Decode step without deferred gating, fused: the write gate on the new token of every (b, h)
 * (same MLP, inputs, `act` flags, floor and rounding as wgkv_gate_scores) writes its admission bit into ring slot
 * `insert_pos` of local_is_global, k_new / v_new go into that ring slot, and cache_seqlens is
 * filled as in wgkv_decode_append -- one launch (reference: the gate call in
 * self_attn_forward_patch :1579 + decode_wrapper :1390-1400, :1429-1432).  Gate inputs are the
 * (B, Hk, D) rows pre_k_new / k_new / v_new selected by input_mask (bit 0 pre_k, 1 post_k = k_new,
 * 2 v = v_new).  Run the layer-0 promotion (wgkv_promote) before this, as it reads the old bit.
 * insert_pos = WGKV_RING_ON_DEVICE reads the position from ring_state, as wgkv_decode_append does.
 */
WGKV_API int wgkv_decode_gate_append(const wgkv_pool* pool, int layer, int insert_pos, int cur_local_len,
                                     const uint16_t* pre_k_new, int64_t pk_sb, int64_t pk_sh, const uint16_t* k_new,
                                     int64_t k_sb, int64_t k_sh, const uint16_t* v_new, int64_t v_sb, int64_t v_sh,
                                     int input_mask, const uint16_t* w1, const uint16_t* b1, const uint16_t* w2,
                                     const uint16_t* b2, const uint16_t* norm_w, float rms_eps, int inner, int act,
                                     float score_floor, float threshold, int32_t* cache_seqlens, void* stream);

/*
 * Decode prologue fused into the above (the q/k/v projection epilogue of the patched attention
 * layers, modeling_llama.py:265-271 and modeling_qwen3.py:236-239, followed by the gate and the
 * ring append).  qkv is each sequence's projection row [q heads | k heads | v heads] x D bf16, rows
 * qkv_sb elements apart.  For every (b, kv head h): optional RMS norm of the k row and the q rows
 * with k_norm / q_norm (D bf16 weights, eps qk_eps; Qwen3), then RoPE at position *position with
 * rope_cos / rope_sin tables (n_positions, D) bf16, rounding as the bf16 torch expressions
 * x*cos + rotate_half(x)*sin do.  The rotated q rows of h's query heads go to q_out (B, q_heads, D);
 * the k row before RoPE is the gate's pre_k, the rotated k row its post_k and the ring's key.  With
 * w1 == NULL (deferred gating) no gate runs and pre_k goes into local_pre_key.  A position outside
 * [0, n_positions) is clamped and flags WGKV_ERR_BAD_POSITION.
 */
WGKV_API int wgkv_decode_prologue(const wgkv_pool* pool, int layer, int insert_pos, int cur_local_len,
                                  const uint16_t* qkv, int64_t qkv_sb, int q_heads, const uint16_t* q_norm,
                                  const uint16_t* k_norm, float qk_eps, const uint16_t* rope_cos,
                                  const uint16_t* rope_sin, const int64_t* position, int64_t n_positions,
                                  uint16_t* q_out, int input_mask, const uint16_t* w1, const uint16_t* b1,
                                  const uint16_t* w2, const uint16_t* b2, const uint16_t* norm_w, float rms_eps,
                                  int inner, int act, float score_floor, float threshold, int32_t* cache_seqlens,
                                  void* stream);

/* ---- KV-head tensor parallelism: o_proj fused with the sum over GPUs ------ */
#define WGKV_TP_MAX_WORLD 8

/*
 * One GPU's view of a tensor-parallel group (one process per GPU).  partial[r] / flags[r] are rank
 * r's buffers as mapped in this process (this rank's own pointers at index `rank`, the peers' through
 * CUDA IPC: wgkv_ipc_handle / wgkv_ipc_open).  partial: wgkv_tp_partial_bytes(max_rows, max_cols),
 * 16-byte aligned; flags: wgkv_tp_flag_bytes(max_cols), zeroed before first use; ctr: two uint32 of
 * this GPU, zeroed before first use.  All ranks must use the same max_rows / max_cols.
 */
typedef struct wgkv_peer_group {
  int32_t rank;
  int32_t world;
  int32_t max_rows;
  int32_t max_cols;
  void* partial[WGKV_TP_MAX_WORLD];
  uint32_t* flags[WGKV_TP_MAX_WORLD];
  uint32_t* ctr;
} wgkv_peer_group;

WGKV_API size_t wgkv_tp_partial_bytes(int max_rows, int max_cols);
WGKV_API size_t wgkv_tp_flag_bytes(int max_cols);

/*
 * Export / import a device buffer for the peers of a group.  wgkv_ipc_handle writes the 64-byte
 * CUDA IPC handle of the allocation holding `ptr` and ptr's byte offset in it; wgkv_ipc_open maps a
 * peer's allocation into this process (base address; add the peer's offset), wgkv_ipc_close unmaps.
 */
WGKV_API int wgkv_ipc_handle(const void* ptr, void* handle_out, size_t* offset_out);
WGKV_API int wgkv_ipc_open(const void* handle, void** base_out);
WGKV_API int wgkv_ipc_close(void* base);

/*
 * y (rows, n_out) bf16 = sum over the group's GPUs of a_r (rows, k) . w_r^T, w_r (n_out, k) the
 * columns of W_o that multiply this GPU's query heads (row-parallel o_proj).  One kernel: each CTA
 * computes 32 output columns of this GPU's product (mma.sync, fp32 accumulate, rounded to bf16 as
 * the unfused GEMM output is), publishes them to the peers and sums the peers' copies of the same
 * columns in rank order (fp32), so every GPU gets identical bits.  Every rank must make the same
 * sequence of calls (same rows, n_out) on its own stream; with world == 1 it is the plain GEMM.
 * Waits on peers are bounded (~2 s): a peer that never arrives sets WGKV_ERR_TIMEOUT in err and the
 * call completes with undefined y.  k % 128 == 0, n_out % 32 == 0, n_out / 32 <= the SM count,
 * rows <= max_rows, 16-byte aligned rows.
 */
WGKV_API int wgkv_oproj_allreduce(const uint16_t* a, int64_t lda, int rows, int k, const uint16_t* w, int n_out,
                                  uint16_t* y, int64_t ldy, const wgkv_peer_group* group, int* err, void* stream);

/* ---- QUEST block selection (use_quest) ------------------------------------ */
/*
 * quest_select_blocks (:452-576) for every (b, h) of `layer`: score each full global page by
 * max_g bf16(sum_d bf16(q_gd * (q_gd >= 0 ? quest_max : quest_min))), keep the ring pages
 * (ceil(cur_local_len / page) of them), the best `capacity - 1` full pages (all when they fit; ties
 * go to the lower position) and the trailing partial page, where capacity = min(ceil(max(budget -
 * cur_local_len, 0) / page), global pages).  Writes out_seqlens (B, Hk) = the tokens kept and
 * out_table (B, Hk, out_stride) = their page ids, ring pages first, then the global pages in
 * position order -- inputs for wgkv_paged_decode.  q (B, q_heads, D) bf16, rows q_sb elements apart.
 * cur_local_len = WGKV_RING_ON_DEVICE takes the ring length from pool->ring_state.  out_stride must
 * be at least wgkv_quest_table_stride(window, page, token_budget, max_blocks_per_head); workspace of
 * wgkv_quest_workspace_size(pool) bytes (page score keys).
 */
WGKV_API size_t wgkv_quest_table_stride(int window, int page, int token_budget, int max_blocks_per_head);
WGKV_API size_t wgkv_quest_workspace_size(const wgkv_pool* pool);
WGKV_API int wgkv_quest_select(const wgkv_pool* pool, int layer, int cur_local_len, const uint16_t* q, int64_t q_sb,
                               int q_heads, int token_budget, int32_t* out_seqlens, int32_t* out_table,
                               int64_t out_stride, void* workspace, size_t workspace_bytes, void* stream);

/* ---- SnapKV eviction (snapkv_enabled) ------------------------------------- */
/*
 * snapkv_evict (:595-671) for every (layer, b, h): scores each global token by the softmax attention
 * of the recorded window queries (bf16(bf16(q . k) * scale), fp32 softmax), max over the head's G
 * query heads, mean over the window, max-pooled with the odd kernel_size; evicts the
 * int(glen * evict_ratio) lowest (ties: lower positions first), packs the kept tokens to the front
 * of the head's pages, returns emptied pages to the free list in (layer, b, h) order (their table
 * entries become total_blocks - 1) and shrinks global_lengths.  queries (layers, batch, window,
 * q_heads, head_dim) bf16 -- the snapkv_query_buffer of :1255-1258 with a batch axis.  Requires
 * pool->free_ids; G = q_heads / kv_heads must divide 16 and window * G must be a multiple of 16.
 * The caller decides when (the reference: total global tokens > snapkv_max_cached_tokens, :1502-1507).
 */
WGKV_API size_t wgkv_snapkv_workspace_size(const wgkv_pool* pool, int window, int q_heads);
WGKV_API int wgkv_snapkv_evict(const wgkv_pool* pool, const uint16_t* queries, int window, int q_heads,
                               float softmax_scale, double evict_ratio, int kernel_size, void* workspace,
                               size_t workspace_bytes, void* stream);

/* ---- decoder plumbing of the end-to-end driver (no reference counterpart on the hot path) ---- */
/*
 * out[r] = (x[r] * rsqrt(mean(x[r]^2) + eps)).to(bf16) * weight, rows of `cols` bf16 (cols % 8 == 0,
 * cols <= 8192), row strides in elements (multiples of 8), 16-byte aligned pointers.  The RMSNorm
 * of the Llama / Qwen3 decoder layers around the patched attention (modeling_llama.py decoder layer).
 */
WGKV_API int wgkv_rms_norm(const uint16_t* x, int64_t x_stride, const uint16_t* weight, int rows, int cols,
                           float eps, uint16_t* out, int64_t out_stride, void* stream);
/*
 * out[r, j] = silu(gate_up[r, j]).to(bf16) * gate_up[r, inter + j]: the MLP activation of the same
 * decoder layers on a fused [gate | up] projection (inter % 8 == 0).
 */
WGKV_API int wgkv_silu_mul(const uint16_t* gate_up, int64_t gu_stride, int rows, int inter, uint16_t* out,
                           int64_t out_stride, void* stream);
/*
 * out[r * out_stride] = argmax_j logits[r, j] (int64; the first index among equal maxima, as
 * torch.argmax) for rows <= 65535 fp32 rows of n entries.  workspace of
 * wgkv_argmax_workspace_size(rows, n) bytes whose first `rows` ints are zero before the first call
 * (the kernel leaves them zero).
 */
WGKV_API size_t wgkv_argmax_workspace_size(int rows, int n);
WGKV_API int wgkv_argmax(const float* logits, int64_t row_stride, int rows, int n, int64_t* out, int64_t out_stride,
                         void* workspace, size_t workspace_bytes, void* stream);

/*
 * y[i, j] = sum_k x[i, k] * w[j, k] (+ residual[i, j]) for the few rows of a decode step
 * (1 <= m <= 8): x (m, k) bf16 rows x_stride apart, w (n, k) bf16 row-major (a torch Linear
 * weight), fp32 accumulation, y bf16 (or fp32 when out_f32, then without residual) rows y_stride
 * apart.  residual may alias y (in-place y += x w^T).  k % 8 == 0, 16-byte aligned x and w.
 * rms_weight != NULL: x is RMS-normalised first, exactly as wgkv_rms_norm would (k weights, eps).
 * paired: w = [gate (n/2 rows) | up (n/2 rows)] and y (m, n/2) = silu(x gate^T) * (x up^T) with the
 * roundings of wgkv_silu_mul on the bf16 projections (no residual, bf16 out).
 */
WGKV_API int wgkv_skinny_gemm(const uint16_t* x, int64_t x_stride, int m, const uint16_t* w, int n, int k, void* y,
                              int64_t y_stride, int out_f32, const uint16_t* residual, int64_t r_stride,
                              const uint16_t* rms_weight, float rms_eps, int paired, void* stream);

/* ---- (a9-a11) vertical-slash sparse indices -------------------------------- */
/*
 * generate_sparse_indices (:385-409) on the device.  Outputs (R = ceil(L / block), P = min(W/block, R)):
 *   block_count (R) int32, block_offset (R, P+1) int32  -- generate_block_offset :321-349
 *   column_count (B, Hk, R) int32, column_index (B, Hk, ci_stride) int32 -- generate_column_index
 *   :352-381: column_index holds every admitted token index in ascending order (entries past the
 *   head's count are left untouched), column_count[i] = #admitted < block*(i-P)+1 for i >= P, else 0.
 *   max_count (device int32, may be NULL) receives max over (b, h) of the admitted count (Gmax, :369),
 *   as an atomicMax: zero it first.  ci_stride must be >= L.  Requires window % block == 0.
 */
WGKV_API size_t wgkv_sparse_indices_workspace_size(int batch, int kv_heads, int seq_len);
WGKV_API int wgkv_sparse_indices(const uint8_t* g_mask, int64_t m_sb, int64_t m_sh, int64_t m_st, int batch,
                                 int kv_heads, int seq_len, int window, int block, int32_t* block_count,
                                 int32_t* block_offset, int32_t* column_count, int32_t* column_index,
                                 int64_t ci_stride, int32_t* max_count, void* workspace, size_t workspace_bytes,
                                 void* stream);

/* ---- (a12) block-sparse causal prefill attention --------------------------- */
/*
 * out[b, q, hq, :] = softmax over keys k of (q . k * scale) V, where k ranges over the union of
 *   - the band blocks [block_offset[i, c], block_offset[i, c] + block) for c < block_count[i], and
 *   - the admitted columns column_index[b, h, 0, 0 .. column_count[b, h, i]),
 * intersected with k <= q (causal), i = q / block, h = hq / (Hq / Hk).  This is the attention that
 * sparse_attn_func computes for the indices of generate_sparse_indices (as pinned by
 * utils/test_sparse_attn.py:34-93); band and column sets are disjoint for such indices.
 *   q   (B, L, Hq, D) bf16, strides (sb, sl, sh) in elements (last axis contiguous)
 *   k,v (B, L, Hk, D) bf16, strides likewise; out (B, L, Hq, D) bf16 strided likewise
 *   block_count (R), block_offset (R, bo_stride), column_count (B, Hk, R), column_index (B, Hk, ci_stride)
 * Constraints: D in {64, 128}; block == 64; Hq % Hk == 0.
 * Even GQA groups with 16-byte-aligned [B*L, H*D] row views run on the tcgen05 kernel (TMA + TMEM);
 * other shapes on an mma.sync kernel.  `err` (device word, may be NULL) receives WGKV_ERR_TIMEOUT if
 * a pipeline wait gives up.
 */
WGKV_API int wgkv_sparse_prefill(const uint16_t* q, int64_t q_sb, int64_t q_sl, int64_t q_sh, const uint16_t* k,
                                 int64_t k_sb, int64_t k_sl, int64_t k_sh, const uint16_t* v, int64_t v_sb,
                                 int64_t v_sl, int64_t v_sh, int batch, int seq_len, int num_q_heads,
                                 int num_kv_heads, int head_dim, const int32_t* block_count,
                                 const int32_t* block_offset, int64_t bo_stride, const int32_t* column_count,
                                 const int32_t* column_index, int64_t ci_stride, float softmax_scale, uint16_t* out,
                                 int64_t o_sb, int64_t o_sl, int64_t o_sh, int* err, void* stream);

/*
 * Same attention, reading the admitted-column keys from the paged pool instead of gathering them
 * from k / v: after wgkv_prefill_admit, the admitted tokens of (b, h) among the first L - window
 * sit in token order in contiguous pool rows starting at table[(b*Hk + h)*table_stride +
 * table_first] * page_size (table = the layer's block_table, table_first = window / page_size),
 * which is exactly column_index's order; every column the indices use lies in that range.  The
 * column tiles then load as plain 2D TMA tiles.  k / v still supply the local band.  The indices
 * must come from the mask the pool was filled with.  Internal to prefill_wrapper's fast path (the
 * reference has no separate interface for it; it computes sparse_attn_func's result).
 */
WGKV_API int wgkv_sparse_prefill_pooled(const uint16_t* q, int64_t q_sb, int64_t q_sl, int64_t q_sh,
                                        const uint16_t* k, int64_t k_sb, int64_t k_sl, int64_t k_sh,
                                        const uint16_t* v, int64_t v_sb, int64_t v_sl, int64_t v_sh, int batch,
                                        int seq_len, int num_q_heads, int num_kv_heads, int head_dim,
                                        const int32_t* block_count, const int32_t* block_offset, int64_t bo_stride,
                                        const int32_t* column_count, const int32_t* column_index, int64_t ci_stride,
                                        float softmax_scale, uint16_t* out, int64_t o_sb, int64_t o_sl, int64_t o_sh,
                                        const uint16_t* pool_k, const uint16_t* pool_v, int64_t pool_rows,
                                        const int32_t* table, int64_t table_stride, int table_first, int page_size,
                                        int* err, void* stream);

/*
 * Helper of the generic sparse_attn_func path: copies, for every (b, h), the K/V rows
 * column_index[b, h, 0 : column_count[b, h, R-1]) (the admitted columns the last row block uses,
 * which include every other row block's) into contiguous rows (b*Hk + h)*cap + c of out_k / out_v
 * ((B*Hk*cap, D) bf16, cap >= that count).  wgkv_sparse_prefill_pooled with a page table of
 * (b*Hk + h)*cap (page size 1) then reads them as plain 2D tiles.  No reference counterpart: the
 * reference gathers inside its (vLLM fork) kernel.
 */
WGKV_API int wgkv_gather_columns(const uint16_t* k, int64_t k_sb, int64_t k_sl, int64_t k_sh, const uint16_t* v,
                                 int64_t v_sb, int64_t v_sl, int64_t v_sh, int batch, int num_kv_heads, int head_dim,
                                 int seq_len, const int32_t* column_count, const int32_t* column_index,
                                 int64_t ci_stride, int64_t cap, uint16_t* out_k, uint16_t* out_v, void* stream);

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

/*
 * Paged decode without any device allocation -- no counterpart in the reference.
 *
 * For callers that cannot call cudaMalloc on the decode path: a serving engine
 * that owns the whole device-memory budget and hands kernels only its own
 * buffers, or a plugin invoked while its host framework captures a stream.
 * Same inputs, outputs and results as wgkv_paged_decode; the split-K scratch
 * (per-head counters + partial softmax states) lives in one static device
 * array of WGKV_PAGED_DECODE_STATIC_SCRATCH_BYTES inside libwgkv.so, which
 * every GPU that loads the library keeps until the process exits.
 *   - Needs (batch*kv_heads*4 rounded up to 256) + (batch*kv_heads + SMs) *
 *     (q_heads/kv_heads) * (head_dim + 2) * 4 bytes; larger problems return
 *     WGKV_ENOSPC and launch nothing (e.g. batch 64 x 8 kv heads x 4 groups x
 *     d 128 needs ~1.4 MiB and fits).
 *   - The first call on a device resolves the array's device address
 *     (cudaGetSymbolAddress) with that device current; make that first call
 *     before any stream capture.
 *   - Each call clears the counters with cudaMemsetAsync on `stream`; it calls
 *     no cudaMalloc / cudaFree.  All calls share the one array, so calls that
 *     can overlap on the GPU (different streams without ordering) race: order them.
 */
#define WGKV_PAGED_DECODE_STATIC_SCRATCH_BYTES (4u << 20)
WGKV_API int wgkv_paged_decode_noalloc(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                       int64_t num_pages, int page_size, const int32_t* cache_seqlens,
                                       const int32_t* block_table, int64_t table_stride, int batch, int num_q_heads,
                                       int num_kv_heads, int head_dim, float softmax_scale, uint16_t* out, int* err,
                                       void* stream);

#ifdef __cplusplus
}
#endif

#endif /* WGKV_H_ */
