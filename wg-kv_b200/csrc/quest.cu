// QUEST block selection over the paged pool (reference: quest_select_blocks,
// src/modeling_layers.py:452-576), one CTA per (sequence, KV head).
//
// Each global page of a head carries the element-wise min and max of its keys (kept by the prefill
// compaction and the lazy promotion).  A page's score is the upper bound of q . k over the page,
// max over the G query heads of bf16(sum_d bf16(q_d * (q_d >= 0 ? kmax_d : kmin_d))) -- the bf16
// products and the float sum rounded to bf16 that the reference's torch expression computes.  The
// head keeps its ring pages, the `capacity - 1` best full global pages (all of them if they fit)
// and its trailing partial page, within a token budget.
//
// Selection: scores become order-preserving 16-bit keys in shared memory; a two-pass 8-bit radix
// histogram finds the k-th largest key; pages above it are taken, and among pages equal to it the
// lowest positions (torch.topk leaves the order of ties unspecified).  The chosen pages are written
// in ascending position order after the ring pages (attention does not depend on the order).
#include "common.cuh"

namespace wgkv {
namespace {

constexpr int kQsThreads = 256;
constexpr int kQsWarps = kQsThreads / 32;

// larger bf16 value -> larger key (negative values bit-flipped, positive ones offset by the sign bit)
WGKV_DEV uint32_t score_key(uint16_t b) { return (b & 0x8000u) ? (~uint32_t(b) & 0xFFFFu) : (uint32_t(b) | 0x8000u); }

// exclusive block scan of one int per thread; returns the block total through *total
WGKV_DEV int block_excl_scan_qs(int v, int* wsum, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffff, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[warp] = x;
  __syncthreads();
  int base = 0, tot = 0;
  for (int w = 0; w < kQsWarps; ++w) {
    if (w < warp) base += wsum[w];
    tot += wsum[w];
  }
  __syncthreads();  // wsum is reused by the next scan
  *total = tot;
  return base + x - v;
}

struct QuestArgs {
  wgkv_pool P;
};

__global__ void __launch_bounds__(kQsThreads) quest_select_kernel(QuestArgs qa, int layer, int cur, const uint16_t* q,
                                                                  int64_t q_sb, int Hq, int budget, int32_t* out_sl,
                                                                  int32_t* out_tab, int64_t out_stride) {
  const wgkv_pool& P = qa.P;
  extern __shared__ __align__(16) uint8_t qs_smem[];
  const int Hk = P.kv_heads, BH = P.batch * Hk, D = P.head_dim, T = P.page, W = P.window;
  const int bh = blockIdx.x, b = bh / Hk, h = bh - b * Hk, G = Hq / Hk;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  __shared__ int hist[256];
  __shared__ int wsum[kQsWarps];
  __shared__ int s_bin, s_take;
  if (cur < 0) {  // device ring position: the length after this step's append (decode_wrapper :1390-1396)
    const int len = P.ring_state[0];
    cur = len < W ? len + 1 : W;
  }
  const int local_blocks = (cur + T - 1) / T;
  const int rest = budget - cur;
  const int budget_blocks = ((rest > 0 ? rest : 0) + T - 1) / T;
  const int glen = P.global_lengths[int64_t(layer) * BH + bh];
  const int full = glen / T, rem = glen - full * T;
  const int nb = full + (rem > 0);
  const int cap = min(budget_blocks, nb);
  const int full_cap = cap > 0 ? cap - (rem > 0) : 0;
  const int32_t* trow = P.block_table + (int64_t(layer) * BH + bh) * P.max_blocks_per_head;
  const int32_t* grow = trow + W / T;
  int32_t* orow = out_tab + int64_t(bh) * out_stride;
  for (int i = tid; i < local_blocks; i += kQsThreads) orow[i] = trow[i];
  int nsel = 0;
  if (full_cap > 0 && full > 0) {
    if (full_cap >= full) {
      for (int i = tid; i < full; i += kQsThreads) orow[local_blocks + i] = grow[i];
      nsel = full;
    } else {
      float* qv = reinterpret_cast<float*>(qs_smem);             // [G][D]
      uint16_t* keys = reinterpret_cast<uint16_t*>(qv + G * D);  // [full]
      const uint16_t* qh = q + int64_t(b) * q_sb + int64_t(h) * G * D;
      for (int i = tid; i < G * D; i += kQsThreads) qv[i] = bf2f(qh[i]);
      __syncthreads();
      // ---- page scores: one warp per page ----
      for (int pos = warp; pos < full; pos += kQsWarps) {
        const int64_t pid = grow[pos];
        const uint16_t* mn = P.quest_min + pid * D;
        const uint16_t* mx = P.quest_max + pid * D;
        float best = -INFINITY;
        for (int g = 0; g < G; ++g) {
          float s = 0.f;
          for (int c = lane; c < D; c += 32) {
            const float x = qv[g * D + c];
            s += bf16_round(x * bf2f(x >= 0.f ? mx[c] : mn[c]));
          }
          for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffff, s, o);
          best = fmaxf(best, bf16_round(s));
        }
        if (lane == 0) keys[pos] = uint16_t(score_key(f2bf(best)));
      }
      // ---- k-th largest key: two 8-bit radix passes ----
      int need = full_cap;  // keys still to take at or below the current prefix
      uint32_t prefix = 0;
      for (int pass = 0; pass < 2; ++pass) {
        const int shift = pass == 0 ? 8 : 0;
        for (int i = tid; i < 256; i += kQsThreads) hist[i] = 0;
        __syncthreads();
        for (int i = tid; i < full; i += kQsThreads) {
          const uint32_t k = keys[i];
          if (pass == 0 || (k >> 8) == prefix) atomicAdd(&hist[(k >> shift) & 0xFF], 1);
        }
        __syncthreads();
        if (tid == 0) {
          int acc = 0, bin = 255;
          for (; bin > 0; --bin) {
            if (acc + hist[bin] >= need) break;
            acc += hist[bin];
          }
          s_bin = bin;          // the bin holding the k-th key
          s_take = need - acc;  // keys still to take from it
        }
        __syncthreads();
        prefix = pass == 0 ? uint32_t(s_bin) : (prefix << 8) | uint32_t(s_bin);
        need = s_take;
        __syncthreads();
      }
      const uint32_t kth = prefix;  // pages with key > kth are taken, plus the first `need` equal to it
      // ---- ordered compaction: contiguous position chunks per thread ----
      const int per = (full + kQsThreads - 1) / kQsThreads;
      const int i0 = min(full, tid * per), i1 = min(full, i0 + per);
      int eq = 0;
      for (int i = i0; i < i1; ++i) eq += keys[i] == kth;
      int tot;
      int eq_rank = block_excl_scan_qs(eq, wsum, &tot);
      int cnt = 0;
      for (int i = i0, r = eq_rank; i < i1; ++i) {
        const uint32_t k = keys[i];
        cnt += k > kth || (k == kth && r < need);
        r += k == kth;
      }
      int base = block_excl_scan_qs(cnt, wsum, &tot);
      for (int i = i0, r = eq_rank; i < i1; ++i) {
        const uint32_t k = keys[i];
        if (k > kth || (k == kth && r < need)) orow[local_blocks + base++] = grow[i];
        r += k == kth;
      }
      nsel = full_cap;
    }
  }
  if (tid == 0) {
    int tokens = cur + nsel * T;
    if (cap > 0 && rem > 0) {  // the trailing partial page is always kept when there is room
      orow[local_blocks + nsel] = grow[full];
      tokens += rem;
    }
    out_sl[bh] = tokens;
  }
}

}  // namespace
}  // namespace wgkv

using namespace wgkv;

extern "C" size_t wgkv_quest_table_stride(int window, int page, int token_budget, int max_blocks_per_head) {
  if (page <= 0 || window <= 0) return 0;
  const int lb = (window + page - 1) / page;
  const int bb = (token_budget > 0 ? token_budget + page - 1 : 0) / page + 1;
  const int g = max_blocks_per_head - window / page;
  return size_t(lb + (bb < g ? bb : g > 0 ? g : 0));
}

extern "C" int wgkv_quest_select(const wgkv_pool* pool, int layer, int cur_local_len, const uint16_t* q, int64_t q_sb,
                                 int q_heads, int token_budget, int32_t* out_seqlens, int32_t* out_table,
                                 int64_t out_stride, void* stream) {
  if (!pool || !pool->quest_min || !pool->quest_max || !q || !out_seqlens || !out_table || layer < 0 ||
      layer >= pool->layers || q_heads <= 0 || q_heads % pool->kv_heads || q_heads / pool->kv_heads > 16)
    return WGKV_EINVAL;
  if (cur_local_len == WGKV_RING_ON_DEVICE ? !pool->ring_state : (cur_local_len <= 0 || cur_local_len > pool->window))
    return WGKV_EINVAL;
  if (out_stride < int64_t(wgkv_quest_table_stride(pool->window, pool->page, token_budget, pool->max_blocks_per_head)))
    return WGKV_EINVAL;
  const int G = q_heads / pool->kv_heads;
  const size_t smem = size_t(G) * pool->head_dim * 4 + size_t(pool->max_blocks_per_head) * 2 + 16;
  constexpr size_t kMaxDyn = 200 * 1024;  // plus ~1 KB of static shared memory
  if (smem > kMaxDyn) return WGKV_EINVAL;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    if (cudaFuncSetAttribute(quest_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kMaxDyn)) !=
        cudaSuccess)
      return WGKV_ECUDA;
    attr[dev] = true;
  }
  QuestArgs qa{*pool};
  quest_select_kernel<<<pool->batch * pool->kv_heads, kQsThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      qa, layer, cur_local_len, q, q_sb, q_heads, token_budget, out_seqlens, out_table, out_stride);
  return cudaGetLastError() == cudaSuccess ? WGKV_OK : WGKV_ECUDA;
}
