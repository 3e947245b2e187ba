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
// Two kernels: the page scores (one CTA per 64 pages of a head, four pages' bounds in flight per
// warp) become order-preserving 16-bit keys in a workspace; per head, a two-pass 8-bit radix
// histogram over them finds the k-th largest key; pages above it are taken, and among pages equal to it the
// lowest positions (torch.topk leaves the order of ties unspecified).  The chosen pages are written
// in ascending position order after the ring pages (attention does not depend on the order).
#include "common.cuh"

namespace wgkv {
namespace {

constexpr int kQsThreads = 256;
constexpr int kQsWarps = kQsThreads / 32;

// larger bf16 value -> larger key (negative values bit-flipped, positive ones offset by the sign bit)
WGKV_DEV uint32_t score_key(uint16_t b) { return (b & 0x8000u) ? (~uint32_t(b) & 0xFFFFu) : (uint32_t(b) | 0x8000u); }


struct QuestArgs {
  wgkv_pool P;
};

// the per-head selection sizes of quest_select_blocks (:478-512)
struct QuestHead {
  int local_blocks, full, rem, cap, full_cap;
  WGKV_DEV QuestHead(const wgkv_pool& P, int layer, int bh, int cur, int budget) {
    const int T = P.page;
    local_blocks = (cur + T - 1) / T;
    const int rest = budget - cur;
    const int budget_blocks = ((rest > 0 ? rest : 0) + T - 1) / T;
    const int glen = P.global_lengths[int64_t(layer) * P.batch * P.kv_heads + bh];
    full = glen / T;
    rem = glen - full * T;
    cap = min(budget_blocks, full + (rem > 0));
    full_cap = cap > 0 ? cap - (rem > 0) : 0;
  }
  WGKV_DEV bool ranks() const { return full_cap > 0 && full > 0 && full_cap < full; }
};

WGKV_DEV int resolve_cur(const wgkv_pool& P, int cur) {
  if (cur >= 0) return cur;
  const int len = P.ring_state[0];  // device ring: the length after this step's append (:1390-1396)
  return len < P.window ? len + 1 : P.window;
}

#ifndef WGKV_QS_PPI
#define WGKV_QS_PPI 4
#endif
constexpr int kQsPPI = WGKV_QS_PPI;                 // pages per 8-lane group
constexpr int kQsPagesPerCta = kQsThreads / 8 * kQsPPI;

WGKV_DEV uint64_t qf2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
WGKV_DEV uint64_t qadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// Page scores of every head that has to rank its pages: eight lanes per page, each reading 16-byte
// chunks sub, sub + 8, ... of the page's min and max rows (so the eight lanes read whole 128-byte
// lines), against the group's queries in shared memory; the partial sums (even and odd dimensions
// in an f32x2 pair) are added over the eight lanes.  Writes order-preserving 16-bit keys to
// keys[bh][position].
template <int D, int G>
__global__ void __launch_bounds__(kQsThreads) quest_score_kernel(QuestArgs qa, int layer, int cur, const uint16_t* q,
                                                                 int64_t q_sb, int budget, uint16_t* keys,
                                                                 int key_stride) {
  constexpr int V = D / 8;    // 16-byte chunks per bound row
  constexpr int CPL = V / 8;  // chunks per lane
  constexpr int kPPI = kQsPPI;
  const wgkv_pool& P = qa.P;
  const int Hk = P.kv_heads, BH = P.batch * Hk;
  const int bh = blockIdx.y, b = bh / Hk, h = bh - b * Hk;
  cur = resolve_cur(P, cur);
  const QuestHead H(P, layer, bh, cur, budget);
  const int p0 = blockIdx.x * kQsPagesPerCta;
  if (!H.ranks() || p0 >= H.full) return;
  // queries as bf16 pairs, and per pair a mask selecting min (q < 0) or max (q >= 0, -0 included)
  __shared__ uint4 q2v[G * V], ngv[G * V];
  uint32_t* q2 = reinterpret_cast<uint32_t*>(q2v);
  uint32_t* ng = reinterpret_cast<uint32_t*>(ngv);
  const uint32_t* qh = reinterpret_cast<const uint32_t*>(q + int64_t(b) * q_sb + int64_t(h) * G * D);
  for (int i = threadIdx.x; i < G * D / 2; i += kQsThreads) {
    const uint32_t v = qh[i];
    q2[i] = v;
    const uint32_t lo_neg = (v & 0x8000u) && (v & 0x7FFFu) ? 0x0000FFFFu : 0u;
    const uint32_t hi_neg = (v & 0x80000000u) && (v & 0x7FFF0000u) ? 0xFFFF0000u : 0u;
    ng[i] = lo_neg | hi_neg;
  }
  __syncthreads();
  const int grp = threadIdx.x >> 3, sub = threadIdx.x & 7;
  const int32_t* grow = P.block_table + (int64_t(layer) * BH + bh) * P.max_blocks_per_head + P.window / P.page;
  uint4 lo[kPPI][CPL], hi[kPPI][CPL];
  int pos[kPPI];
#pragma unroll
  for (int u = 0; u < kPPI; ++u) {
    pos[u] = p0 + u * (kQsThreads / 8) + grp;
    const int64_t pid = pos[u] < H.full ? __ldg(grow + pos[u]) : 0;
    const uint4* mn4 = reinterpret_cast<const uint4*>(P.quest_min + pid * D);
    const uint4* mx4 = reinterpret_cast<const uint4*>(P.quest_max + pid * D);
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      if (pos[u] < H.full) {
        lo[u][i] = __ldg(mn4 + sub + 8 * i);
        hi[u][i] = __ldg(mx4 + sub + 8 * i);
      } else {
        lo[u][i] = hi[u][i] = make_uint4(0, 0, 0, 0);
      }
    }
  }
#pragma unroll
  for (int u = 0; u < kPPI; ++u) {
    uint64_t sum[G];
#pragma unroll
    for (int g = 0; g < G; ++g) sum[g] = qf2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      const int c = sub + 8 * i;
      const uint32_t lw[4] = {lo[u][i].x, lo[u][i].y, lo[u][i].z, lo[u][i].w};
      const uint32_t hw[4] = {hi[u][i].x, hi[u][i].y, hi[u][i].z, hi[u][i].w};
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const uint4 qq = q2v[g * V + c], nn = ngv[g * V + c];
        const uint32_t qw[4] = {qq.x, qq.y, qq.z, qq.w}, nw[4] = {nn.x, nn.y, nn.z, nn.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t sel = (hw[e] & ~nw[e]) | (lw[e] & nw[e]);
          // bf16(q * bound) for both halves: one round-to-nearest bf16x2 multiply
          const __nv_bfloat162 pr = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&qw[e]),
                                            *reinterpret_cast<const __nv_bfloat162*>(&sel));
          const uint32_t pu = *reinterpret_cast<const uint32_t*>(&pr);
          sum[g] = qadd2(sum[g], qf2(__uint_as_float(pu << 16), __uint_as_float(pu & 0xffff0000u)));
        }
      }
    }
    float best = -INFINITY;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float x, y;
      asm("mov.b64 {%0, %1}, %2;" : "=f"(x), "=f"(y) : "l"(sum[g]));
      float t = x + y;
      t += __shfl_xor_sync(0xffffffff, t, 1);
      t += __shfl_xor_sync(0xffffffff, t, 2);
      t += __shfl_xor_sync(0xffffffff, t, 4);
      best = fmaxf(best, bf16_round(t));
    }
    if (sub == 0 && pos[u] < H.full) keys[int64_t(bh) * key_stride + pos[u]] = uint16_t(score_key(f2bf(best)));
  }
}

__global__ void __launch_bounds__(kQsThreads) quest_select_kernel(QuestArgs qa, int layer, int cur, int budget,
                                                                  const uint16_t* gkeys, int key_stride,
                                                                  int32_t* out_sl, int32_t* out_tab,
                                                                  int64_t out_stride) {
  const wgkv_pool& P = qa.P;
  extern __shared__ __align__(16) uint8_t qs_smem[];
  const int Hk = P.kv_heads, BH = P.batch * Hk, T = P.page, W = P.window;
  const int bh = blockIdx.x;
  const int tid = threadIdx.x;
  __shared__ int hist[256];
  __shared__ int wsum[kQsWarps];
  __shared__ int s_bin, s_take;
  cur = resolve_cur(P, cur);
  const QuestHead H(P, layer, bh, cur, budget);
  const int local_blocks = H.local_blocks, full = H.full, full_cap = H.full_cap;
  // the pool's table is only read here and the output table only written: no aliasing
  const int32_t* __restrict__ trow = P.block_table + (int64_t(layer) * BH + bh) * P.max_blocks_per_head;
  const int32_t* __restrict__ grow = trow + W / T;
  int32_t* __restrict__ orow = out_tab + int64_t(bh) * out_stride;
  for (int i = tid; i < local_blocks; i += kQsThreads) orow[i] = trow[i];
  int nsel = 0;
  if (full_cap > 0 && full > 0) {
    if (full_cap >= full) {
      for (int i = tid; i < full; i += kQsThreads) orow[local_blocks + i] = grow[i];
      nsel = full;
    } else {
      uint16_t* keys = reinterpret_cast<uint16_t*>(qs_smem);  // [full]
      for (int i = tid; i < full; i += kQsThreads) keys[i] = gkeys[int64_t(bh) * key_stride + i];
      __syncthreads();
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
        // the bin holding the k-th key, and the keys still to take from it
        if (tid < 32) warp_pick_bin<true>(hist, need, &s_bin, &s_take);
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
      int eq_rank = block_excl_scan<kQsThreads>(eq, wsum, tot);
      int cnt = 0;
      for (int i = i0, r = eq_rank; i < i1; ++i) {
        const uint32_t k = keys[i];
        cnt += k > kth || (k == kth && r < need);
        r += k == kth;
      }
      int base = block_excl_scan<kQsThreads>(cnt, wsum, tot);
      // this thread's chosen pages: their table entries loaded together, then stored in order
      constexpr int kB = 8;
      for (int c0 = i0, r = eq_rank; c0 < i1; c0 += kB) {
        int32_t pid[kB];
        bool take[kB];
#pragma unroll
        for (int u = 0; u < kB; ++u) {
          const int i = c0 + u;
          const uint32_t k = i < i1 ? keys[i] : 0u;
          take[u] = i < i1 && (k > kth || (k == kth && r < need));
          r += i < i1 && k == kth;
          pid[u] = take[u] ? __ldg(grow + i) : 0;
        }
#pragma unroll
        for (int u = 0; u < kB; ++u)
          if (take[u]) orow[local_blocks + base++] = pid[u];
      }
      nsel = full_cap;
    }
  }
  if (tid == 0) {
    int tokens = cur + nsel * T;
    if (H.cap > 0 && H.rem > 0) {  // the trailing partial page is always kept when there is room
      orow[local_blocks + nsel] = grow[full];
      tokens += H.rem;
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

extern "C" size_t wgkv_quest_workspace_size(const wgkv_pool* pool) {
  if (!pool) return 0;
  return size_t(pool->batch) * pool->kv_heads * size_t(pool->max_blocks_per_head) * 2 + 256;
}

extern "C" int wgkv_quest_select(const wgkv_pool* pool, int layer, int cur_local_len, const uint16_t* q, int64_t q_sb,
                                 int q_heads, int token_budget, int32_t* out_seqlens, int32_t* out_table,
                                 int64_t out_stride, void* workspace, size_t workspace_bytes, void* stream) {
  if (!pool || !pool->quest_min || !pool->quest_max || !q || !out_seqlens || !out_table || !workspace ||
      layer < 0 || layer >= pool->layers || q_heads <= 0 || q_heads % pool->kv_heads ||
      q_heads / pool->kv_heads > 16)
    return WGKV_EINVAL;
  if (cur_local_len == WGKV_RING_ON_DEVICE ? !pool->ring_state : (cur_local_len <= 0 || cur_local_len > pool->window))
    return WGKV_EINVAL;
  if (out_stride < int64_t(wgkv_quest_table_stride(pool->window, pool->page, token_budget, pool->max_blocks_per_head)))
    return WGKV_EINVAL;
  if (workspace_bytes < wgkv_quest_workspace_size(pool)) return WGKV_ENOSPC;
  const size_t smem = size_t(pool->max_blocks_per_head) * 2 + 16;
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
  const int BH = pool->batch * pool->kv_heads;
  uint16_t* keys = static_cast<uint16_t*>(workspace);
  const int ks = pool->max_blocks_per_head;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 g1((pool->max_blocks_per_head + kQsPagesPerCta - 1) / kQsPagesPerCta, BH);
  const int G = q_heads / pool->kv_heads;
#define WGKV_QS(DD, GG) quest_score_kernel<DD, GG><<<g1, kQsThreads, 0, s>>>(qa, layer, cur_local_len, q, q_sb, token_budget, keys, ks)
#define WGKV_QS_D(GG) (pool->head_dim == 128 ? WGKV_QS(128, GG) : WGKV_QS(64, GG))
  switch (G) {
    case 1: WGKV_QS_D(1); break;
    case 2: WGKV_QS_D(2); break;
    case 3: WGKV_QS_D(3); break;
    case 4: WGKV_QS_D(4); break;
    case 5: WGKV_QS_D(5); break;
    case 6: WGKV_QS_D(6); break;
    case 7: WGKV_QS_D(7); break;
    case 8: WGKV_QS_D(8); break;
    case 9: WGKV_QS_D(9); break;
    case 10: WGKV_QS_D(10); break;
    case 11: WGKV_QS_D(11); break;
    case 12: WGKV_QS_D(12); break;
    case 13: WGKV_QS_D(13); break;
    case 14: WGKV_QS_D(14); break;
    case 15: WGKV_QS_D(15); break;
    case 16: WGKV_QS_D(16); break;
    default: return WGKV_EINVAL;
  }
#undef WGKV_QS_D
#undef WGKV_QS
  quest_select_kernel<<<BH, kQsThreads, smem, s>>>(qa, layer, cur_local_len, token_budget, keys, ks, out_seqlens,
                                                   out_table, out_stride);
  return cudaGetLastError() == cudaSuccess ? WGKV_OK : WGKV_ECUDA;
}
