// SnapKV eviction over the paged pool (reference: snapkv_evict, src/modeling_layers.py:595-671),
// for every (layer, sequence, KV head) at once.
//
// Per head: the window of recorded queries (win x G rows, post-RoPE) attends to the head's global
// keys; each key's score is the max over the G query heads of its softmax probability, averaged
// over the window, then max-pooled (odd kernel, padding kernel / 2).  The int(glen * ratio) lowest
// pooled scores are evicted (ties: lower positions first -- torch.topk leaves their order open),
// the kept tokens are packed to the front of the head's pages and the emptied pages go to the
// pool's free list in (layer, b, h) order, where the next promotions take them from (:694-709).
//
// Numerics follow the reference's torch expressions: the q . k products accumulate in fp32 and are
// rounded to bf16, the scaled score is rounded to bf16 again, the softmax is fp32.
//
// Kernels (per layer): row statistics and key scores on the tensor cores (snapkv_tc.cu) where the
// shape fits them, else here on mma.sync m16n8k16 (row statistics: online max / sum over all
// keys, one CTA per 128 window rows; key scores: one CTA per 64-key chunk, all window rows);
// max-pooling (one grid), selection (one CTA per head: radix bottom-k, keep bits, new length).
// After all layers: the compaction of every (layer, head) in one launch, then the free-list slots
// (one CTA) and the freed pages (one CTA per head).
#include "common.cuh"

namespace wgkv {
namespace {

constexpr int kSnThreads = 256;
constexpr int kSnWarps = kSnThreads / 32;
constexpr int kKeys = 64;                 // keys per shared-memory chunk
constexpr int kRowsPerCta = 16 * kSnWarps;  // row statistics: one 16-row tile per warp

struct SnapArgs {
  wgkv_pool P;
  const uint16_t* qbuf;  // (layers, batch, win, Hq, D)
  int win, Hq, G, R;     // R = win * G rows per head
  float scale;
  int layer;
  float2* rowml;   // [BH][R] (max, sum)
  float* scores;   // [BH][max_tokens]
  int max_tok;
};

// Q fragment rows r0 = tile*16 + g, r1 = r0 + 8 of head bh; row r = w * G + g_idx.
WGKV_DEV const uint16_t* qrow(const SnapArgs& a, int b, int h, int r) {
  const int w = r / a.G, gi = r - w * a.G;
  return a.qbuf + ((int64_t(a.layer) * a.P.batch + b) * a.win + w) * int64_t(a.Hq) * a.P.head_dim +
         int64_t(h * a.G + gi) * a.P.head_dim;
}

template <int D>
WGKV_DEV void load_q_frag(const SnapArgs& a, int b, int h, int tile, uint32_t (&qa)[D / 16][4]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const int r0 = tile * 16 + g, r1 = r0 + 8;
  const uint32_t* q0 = reinterpret_cast<const uint32_t*>(qrow(a, b, h, r0));
  const uint32_t* q1 = reinterpret_cast<const uint32_t*>(qrow(a, b, h, r1));
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const int c = kk * 16 + 2 * t4;
    qa[kk][0] = __ldg(q0 + c / 2);
    qa[kk][1] = __ldg(q1 + c / 2);
    qa[kk][2] = __ldg(q0 + (c + 8) / 2);
    qa[kk][3] = __ldg(q1 + (c + 8) / 2);
  }
}

// keys [k0, k0 + kKeys) of head bh into shared memory (rows padded to D + 8), zeros past glen
template <int D>
WGKV_DEV void load_keys(const wgkv_pool& P, const int32_t* grow, int k0, int glen, uint16_t* ks) {
  constexpr int V = D / 8;  // 16-byte vectors per row
  const int T = P.page;
  for (int e = threadIdx.x; e < kKeys * V; e += kSnThreads) {
    const int r = e / V, c = e - r * V, p = k0 + r;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (p < glen) {
      const int64_t row = int64_t(grow[p / T]) * T + p % T;
      v = *reinterpret_cast<const uint4*>(P.k + row * D + c * 8);
    }
    *reinterpret_cast<uint4*>(ks + r * (D + 8) + c * 8) = v;
  }
}

// S tile (16 rows x 64 keys) of one warp, rounded as bf16(bf16(q . k) * scale)
template <int D>
WGKV_DEV void score_tile(const uint32_t (&qa)[D / 16][4], const uint16_t* ks, float scale, float (&s)[8][4]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
  // B fragments of two 8-key n-tiles per ldmatrix.x4: lanes 0-15 address the first tile's keys
  // (columns kk*16 and kk*16 + 8), lanes 16-31 the second's; rows are D + 8 elements apart
  const uint32_t base = smem_u32(ks) + uint32_t(((lane & 7) + ((lane >> 4) << 3)) * (D + 8) +
                                                ((lane >> 3) & 1) * 8) * 2;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
    for (int jp = 0; jp < 4; ++jp) {
      uint32_t b0, b1, b2, b3;
      ldmatrix_x4(b0, b1, b2, b3, base + uint32_t((jp * 16 * (D + 8) + kk * 16) * 2));
      mma_bf16_16816(s[2 * jp], qa[kk], b0, b1);
      mma_bf16_16816(s[2 * jp + 1], qa[kk], b2, b3);
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) s[j][e] = bf16_round(bf16_round(s[j][e]) * scale);
}

// ---- row statistics: max and sum of exp over all of the head's keys, online ----
template <int D>
__global__ void __launch_bounds__(kSnThreads) snap_rowstats_kernel(SnapArgs a) {
  extern __shared__ __align__(16) uint8_t sn_smem[];
  uint16_t* ks = reinterpret_cast<uint16_t*>(sn_smem);
  const wgkv_pool& P = a.P;
  const int Hk = P.kv_heads, BH = P.batch * Hk;
  const int bh = blockIdx.y, b = bh / Hk, h = bh - b * Hk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const int glen = P.global_lengths[int64_t(a.layer) * BH + bh];
  if (glen == 0) return;
  const int32_t* grow = P.block_table + (int64_t(a.layer) * BH + bh) * P.max_blocks_per_head + P.window / P.page;
  const int tile = blockIdx.x * kSnWarps + warp;
  const bool active = tile * 16 < a.R;
  uint32_t qa[D / 16][4];
  if (active) load_q_frag<D>(a, b, h, tile, qa);
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  for (int k0 = 0; k0 < glen; k0 += kKeys) {
    __syncthreads();
    load_keys<D>(P, grow, k0, glen, ks);
    __syncthreads();
    if (!active) continue;
    float s[8][4];
    score_tile<D>(qa, ks, a.scale, s);
    float x0 = -INFINITY, x1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = k0 + j * 8 + 2 * t4;
      if (c < glen) { x0 = fmaxf(x0, s[j][0]); x1 = fmaxf(x1, s[j][2]); }
      if (c + 1 < glen) { x0 = fmaxf(x0, s[j][1]); x1 = fmaxf(x1, s[j][3]); }
    }
    for (int o = 1; o < 4; o <<= 1) {
      x0 = fmaxf(x0, __shfl_xor_sync(0xffffffff, x0, o));
      x1 = fmaxf(x1, __shfl_xor_sync(0xffffffff, x1, o));
    }
    const float n0 = fmaxf(m0, x0), n1 = fmaxf(m1, x1);
    float e0 = 0.f, e1 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = k0 + j * 8 + 2 * t4;
      if (c < glen) { e0 += expf(s[j][0] - n0); e1 += expf(s[j][2] - n1); }
      if (c + 1 < glen) { e0 += expf(s[j][1] - n0); e1 += expf(s[j][3] - n1); }
    }
    for (int o = 1; o < 4; o <<= 1) {
      e0 += __shfl_xor_sync(0xffffffff, e0, o);
      e1 += __shfl_xor_sync(0xffffffff, e1, o);
    }
    l0 = l0 * expf(m0 - n0) + e0;  // expf(-inf) = 0 on the first chunk
    l1 = l1 * expf(m1 - n1) + e1;
    m0 = n0;
    m1 = n1;
  }
  if (active && t4 == 0) {
    const int r0 = tile * 16 + g;
    a.rowml[int64_t(bh) * a.R + r0] = make_float2(m0, l0);
    a.rowml[int64_t(bh) * a.R + r0 + 8] = make_float2(m1, l1);
  }
}

// ---- key scores: softmax probability, max over the group, mean over the window ----
template <int D>
__global__ void __launch_bounds__(kSnThreads) snap_scores_kernel(SnapArgs a) {
  extern __shared__ __align__(16) uint8_t sn_smem[];
  uint16_t* ks = reinterpret_cast<uint16_t*>(sn_smem);
  float* acc = reinterpret_cast<float*>(ks + kKeys * (D + 8));  // [kKeys]
  const wgkv_pool& P = a.P;
  const int Hk = P.kv_heads, BH = P.batch * Hk;
  const int bh = blockIdx.y, b = bh / Hk, h = bh - b * Hk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const int glen = P.global_lengths[int64_t(a.layer) * BH + bh];
  const int k0 = blockIdx.x * kKeys;
  if (k0 >= glen) return;
  const int32_t* grow = P.block_table + (int64_t(a.layer) * BH + bh) * P.max_blocks_per_head + P.window / P.page;
  for (int i = threadIdx.x; i < kKeys; i += kSnThreads) acc[i] = 0.f;
  load_keys<D>(P, grow, k0, glen, ks);
  __syncthreads();
  float col[8][2];
#pragma unroll
  for (int j = 0; j < 8; ++j) col[j][0] = col[j][1] = 0.f;
  const int G = a.G;
  for (int tile = warp; tile * 16 < a.R; tile += kSnWarps) {
    uint32_t qa[D / 16][4];
    load_q_frag<D>(a, b, h, tile, qa);
    float s[8][4];
    score_tile<D>(qa, ks, a.scale, s);
    const int r0 = tile * 16 + g, r1 = r0 + 8;
    const float2 ml0 = a.rowml[int64_t(bh) * a.R + r0], ml1 = a.rowml[int64_t(bh) * a.R + r1];
    const float inv0 = 1.f / ml0.y, inv1 = 1.f / ml1.y;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float p0 = expf(s[j][e] - ml0.x) * inv0;      // row r0
        float p1 = expf(s[j][2 + e] - ml1.x) * inv1;  // row r1
        // max over the G rows of a window position (rows w * G .. w * G + G - 1)
        for (int o = 4; o < 4 * G && o < 32; o <<= 1) {
          p0 = fmaxf(p0, __shfl_xor_sync(0xffffffff, p0, o));
          p1 = fmaxf(p1, __shfl_xor_sync(0xffffffff, p1, o));
        }
        if (G == 16) p0 = p1 = fmaxf(p0, p1);
        // one contribution per window position
        col[j][e] += (r0 % G == 0 ? p0 : 0.f) + (r1 % G == 0 ? p1 : 0.f);
      }
    }
  }
  // sum over the lanes of a key column, then over warps
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float v = col[j][e];
      for (int o = 4; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffff, v, o);
      if (g == 0) atomicAdd(&acc[j * 8 + 2 * t4 + e], v);
    }
  __syncthreads();
  const float inv_win = 1.f / float(a.win);
  for (int i = threadIdx.x; i < kKeys; i += kSnThreads)
    if (k0 + i < glen) a.scores[int64_t(bh) * a.max_tok + k0 + i] = acc[i] * inv_win;
}

// ---- per head: max-pool, bottom-k, compaction ----
WGKV_DEV uint32_t float_key(float f) {  // ascending float order -> ascending unsigned order
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}


struct SelectArgs {
  wgkv_pool P;
  int layer, ks;
  double ratio;
  const float* scores;  // [BH][max_tok]
  float* pooled;        // [BH][max_tok]
  int max_tok;
  int* nb;              // [layers][BH][2]: pages before / after
  int* olen;            // [layers][BH]: global length before the eviction
  uint32_t* keep;       // [layers][BH][kw]: keep bit per position
  int kw;               // keep words per head
};

// max-pooled scores of every head (odd kernel, padding kernel / 2) as ascending 32-bit keys,
// one thread per position
__global__ void __launch_bounds__(256) snap_pool_kernel(SelectArgs a) {
  const wgkv_pool& P = a.P;
  const int BH = P.batch * P.kv_heads, bh = blockIdx.y;
  const int glen = P.global_lengths[int64_t(a.layer) * BH + bh];
  const int p = blockIdx.x * 256 + threadIdx.x;
  if (p >= glen || int(double(glen) * a.ratio) == 0) return;
  const float* sc = a.scores + int64_t(bh) * a.max_tok;
  const int pad = a.ks / 2, lo = max(0, p - pad), hi = min(glen - 1, p + pad);
  float m = -INFINITY;
  for (int q = lo; q <= hi; ++q) m = fmaxf(m, sc[q]);
  reinterpret_cast<uint32_t*>(a.pooled)[int64_t(bh) * a.max_tok + p] = float_key(m);
}

constexpr int kSelThreads = 1024;
constexpr int kSelWarps = kSelThreads / 32;

// Per head: the n_ev-th smallest pooled key by four 8-bit radix passes (several keys in flight per
// thread), then a keep bit per position (keys below it and the first `need` equal to it -- the
// lowest positions -- are evicted) and the new length; the rows move later, for all layers at once.
__global__ void __launch_bounds__(kSelThreads) snap_select_kernel(SelectArgs a) {
  const wgkv_pool& P = a.P;
  const int Hk = P.kv_heads, BH = P.batch * Hk, T = P.page;
  const int bh = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ int hist[256];
  __shared__ int wsum[kSelWarps];
  __shared__ int s_bin, s_take;
  const int64_t hi = int64_t(a.layer) * BH + bh;
  int* gl = P.global_lengths + hi;
  const int glen = *gl;
  const int nb_old = (glen + T - 1) / T;
  const int n_ev = int(double(glen) * a.ratio);
  int* nb = a.nb + hi * 2;
  if (tid == 0) a.olen[hi] = glen;
  if (n_ev == 0) {
    if (tid == 0) { nb[0] = nb_old; nb[1] = nb_old; }
    return;
  }
  const uint32_t* pk = reinterpret_cast<const uint32_t*>(a.pooled) + int64_t(bh) * a.max_tok;
  // n_ev-th smallest key, four 8-bit passes from the top byte
  int need = n_ev;
  uint32_t prefix = 0;
  constexpr int kU = 4;  // keys in flight per thread
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = tid; i < 256; i += kSelThreads) hist[i] = 0;
    __syncthreads();
    for (int b0 = 0; b0 < glen; b0 += kU * kSelThreads) {
      uint32_t kk[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int p = b0 + u * kSelThreads + tid;
        kk[u] = p < glen ? __ldg(pk + p) : 0u;
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int p = b0 + u * kSelThreads + tid;
        if (p < glen && (pass == 0 || (kk[u] >> (shift + 8)) == prefix)) atomicAdd(&hist[(kk[u] >> shift) & 0xFF], 1);
      }
    }
    __syncthreads();
    if (tid < 32) warp_pick_bin<false>(hist, need, &s_bin, &s_take);
    __syncthreads();
    prefix = (prefix << 8) | uint32_t(s_bin);
    need = s_take;
    __syncthreads();
  }
  const uint32_t kth = prefix;  // evict keys < kth and the first `need` equal to it
  uint32_t* kb = a.keep + hi * a.kw;
  int eq_seen = 0, kept = 0;
  for (int c0 = 0; c0 < glen; c0 += kSelThreads) {
    const int p = c0 + tid;
    const uint32_t k = p < glen ? __ldg(pk + p) : 0u;
    const int is_eq = p < glen && k == kth;
    int tot_eq;
    const int eq_rank = eq_seen + block_excl_scan<kSelThreads>(is_eq, wsum, tot_eq);
    const bool keep = p < glen && !(k < kth || (is_eq && eq_rank < need));
    const unsigned w = __ballot_sync(0xffffffff, keep);
    if (lane == 0) kb[(c0 >> 5) + warp] = w;
    kept += __syncthreads_count(keep);
    eq_seen += tot_eq;
  }
  if (tid == 0) {
    *gl = kept;
    nb[0] = nb_old;
    nb[1] = (kept + T - 1) / T;
  }
}

// Every (layer, head) of the eviction at once: the in-place front compaction of the kept tokens in
// 1024-position chunks, each moved in four rounds of 256 rows (four threads per row, the row's K
// and V parts held in registers between the round's reads and its writes).  A round reads all its
// rows before any is written, and a kept token only moves to a lower position, so no row is
// overwritten before it is read.
template <int D>
__global__ void __launch_bounds__(kSelThreads) snap_compact_kernel(SelectArgs a) {
  const wgkv_pool& P = a.P;
  const int BH = P.batch * P.kv_heads, T = P.page;
  const int64_t hi = blockIdx.x;  // layer * BH + bh
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ int wsum[kSelWarps];
  __shared__ int dsts[kSelThreads];
  const int olen = a.olen[hi], nlen = P.global_lengths[hi];
  if (nlen == olen) return;
  const int32_t* grow = P.block_table + hi * P.max_blocks_per_head + P.window / T;
  const uint32_t* kb = a.keep + hi * a.kw;
  constexpr int V = D / 8;   // 16-byte vectors per row
  constexpr int VP = V / 4;  // per thread (four threads per row)
  int kept_base = 0;
  for (int c0 = 0; c0 < olen; c0 += kSelThreads) {
    const int p = c0 + tid;
    const uint32_t w = p - lane < olen ? __ldg(kb + (c0 >> 5) + warp) : 0u;
    const bool keep = p < olen && ((w >> lane) & 1u);
    if (lane == 0) wsum[warp] = __popc(w);
    __syncthreads();
    int before = 0, tot = 0;
    for (int i = 0; i < kSelWarps; ++i) {
      before += i < warp ? wsum[i] : 0;
      tot += wsum[i];
    }
    const int dst = kept_base + before + __popc(w & ((1u << lane) - 1u));
    dsts[tid] = keep && dst != p ? dst : -1;
    __syncthreads();
    for (int r0 = 0; r0 < kSelThreads && c0 + r0 < olen; r0 += 256) {
      const int rl = r0 + (tid >> 2), part = tid & 3;
      const int src = c0 + rl, d = dsts[rl];
      uint4 kv[2 * VP];
      if (d >= 0) {
        const int64_t row = int64_t(__ldg(grow + src / T)) * T + src % T;
        const uint4* kr = reinterpret_cast<const uint4*>(P.k + row * D) + part * VP;
        const uint4* vr = reinterpret_cast<const uint4*>(P.v + row * D) + part * VP;
#pragma unroll
        for (int c = 0; c < VP; ++c) {
          kv[c] = kr[c];
          kv[VP + c] = vr[c];
        }
      }
      __syncthreads();
      if (d >= 0) {
        const int64_t row = int64_t(__ldg(grow + d / T)) * T + d % T;
        uint4* kw = reinterpret_cast<uint4*>(P.k + row * D) + part * VP;
        uint4* vw = reinterpret_cast<uint4*>(P.v + row * D) + part * VP;
#pragma unroll
        for (int c = 0; c < VP; ++c) {
          kw[c] = kv[c];
          vw[c] = kv[VP + c];
        }
      }
      __syncthreads();
    }
    kept_base += tot;
  }
}

// ---- freed pages -> the free list, (layer, b, h) order; their table entries -> sentinel ----
constexpr int kFreeThreads = 1024;

// (one CTA: each head's first free-list slot, the list's new length)
__global__ void __launch_bounds__(kFreeThreads) snap_free_kernel(wgkv_pool P, const int* nb, int* offs) {
  const int N = P.layers * P.batch * P.kv_heads;
  const int per = (N + kFreeThreads - 1) / kFreeThreads;
  const int i0 = min(N, int(threadIdx.x) * per), i1 = min(N, i0 + per);
  int cnt = 0;
  for (int i = i0; i < i1; ++i) cnt += nb[2 * i] - nb[2 * i + 1];
  __shared__ int wsum[kFreeThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = cnt;
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffff, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[warp] = x;
  __syncthreads();
  int base = 0, tot = 0;
  for (int w = 0; w < kFreeThreads / 32; ++w) {
    if (w < warp) base += wsum[w];
    tot += wsum[w];
  }
  const int fc = *P.free_count;
  int off = fc + base + x - cnt;
  for (int i = i0; i < i1; ++i) {
    offs[i] = off;
    off += nb[2 * i] - nb[2 * i + 1];
  }
  __syncthreads();
  if (threadIdx.x == 0) *P.free_count = fc + tot;
}

// one CTA per head: its freed pages to the list from its slot on, their table entries -> sentinel
__global__ void __launch_bounds__(128) snap_free_write_kernel(wgkv_pool P, const int* nb, const int* offs) {
  const int i = blockIdx.x;
  const int j0 = nb[2 * i + 1], j1 = nb[2 * i], off = offs[i];
  int32_t* row = P.block_table + int64_t(i) * P.max_blocks_per_head + P.window / P.page;
  const int sentinel = int(P.total_blocks - 1);
  for (int j = j0 + threadIdx.x; j < j1; j += 128) {
    P.free_ids[off + j - j0] = row[j];
    row[j] = sentinel;
  }
}

size_t round256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace
}  // namespace wgkv

namespace wgkv {
int snapkv_scores_tc(const wgkv_pool& P, int layer, const uint16_t* queries, int win, int Hq, float scale,
                     float2* rowml, float* scores, cudaStream_t s);  // snapkv_tc.cu
size_t snapkv_tc_rowml_splits(int max_tokens_per_head);                  // snapkv_tc.cu
}

using namespace wgkv;

extern "C" size_t wgkv_snapkv_workspace_size(const wgkv_pool* pool, int window, int q_heads) {
  if (!pool || pool->kv_heads <= 0) return 0;
  const size_t BH = size_t(pool->batch) * pool->kv_heads;
  const size_t R = size_t(window) * (q_heads / pool->kv_heads);
  return round256(BH * R * 8 * snapkv_tc_rowml_splits(pool->max_tokens_per_head)) + 2 * round256(BH * size_t(pool->max_tokens_per_head) * 4) +
         round256(size_t(pool->layers) * BH * 8) + 2 * round256(size_t(pool->layers) * BH * 4) +
         round256(size_t(pool->layers) * BH * ((size_t(pool->max_tokens_per_head) + 31) / 32 + kSelWarps) * 4);
}

extern "C" int wgkv_snapkv_evict(const wgkv_pool* pool, const uint16_t* queries, int window, int q_heads,
                                 float softmax_scale, double evict_ratio, int kernel_size, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  if (!pool || !pool->free_ids || !pool->free_count || !queries || !workspace || window <= 0 || q_heads <= 0 ||
      q_heads % pool->kv_heads || kernel_size <= 0 || kernel_size % 2 == 0 || !(evict_ratio > 0.0) ||
      evict_ratio > 1.0)
    return WGKV_EINVAL;
  const int G = q_heads / pool->kv_heads, D = pool->head_dim;
  if (16 % G || (window * G) % 16 || (D != 64 && D != 128)) return WGKV_EINVAL;
  if (workspace_bytes < wgkv_snapkv_workspace_size(pool, window, q_heads)) return WGKV_ENOSPC;
  const int BH = pool->batch * pool->kv_heads;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t R = size_t(window) * G;
  SnapArgs a{};
  a.P = *pool;
  a.qbuf = queries;
  a.win = window;
  a.Hq = q_heads;
  a.G = G;
  a.R = int(R);
  a.scale = softmax_scale;
  a.rowml = reinterpret_cast<float2*>(ws);
  a.max_tok = pool->max_tokens_per_head;
  a.scores = reinterpret_cast<float*>(ws + round256(size_t(BH) * R * 8 * snapkv_tc_rowml_splits(a.max_tok)));
  SelectArgs sa{};
  sa.P = *pool;
  sa.ks = kernel_size;
  sa.ratio = evict_ratio;
  sa.scores = a.scores;
  sa.pooled = a.scores + round256(size_t(BH) * a.max_tok * 4) / 4;
  sa.max_tok = a.max_tok;
  sa.nb = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(sa.pooled) + round256(size_t(BH) * a.max_tok * 4));
  sa.olen = sa.nb + (round256(size_t(pool->layers) * BH * 8) + round256(size_t(pool->layers) * BH * 4)) / 4;
  sa.kw = (a.max_tok + 31) / 32 + kSelWarps;  // + slack: a chunk's words past the head's end
  sa.keep = reinterpret_cast<uint32_t*>(sa.olen + round256(size_t(pool->layers) * BH * 4) / 4);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t smem_keys = size_t(kKeys) * (D + 8) * 2;
  const size_t smem_scores = smem_keys + kKeys * 4;
  const int max_chunks = (pool->max_tokens_per_head + kKeys - 1) / kKeys;
  for (int l = 0; l < pool->layers; ++l) {
    a.layer = l;
    sa.layer = l;
    const dim3 g1((a.R + kRowsPerCta - 1) / kRowsPerCta, BH), g2(max_chunks, BH);
    // the two score passes on the tensor cores where the shape fits them, else on mma.sync
    const int tc = snapkv_scores_tc(*pool, l, queries, window, q_heads, softmax_scale, a.rowml, a.scores, s);
    if (tc != 1 && tc != WGKV_OK) return tc;
    if (D == 128) {
      if (tc == 1) {
        snap_rowstats_kernel<128><<<g1, kSnThreads, smem_keys, s>>>(a);
        snap_scores_kernel<128><<<g2, kSnThreads, smem_scores, s>>>(a);
      }
      snap_pool_kernel<<<dim3(max_chunks * kKeys / 256 + 1, BH), 256, 0, s>>>(sa);
      snap_select_kernel<<<BH, kSelThreads, 0, s>>>(sa);
    } else {
      if (tc == 1) {
        snap_rowstats_kernel<64><<<g1, kSnThreads, smem_keys, s>>>(a);
        snap_scores_kernel<64><<<g2, kSnThreads, smem_scores, s>>>(a);
      }
      snap_pool_kernel<<<dim3(max_chunks * kKeys / 256 + 1, BH), 256, 0, s>>>(sa);
      snap_select_kernel<<<BH, kSelThreads, 0, s>>>(sa);
    }
  }
  // the rows of every layer move in one launch (one CTA per (layer, head)), then the freed pages
  if (D == 128)
    snap_compact_kernel<128><<<pool->layers * BH, kSelThreads, 0, s>>>(sa);
  else
    snap_compact_kernel<64><<<pool->layers * BH, kSelThreads, 0, s>>>(sa);
  int* offs = sa.nb + round256(size_t(pool->layers) * BH * 8) / 4;
  snap_free_kernel<<<1, kFreeThreads, 0, s>>>(*pool, sa.nb, offs);
  snap_free_write_kernel<<<pool->layers * BH, 128, 0, s>>>(*pool, sa.nb, offs);
  return cudaGetLastError() == cudaSuccess ? WGKV_OK : WGKV_ECUDA;
}
