// SnapKV key scoring on the 5th-gen tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// The two contraction passes of the eviction in snapkv.cu (reference snapkv_evict,
// src/modeling_layers.py:616-626: softmax of the window queries against a head's global keys, max
// over the query group, mean over the window), with the same numerics as the mma.sync kernels
// there: q . k accumulated in fp32 and rounded to bf16, times the scale rounded to bf16 again,
// then an fp32 softmax (expf, online max / sum in 128-key steps).
//
//   pass 1  row statistics.  One CTA per (head, 512 window rows, 32 K tiles): four M-tiles of 128
//           rows (Q resident in shared memory), K tiles of 128 keys streamed by TMA (one box per
//           page and 64 columns) through a 3-stage ring; S = Q K^T (M=128, N=128) into a TMEM slot
//           per M-tile; one warpgroup per M-tile, a thread per row (TMEM lane = row), keeps the
//           running max and sum of exp over the tile's two 64-key halves (the slot is refilled
//           while the second half is scored).  Pass 2 merges the key splits.
//   pass 2  key scores, transposed: the keys are the M dimension, so a thread owns a key and
//           sees all window rows of its TMEM lane, and the max over the group and the sum over
//           the window need no exchange between threads.  One CTA per (head, 16 consecutive
//           128-key tiles): S^T = K Q^T (M=128 keys, N=128 window rows per MMA, Q chunks streamed
//           by TMA through a 2-stage ring); the CTA's tiles go in groups of four, one per compute
//           warpgroup, each with its own 128-column TMEM slot, and the four tiles of a group share
//           every Q chunk (four warps per scheduler hide the epilogue's latencies).
//
// Warp 0 issues the TMA loads (no multicast), lane 0 of warp 1 the MMAs (warps 2-3 idle); every wait is bounded and
// a wait that runs out sets WGKV_ERR_TIMEOUT in the pool's error word (outputs are then undefined).
#include "common.cuh"
#include "runtime.h"
#include "tc.cuh"

namespace wgkv {
namespace {

constexpr int kTK = 128;       // keys per K tile
constexpr int kW1 = 4;                 // pass 1: M-tiles (compute warpgroups, TMEM slots) per CTA
constexpr int kW2 = 4;                 // pass 2: compute warpgroups, each with its own TMEM slot
constexpr int kNC2 = 512 / kW2;        // pass 2: window rows per MMA (N) = the slot's columns
constexpr int kMaxRows = 2048; // window rows per head (win x G) the pass-2 statistics table holds
constexpr int kTilesPerCta = 16;  // pass 2: consecutive K tiles per CTA
constexpr int kSplit = 32;     // pass 1: K tiles per CTA (a head's keys split over CTAs, merged in pass 2)

template <int D>
struct SnL {
  static constexpr int kDB = D / 64;          // 64-column boxes per row
  static constexpr int kBox = 128 * 128;      // one box of 128 rows x 128 B
  static constexpr int kKTile = kDB * kBox;   // 128 keys
  static constexpr int kQ1 = kDB * kBox;      // pass 1: one 128-row M-tile of Q
  static constexpr int kQ2 = kDB * (kNC2 / 128) * kBox;  // pass 2: one kNC2-row chunk of Q
  static constexpr int kK1 = 3;               // pass-1 K stages
  static constexpr int kSmem1 = kW1 * kQ1 + kK1 * kKTile + 256 + 1024;
  static constexpr int kSmem2 = kW2 * kKTile + 2 * kQ2 + kMaxRows * 8 + 256 + 1024;
};

constexpr int kThreads2 = 128 + 128 * kW2;  // pass 2
constexpr int kThreads1 = 128 + 128 * kW1;  // pass 1

struct SnTcArgs {
  int layer, B, Hk, G, win, R, T, window_pages, max_blocks, max_tok;
  const int32_t* block_table;
  const int32_t* lengths;
  float scale, inv_win;
  float2* rowml;   // [split][BH][R] (max, sum) of each pass-1 key split
  float* scores;   // [BH][max_tok]
  int* err;
};

WGKV_DEV uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
WGKV_DEV void f2_split(uint64_t v, float& lo, float& hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v)); }
WGKV_DEV uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// (x0, x1) <- bf16(bf16(x) * scale), the rounding of torch.matmul(bf16) * scaling on bf16 tensors
WGKV_DEV void round_scaled2(float& x0, float& x1, uint64_t sc2) {
  uint32_t p = pack_bf16x2(x0, x1);
  float y0, y1;
  f2_split(mul2(f2(__uint_as_float(p << 16), __uint_as_float(p & 0xFFFF0000u)), sc2), y0, y1);
  p = pack_bf16x2(y0, y1);
  x0 = __uint_as_float(p << 16);
  x1 = __uint_as_float(p & 0xFFFF0000u);
}

// e^d = 2^(d log2 e) on the SFU for d = s - m <= 0: the argument's rounding error grows with |d|,
// i.e. it is smallest for the terms that dominate the sums and maxima (relative error ~2^-22 there)
WGKV_DEV float exp_sfu(float d) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(d * 1.4426950408889634f));
  return y;
}
WGKV_DEV float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
WGKV_DEV uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// K tile `kt` of a head (pages of T rows, T | 128) into `dst`: lane i issues page i's boxes.
// Pages past the head's last one repeat it (their keys are masked or never stored).
template <int D>
WGKV_DEV void load_k_tile(int lane, uint8_t* dst, const CUtensorMap* tm, uint64_t* bar, const int32_t* grow, int nb,
                          int kt, int T) {
  const int ppt = kTK / T;
  for (int pi = lane; pi < ppt; pi += 32) {
    const int pg = min(kt * ppt + pi, nb - 1);
    const int id = __ldg(grow + pg);
#pragma unroll
    for (int d = 0; d < SnL<D>::kDB; ++d) tma_load_2d(dst + d * SnL<D>::kBox + pi * T * 128, tm, bar, d * 64, id * T);
  }
}

// ============================== pass 1: row statistics ==============================
struct Bars1 {
  uint64_t qfull;
  uint64_t kfull[SnL<128>::kK1], kempty[SnL<128>::kK1];
  uint64_t sfull[kW1], sfree[kW1];
  uint32_t tmem;
};

// running max / sum of e^(s - max) over 64 more scores of a row (masked ones are -inf)
WGKV_DEV void rowstats_update(float (&sv)[64], float& m, float& l) {
  float mx[8];
#pragma unroll
  for (int u8 = 0; u8 < 8; ++u8) mx[u8] = fmaxf(sv[u8], sv[u8 + 8]);
#pragma unroll
  for (int c = 16; c < 64; c += 16)
#pragma unroll
    for (int u8 = 0; u8 < 8; ++u8) mx[u8] = max3f(mx[u8], sv[c + u8], sv[c + 8 + u8]);
  const float x = max3f(max3f(mx[0], mx[1], mx[2]), max3f(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
  const float nm = fmaxf(m, x);
  if (nm == -INFINITY) return;  // nothing visible yet
  uint64_t e0 = f2(0.f, 0.f), e1 = f2(0.f, 0.f);
#pragma unroll
  for (int c = 0; c < 64; c += 4) {
    e0 = add2(e0, f2(exp_sfu(sv[c] - nm), exp_sfu(sv[c + 1] - nm)));
    e1 = add2(e1, f2(exp_sfu(sv[c + 2] - nm), exp_sfu(sv[c + 3] - nm)));
  }
  float ea, eb, ec, ed;
  f2_split(e0, ea, eb);
  f2_split(e1, ec, ed);
  l = l * expf(m - nm) + ((ea + eb) + (ec + ed));  // expf(-inf) = 0 on the first scores
  m = nm;
}

template <int D>
__global__ void __launch_bounds__(kThreads1, 1)
    snap_rowstats_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                            SnTcArgs a) {
  using L = SnL<D>;
  constexpr int kStg = L::kK1;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = sm + kW1 * L::kQ1;
  Bars1* bar = reinterpret_cast<Bars1*>(sK + kStg * L::kKTile);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.y, b = bh / a.Hk, h = bh - b * a.Hk;
  const int glen = a.lengths[int64_t(a.layer) * a.B * a.Hk + bh];
  if (glen <= 0) return;
  const int row0 = blockIdx.x * 128 * kW1;
  const int nt = min(kW1, (a.R - row0 + 127) / 128);  // M-tiles of this CTA
  const int j0 = blockIdx.z * kSplit;                 // first K tile of this CTA's key split
  if (j0 * kTK >= glen) return;
  const int n = min(kSplit, (glen + kTK - 1) / kTK - j0);  // K tiles of this CTA
  const int nb = (glen + a.T - 1) / a.T;
  const int32_t* grow = a.block_table + (int64_t(a.layer) * a.B * a.Hk + bh) * a.max_blocks + a.window_pages;

  if (tid == 0) {
    mbar_init(&bar->qfull, 1);
    for (int s = 0; s < kStg; ++s) {
      mbar_init(&bar->kfull[s], 1);
      mbar_init(&bar->kempty[s], 1);
    }
    for (int t = 0; t < kW1; ++t) {
      mbar_init(&bar->sfull[t], 1);
      mbar_init(&bar->sfree[t], 4);
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc<512>(&bar->tmem);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem;
  bool ok = true;
  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tensormap(&tmQ);
      prefetch_tensormap(&tmK);
      mbar_arrive_expect_tx(&bar->qfull, nt * L::kQ1);
      const int z0 = (a.layer * a.B + b) * a.win;
      for (int t = 0; t < nt; ++t)
        for (int d = 0; d < L::kDB; ++d)
          tma_load_3d(sm + t * L::kQ1 + d * L::kBox, &tmQ, &bar->qfull, d * 64, h * a.G, z0 + (row0 + t * 128) / a.G);
    }
    for (int j = 0; j < n; ++j) {
      const int s = j % kStg;
      if (!mbar_wait(&bar->kempty[s], ((j / kStg) & 1) ^ 1)) { ok = false; break; }
      if (lane == 0) mbar_arrive_expect_tx(&bar->kfull[s], L::kKTile);
      __syncwarp();
      load_k_tile<D>(lane, sK + s * L::kKTile, &tmK, &bar->kfull[s], grow, nb, j0 + j, a.T);
      __syncwarp();
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(128, kTK, 0, 0);
      if (!mbar_wait(&bar->qfull, 0)) ok = false;
      for (int j = 0; j < n && ok; ++j) {
        const int s = j % kStg;
        if (!mbar_wait(&bar->kfull[s], (j / kStg) & 1)) { ok = false; break; }
        const uint32_t ks = smem_u32(sK + s * L::kKTile);
        for (int t = 0; t < nt; ++t) {
          if (!mbar_wait(&bar->sfree[t], (j & 1) ^ 1)) { ok = false; break; }
          tc_fence_after();
          const uint32_t qt = smem_u32(sm + t * L::kQ1);
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint64_t da = umma_desc_sw128(qt + (k >> 2) * L::kBox + (k & 3) * 32, 16, 1024);
            const uint64_t db = umma_desc_sw128(ks + (k >> 2) * L::kBox + (k & 3) * 32, 16, 1024);
            umma_ss(tmem + t * 128, da, db, idesc, k > 0 ? 1u : 0u);
          }
          umma_commit(&bar->sfull[t]);
        }
        if (!ok) break;
        umma_commit(&bar->kempty[s]);
      }
    }
    __syncwarp();
  } else if (warp >= 4 && (warp - 4) / 4 < nt) {
    // ---------------- row statistics: a thread per window row ----------------
    const int t = (warp - 4) / 4, quad = warp & 3;
    const int r = row0 + t * 128 + quad * 32 + lane;
    const uint32_t trow = tmem + (uint32_t(quad * 32) << 16) + t * 128;
    const uint64_t sc2 = f2(a.scale, a.scale);
    float m = -INFINITY, l = 0.f;
    for (int j = 0; j < n; ++j) {
      if (!mbar_wait(&bar->sfull[t], j & 1)) { ok = false; break; }
      tc_fence_after();
      const int lim = glen - (j0 + j) * kTK;  // valid keys of this tile
      // the tile's two 64-key halves in turn; the slot is released once the second is loaded
      for (int hf = 0; hf < 2; ++hf) {
        float sv[64];
        tmem_ld32(trow + hf * 64, sv);
        tmem_ld32(trow + hf * 64 + 32, sv + 32);
        tmem_wait_ld();
        if (hf == 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bar->sfree[t]);
        }
#pragma unroll
        for (int c = 0; c < 64; c += 2) round_scaled2(sv[c], sv[c + 1], sc2);
        if (lim - hf * 64 < 64) {
#pragma unroll
          for (int c = 0; c < 64; ++c) sv[c] = c < lim - hf * 64 ? sv[c] : -INFINITY;
        }
        rowstats_update(sv, m, l);
      }
    }
    if (ok && r < a.R) a.rowml[(int64_t(blockIdx.z) * a.B * a.Hk + bh) * a.R + r] = make_float2(m, l);
  }
  if (!ok) set_error(a.err, WGKV_ERR_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<512>(tmem);
  }
}

// ============================== pass 2: key scores ==============================
struct Bars2 {
  uint64_t kfull[kW2], kempty[kW2], qfull[2], qempty[2];
  uint64_t sfull[kW2], sfree[kW2];
  uint32_t tmem;
};

template <int D, int G>
__global__ void __launch_bounds__(kThreads2, 1)
    snap_scores_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          SnTcArgs a) {
  using L = SnL<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = sm;
  uint8_t* sQ = sm + kW2 * L::kKTile;
  float2* st = reinterpret_cast<float2*>(sQ + 2 * L::kQ2);  // per window row: (max, 1 / sum)
  Bars2* bar = reinterpret_cast<Bars2*>(reinterpret_cast<uint8_t*>(st) + kMaxRows * 8);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.y, b = bh / a.Hk, h = bh - b * a.Hk;
  const int glen = a.lengths[int64_t(a.layer) * a.B * a.Hk + bh];
  const int ntile = (glen + kTK - 1) / kTK;
  const int kt0 = blockIdx.x * kTilesPerCta;  // this CTA's tiles: kt0 .. kt0 + ni - 1
  if (kt0 >= ntile) return;
  const int ni = min(kTilesPerCta, ntile - kt0);
  const int nc = (a.R + kNC2 - 1) / kNC2;                                             // Q chunks per tile
  const int nb = (glen + a.T - 1) / a.T;
  const int32_t* grow = a.block_table + (int64_t(a.layer) * a.B * a.Hk + bh) * a.max_blocks + a.window_pages;

  // row statistics: merge pass 1's key splits (max, then the sums rescaled to it)
  const int nsplit = (ntile + kSplit - 1) / kSplit;
  const int64_t sstride = int64_t(a.B) * a.Hk * a.R;
  for (int r = tid; r < a.R; r += kThreads2) {
    const float2* src = a.rowml + int64_t(bh) * a.R + r;
    float m = -INFINITY;
    for (int z = 0; z < nsplit; ++z) m = fmaxf(m, src[z * sstride].x);
    float l = 0.f;
    for (int z = 0; z < nsplit; ++z) {
      const float2 ml = src[z * sstride];
      l += ml.y * expf(ml.x - m);
    }
    st[r] = make_float2(m, 1.f / l);
  }
  if (tid == 0) {
    for (int s = 0; s < kW2; ++s) {
      mbar_init(&bar->kfull[s], 1);
      mbar_init(&bar->kempty[s], 1);
      mbar_init(&bar->sfull[s], 1);
      mbar_init(&bar->sfree[s], 4);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar->qfull[s], 1);
      mbar_init(&bar->qempty[s], 1);
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc<512>(&bar->tmem);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem;
  bool ok = true;
  if (warp == 0) {
    // ------- TMA producer: tiles in groups (one per warpgroup); the group's K, then Q chunks -------
    if (lane == 0) {
      prefetch_tensormap(&tmQ);
      prefetch_tensormap(&tmK);
    }
    const int z0 = (a.layer * a.B + b) * a.win;
    int q = 0;
    for (int pr = 0; kW2 * pr < ni && ok; ++pr) {
      for (int w = 0; w < kW2 && kW2 * pr + w < ni; ++w) {
        const int kt = kt0 + kW2 * pr + w;
        if (!mbar_wait(&bar->kempty[w], (pr & 1) ^ 1)) { ok = false; break; }
        if (lane == 0) mbar_arrive_expect_tx(&bar->kfull[w], L::kKTile);
        __syncwarp();
        load_k_tile<D>(lane, sK + w * L::kKTile, &tmK, &bar->kfull[w], grow, nb, kt, a.T);
        __syncwarp();
      }
      for (int c = 0; c < nc && ok; ++c, ++q) {
        const int qs = q & 1;
        if (!mbar_wait(&bar->qempty[qs], ((q >> 1) & 1) ^ 1)) { ok = false; break; }
        if (lane == 0) {
          mbar_arrive_expect_tx(&bar->qfull[qs], L::kQ2);
          for (int d = 0; d < L::kDB; ++d)
            tma_load_3d(sQ + qs * L::kQ2 + d * (kNC2 / 128) * L::kBox, &tmQ, &bar->qfull[qs], d * 64, h * a.G,
                        z0 + c * (kNC2 / a.G));
        }
        __syncwarp();
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: S^T = K Q^T per (tile, chunk), a group's tiles alternating ----------------
    if (lane == 0) {
      int q = 0;
      for (int pr = 0; kW2 * pr < ni && ok; ++pr) {
        const int nw = min(kW2, ni - kW2 * pr);  // tiles in this group
        for (int w = 0; w < nw; ++w)
          if (!mbar_wait(&bar->kfull[w], pr & 1)) { ok = false; break; }
        for (int c = 0; c < nc && ok; ++c, ++q) {
          const int qs = q & 1, uw = pr * nc + c;  // uw-th use of each warpgroup's slot
          if (!mbar_wait(&bar->qfull[qs], (q >> 1) & 1)) { ok = false; break; }
          const int N = min(kNC2, a.R - c * kNC2);
          const uint32_t idesc = umma_idesc_bf16(128, N, 0, 0);
          const uint32_t qa = smem_u32(sQ + qs * L::kQ2);
          for (int w = 0; w < nw; ++w) {
            if (!mbar_wait(&bar->sfree[w], (uw & 1) ^ 1)) { ok = false; break; }
            tc_fence_after();
            const uint32_t ks = smem_u32(sK + w * L::kKTile);
#pragma unroll
            for (int k = 0; k < D / 16; ++k) {
              const uint64_t da = umma_desc_sw128(ks + (k >> 2) * L::kBox + (k & 3) * 32, 16, 1024);
              const uint64_t db = umma_desc_sw128(qa + (k >> 2) * (kNC2 / 128) * L::kBox + (k & 3) * 32, 16, 1024);
              umma_ss(tmem + w * kNC2, da, db, idesc, k > 0 ? 1u : 0u);
            }
            umma_commit(&bar->sfull[w]);
          }
          if (!ok) break;
          umma_commit(&bar->qempty[qs]);
        }
        if (!ok) break;
        for (int w = 0; w < nw; ++w) umma_commit(&bar->kempty[w]);
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ---------------- scores: a thread per key, warpgroup w takes tile w of every group ----------------
    const int w = (warp - 4) / 4, quad = warp & 3;
    const uint32_t trow = tmem + (uint32_t(quad * 32) << 16) + w * kNC2;
    const uint64_t sc2 = f2(a.scale, a.scale);
    for (int i = w; i < ni && ok; i += kW2) {
      const int kt = kt0 + i;
      float acc = 0.f;
      for (int c = 0; c < nc; ++c) {
        const int uw = (i / kW2) * nc + c;
        if (!mbar_wait(&bar->sfull[w], uw & 1)) { ok = false; break; }
        tc_fence_after();
        const int ncols = min(kNC2, a.R - c * kNC2);
        // 32-column pieces, the next one's TMEM load in flight while this one is scored
        auto score_piece = [&](float (&v)[32], int p0) {
#pragma unroll
          for (int cc = 0; cc < 32; cc += 2) round_scaled2(v[cc], v[cc + 1], sc2);
          const int rb = c * kNC2 + p0;  // window row of v[0]
          // rows rb + g*G .. rb + g*G + G - 1 are the G query heads of one window position: max over
          // them, then the sum over window positions (rows past R, in a last partial piece, skipped)
          const int gl = min(32, a.R - rb);
#pragma unroll
          for (int g0 = 0; g0 < 32; g0 += G) {
            if (g0 < gl) {
              float gm = 0.f;
#pragma unroll
              for (int e = 0; e < G; ++e) {
                const float2 ml = st[rb + g0 + e];
                gm = fmaxf(gm, exp_sfu(v[g0 + e] - ml.x) * ml.y);
              }
              acc += gm;
            }
          }
        };
        float sa[32], sb[32];
        tmem_ld32(trow, sa);
        tmem_wait_ld();
        for (int p0 = 0; p0 < ncols; p0 += 64) {
          if (p0 + 32 < ncols) tmem_ld32(trow + p0 + 32, sb);
          score_piece(sa, p0);
          tmem_wait_ld();
          if (p0 + 32 >= ncols) break;
          if (p0 + 64 < ncols) tmem_ld32(trow + p0 + 64, sa);
          score_piece(sb, p0 + 32);
          tmem_wait_ld();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->sfree[w]);
      }
      const int key = kt * kTK + quad * 32 + lane;
      if (ok && key < glen) a.scores[int64_t(bh) * a.max_tok + key] = acc * a.inv_win;
    }
  }
  if (!ok) set_error(a.err, WGKV_ERR_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<512>(tmem);
  }
}

template <int D, int G>
int launch_passes(const CUtensorMap& q1, const CUtensorMap& q2, const CUtensorMap& km, const SnTcArgs& a, dim3 g1,
                  dim3 g2, cudaStream_t s) {
  using L = SnL<D>;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    if (cudaFuncSetAttribute(snap_rowstats_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmem1) !=
            cudaSuccess ||
        cudaFuncSetAttribute(snap_scores_tc_kernel<D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmem2) !=
            cudaSuccess)
      return WGKV_ECUDA;
    attr[dev] = true;
  }
  snap_rowstats_tc_kernel<D><<<g1, kThreads1, L::kSmem1, s>>>(q1, km, a);
  snap_scores_tc_kernel<D, G><<<g2, kThreads2, L::kSmem2, s>>>(q2, km, a);
  return cudaGetLastError() == cudaSuccess ? WGKV_OK : WGKV_ECUDA;
}

}  // namespace

// Per layer: the two score passes on the tensor cores.  Returns 1 when the shape does not fit
// them (the caller runs the mma.sync kernels), else a WGKV status.
int snapkv_scores_tc(const wgkv_pool& P, int layer, const uint16_t* queries, int win, int Hq, float scale,
                     float2* rowml, float* scores, cudaStream_t s) {
  const int Hk = P.kv_heads, G = Hq / Hk, D = P.head_dim, T = P.page, R = win * G;
  if (D != 64 && D != 128) return 1;
  if (16 % G || R % 16 || R > kMaxRows || T % 8 || kTK % T) return 1;
  if ((reinterpret_cast<uintptr_t>(queries) | reinterpret_cast<uintptr_t>(P.k)) & 15) return 1;
  if (uint64_t(P.total_blocks) * T >= (uint64_t(1) << 31) ||
      uint64_t(P.layers) * P.batch * win >= (uint64_t(1) << 31))
    return 1;
  static const bool off = [] {
    const char* e = getenv("WGKV_SNAPKV_MMA_SYNC");
    return e && e[0] == '1';
  }();
  if (off) return 1;
  // tensor maps are encoded per call (cheap host work next to the passes)
  CUtensorMap q1, q2, km;
  const uint64_t dims[3] = {uint64_t(D), uint64_t(Hq), uint64_t(P.layers) * P.batch * win};
  const uint64_t str[2] = {uint64_t(D), uint64_t(Hq) * D};
  const uint32_t box1[3] = {64, uint32_t(G), uint32_t(128 / G)}, box2[3] = {64, uint32_t(G), uint32_t(kNC2 / G)};
  if (!encode_3d_bf16(&q1, queries, dims, str, box1, true) || !encode_3d_bf16(&q2, queries, dims, str, box2, true) ||
      !encode_2d_bf16(&km, P.k, D, uint64_t(P.total_blocks) * T, D, 64, uint32_t(T), true))
    return WGKV_ECUDA;
  SnTcArgs a{};
  a.layer = layer;
  a.B = P.batch;
  a.Hk = Hk;
  a.G = G;
  a.win = win;
  a.R = R;
  a.T = T;
  a.window_pages = P.window / T;
  a.max_blocks = P.max_blocks_per_head;
  a.max_tok = P.max_tokens_per_head;
  a.block_table = P.block_table;
  a.lengths = P.global_lengths;
  a.scale = scale;
  a.inv_win = 1.f / float(win);
  a.rowml = rowml;
  a.scores = scores;
  a.err = P.err;
  const int BH = P.batch * Hk;
  // pass 1: key splits of kSplit tiles; pass 2: kTilesPerCta consecutive key tiles per CTA
  const int max_tiles = (P.max_tokens_per_head + kTK - 1) / kTK;
  const dim3 g1((R + 128 * kW1 - 1) / (128 * kW1), BH, (max_tiles + kSplit - 1) / kSplit), g2((max_tiles + kTilesPerCta - 1) / kTilesPerCta, BH);
  int st;
  switch (G) {
    case 1: st = D == 128 ? launch_passes<128, 1>(q1, q2, km, a, g1, g2, s) : launch_passes<64, 1>(q1, q2, km, a, g1, g2, s); break;
    case 2: st = D == 128 ? launch_passes<128, 2>(q1, q2, km, a, g1, g2, s) : launch_passes<64, 2>(q1, q2, km, a, g1, g2, s); break;
    case 4: st = D == 128 ? launch_passes<128, 4>(q1, q2, km, a, g1, g2, s) : launch_passes<64, 4>(q1, q2, km, a, g1, g2, s); break;
    case 8: st = D == 128 ? launch_passes<128, 8>(q1, q2, km, a, g1, g2, s) : launch_passes<64, 8>(q1, q2, km, a, g1, g2, s); break;
    case 16: st = D == 128 ? launch_passes<128, 16>(q1, q2, km, a, g1, g2, s) : launch_passes<64, 16>(q1, q2, km, a, g1, g2, s); break;
    default: return 1;
  }
  return st;
}

// Row-statistics entries pass 1 writes per (head, window row): one per key split of the longest head.
size_t snapkv_tc_rowml_splits(int max_tokens_per_head) {
  const int max_tiles = (max_tokens_per_head + kTK - 1) / kTK;
  return size_t(max(1, (max_tiles + kSplit - 1) / kSplit));
}

}  // namespace wgkv
