// Block-sparse (vertical-slash) causal prefill attention on the 5th-gen
// tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// Same contract as the mma.sync kernel in sparse_prefill.cu (the attention
// sparse_attn_func computes for generate_sparse_indices' indices, pinned by
// utils/test_sparse_attn.py:34-93).  One CTA owns one 64-query row block of
// one KV head and 2*NM query heads of its GQA group, i.e. NM M-tiles of 128
// rows (two heads x 64 queries each) that share every K/V tile.  K/V tiles
// hold 128 keys (two 64-key halves), so both MMAs run at N >= 128, where a
// 128-row tcgen05 MMA reaches full rate (at N = 64 it does not):
//
//   warp 0      TMA producer: Q once; per tile, K and V into 2-stage rings.
//               Admitted-column halves are gathered with tile::gather4 (four
//               key rows per instruction, from column_index) or, in pooled
//               mode, loaded as contiguous rows of the compacted pool; band
//               halves are plain 2D tiles.  SWIZZLE_128B, no multicast.
//   warp 1      TMEM allocator + single-thread MMA issuer, per M-tile t:
//               S_t = Q_t K^T (M=128, N=128, K=D, A/B in shared memory), then,
//               once the softmax has written P_t into the S columns,
//               O_t += P_t V (M=128, N=D, K=128, A = P from TMEM).  The two
//               M-tiles alternate, so one tile's softmax overlaps the other's MMAs.
//   warps 2..   two warpgroups per M-tile, one per 64-key half: each thread owns
//               one row of its half (TMEM lane = row); masks (column tail /
//               causal band), swaps the tile's row max with its partner half,
//               online softmax in base 2 with a lazy running max (O rescaled in
//               TMEM only when the max grows by more than 2^8), writes P as
//               packed bf16 into TMEM, and finally normalises its half of O.
#include "common.cuh"
#include "runtime.h"
#include "tc.cuh"

namespace wgkv {
namespace {

constexpr int kKeys = 128;  // keys per K/V tile (two 64-key halves)
constexpr int kStg = 2;     // K and V stages
constexpr float kRescaleThreshold = 8.f;  // log2 of the largest tolerated growth of unnormalised terms

template <int D, int NM, int HV>
struct Tc {
  static constexpr int kDB = D / 64;                 // 64-column boxes per row
  static constexpr int kQTile = kDB * 16384;         // one M-tile of Q: kDB boxes x 128 rows x 128 B
  static constexpr int kBox = kKeys * 128;           // one 64-column box of a K/V tile (128 rows x 128 B)
  static constexpr int kKV = kDB * kBox;             // one K or V stage
  static constexpr int kOffK = NM * kQTile;
  static constexpr int kOffV = kOffK + kStg * kKV;
  static constexpr int kOffBar = kOffV + kStg * kKV;
  static constexpr int kOffX = kOffBar + 512;        // row-max / row-sum exchange [3][NM][2][128] floats
  static constexpr int kSmem = kOffX + 3 * NM * 2 * 128 * 4 + 1024;  // + alignment slack
  // warpgroup 0: producer, MMA issuer, two idle warps; then per M-tile HV softmax warpgroups, the
  // threads of a row splitting its 128 keys HV ways
  static constexpr int kThreads = 128 + 128 * NM * HV;
  static constexpr int kSoftWarps = 4 * HV;          // softmax warps per M-tile
  static constexpr int kTmemCols = NM == 2 ? 512 : 256;
  // register split (setmaxnreg) between warpgroup 0 and the softmax warpgroups, within the launch's
  // threads x registers: 384 threads launch at 168 (128 x 64 + 256 x 216), 640 at 96 (128 x 64 + 512 x 104)
  static constexpr int kRegLo = 64;
  static constexpr int kRegHi = kThreads == 640 ? 104 : 216;
  static constexpr bool kRegSplit = kThreads > 256;
};

// 2^x on the SFU (ex2.approx, flush-to-zero): the softmax terms are rounded to
// bf16 before PV, so its ~2-ulp fp32 error is far below what the result keeps.
WGKV_DEV float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Paired fp32 arithmetic (sm_100 f32x2 instructions): two lanes of a 64-bit register pair per
// instruction, same rounding as the scalar forms.
WGKV_DEV uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
WGKV_DEV void f2_split(uint64_t v, float& lo, float& hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v)); }
WGKV_DEV uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
WGKV_DEV uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
WGKV_DEV float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x on the FMA pipe for a pair of lanes, to take part of the softmax exponentials off the SFU
// (which would otherwise bound the softmax): x = n + r with n = round(x) (the 1.5 * 2^23 shifter),
// r in [-1/2, 1/2]; 2^r from a cubic fitted here to 2^r on [-1/2, 1/2] by least squares in relative
// error at Chebyshev nodes (max relative error 7.7e-5, far below the bf16 rounding P gets); 2^n
// added to the exponent field.  Inputs below -120 (masked keys are -inf) give 2^-120, zero for
// every practical purpose next to a row sum >= 1.
WGKV_DEV uint64_t exp2_fma2(uint64_t x) {
  float a, b;
  f2_split(x, a, b);
  x = f2(fmaxf(a, -120.f), fmaxf(b, -120.f));
  const uint64_t t = add2(x, f2(12582912.f, 12582912.f));
  const uint64_t r = fma2(add2(t, f2(-12582912.f, -12582912.f)), f2(-1.f, -1.f), x);
  uint64_t q = fma2(f2(0.05508868f, 0.05508868f), r, f2(0.24260405f, 0.24260405f));
  q = fma2(q, r, f2(0.69327624f, 0.69327624f));
  q = fma2(q, r, f2(0.99992894f, 0.99992894f));
  float ta, tb, qa, qb;
  f2_split(t, ta, tb);
  f2_split(q, qa, qb);
  // the shifter's low mantissa bits hold n; shifted by 23 they are n in the exponent field
  return f2(__int_as_float(__float_as_int(ta) * (1 << 23) + __float_as_int(qa)),
            __int_as_float(__float_as_int(tb) * (1 << 23) + __float_as_int(qb)));
}

#ifndef WGKV_EMU_PERIOD
#define WGKV_EMU_PERIOD 4  // of every WGKV_EMU_PERIOD pairs of P, WGKV_EMU_COUNT use exp2_fma2
#endif
#ifndef WGKV_EMU_COUNT
#define WGKV_EMU_COUNT 1
#endif

// p = 2^x for one pair of scores, and its packed bf16 pair for P: by pair index on the FMA pipe
// (exp2_fma2) or as two fp32 SFU ops.  (The packed bf16 SFU form, ex2.approx.ftz.bf16x2, for one,
// two or all four pairs in four measured 3-5 % slower on the C3 shape.)
WGKV_DEV void exp2_pair(int pi, uint64_t x2, float x0, float x1, float& p0, float& p1, uint32_t& packed) {
  if ((pi % WGKV_EMU_PERIOD) < WGKV_EMU_COUNT) {
    f2_split(exp2_fma2(x2), p0, p1);
  } else {
    p0 = fast_exp2(x0);
    p1 = fast_exp2(x1);
  }
  packed = pack_bf16x2(p0, p1);
}

struct TcParams {
  int B, L, Hk, G, R, n_hg;
  const int32_t *bc, *bo, *cc, *ci;
  int64_t bo_stride, ci_stride;
  float scale_log2;
  uint16_t* out;
  int64_t o_sb, o_sl, o_sh;
  int* err;
  // pooled mode: admitted columns of (b, h) are pool rows table[(b*Hk+h)*t_stride + t_first] * t_page + c
  const int32_t* table;
  int64_t t_stride;
  int t_first, t_page;
};

#ifdef WGKV_EXPERIMENT_TRACE  // timing experiment only: clock64 stamps of one CTA's pipeline events
__device__ long long g_trace[16][256];
#define WGKV_TRACE(row, j)                                                                     \
  if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && (j) >= 0 && (j) < 256) g_trace[row][j] = clock64();
#else
#define WGKV_TRACE(row, j)
#endif

struct Bars {
  uint64_t qfull;
  uint64_t kfull[kStg], kempty[kStg];
  uint64_t vfull[kStg], vempty[kStg];
  uint64_t sfull[2], pfull[2], odone[2];
  uint32_t tmem;
};

template <int D, int NM, bool POOL, int HV>
__global__ void __launch_bounds__(Tc<D, NM, HV>::kThreads, 1)
    sparse_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                             const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmKg,
                             const __grid_constant__ CUtensorMap tmVg, const __grid_constant__ CUtensorMap tmKp,
                             const __grid_constant__ CUtensorMap tmVp, TcParams p) {
  using C = Tc<D, NM, HV>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bar = reinterpret_cast<Bars*>(sm + C::kOffBar);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const int i = p.R - 1 - blockIdx.x;  // heaviest row blocks first
  const int hg = blockIdx.y % p.n_hg;
  const int h = blockIdx.y / p.n_hg;
  const int b = blockIdx.z;
  const int s0 = i * 64;
  const int hq0 = h * p.G + hg * 2 * NM;  // first query head of this CTA
  const int ncol = p.cc[(int64_t(b) * p.Hk + h) * p.R + i];
  const int nband = p.bc[i];               // 64-key band blocks
  const int ntc = (ncol + kKeys - 1) / kKeys;
  const int ntb = (nband + 1) / 2;         // band tiles: block pairs (2m, 2m+1)
  const int n = ntc + ntb;
  const int32_t* bo_row = p.bo + int64_t(i) * p.bo_stride;

  if (tid == 0) {
    mbar_init(&bar->qfull, 1);
    for (int s = 0; s < kStg; ++s) {
      mbar_init(&bar->kfull[s], 1);
      mbar_init(&bar->kempty[s], 1);
      mbar_init(&bar->vfull[s], 1);
      mbar_init(&bar->vempty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bar->sfull[t], 1);
      mbar_init(&bar->pfull[t], C::kSoftWarps);
      mbar_init(&bar->odone[t], 1);
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc<C::kTmemCols>(&bar->tmem);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem;
  bool ok = true;
  if (warp < 4) {
  if constexpr (C::kRegSplit) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(C::kRegLo));
  if (warp == 0) {
    // ================================ producer ================================
    if (lane == 0) {
      prefetch_tensormap(&tmQ);
      prefetch_tensormap(&tmK);
      prefetch_tensormap(&tmV);
      prefetch_tensormap(&tmKg);
      prefetch_tensormap(&tmVg);
      if (POOL) {
        prefetch_tensormap(&tmKp);
        prefetch_tensormap(&tmVp);
      }
      mbar_arrive_expect_tx(&bar->qfull, NM * 2 * C::kDB * 8192);
      for (int t = 0; t < NM; ++t)
        for (int hh = 0; hh < 2; ++hh)
          for (int d = 0; d < C::kDB; ++d)
            tma_load_2d(sm + t * C::kQTile + d * 16384 + hh * 8192, &tmQ, &bar->qfull,
                        (hq0 + 2 * t + hh) * D + d * 64, b * p.L + s0);
    }
    const int32_t* cib = p.ci + (int64_t(b) * p.Hk + h) * p.ci_stride;
    const int pool_row0 =
        POOL && ncol > 0 ? __ldg(p.table + (int64_t(b) * p.Hk + h) * p.t_stride + p.t_first) * p.t_page : 0;
    // gathered column tiles: lane -> 4-row group `grp` of the 128 rows, both 64-column boxes
    // (D = 128: lanes 0-31 cover rows 0..127 of box 0 and then box 1)
    auto fetch = [&](int j, int* r4) {
      const bool gath = j < ntc && (!POOL || ncol - j * kKeys < kKeys);
      if (gath) {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          int e = j * kKeys + lane * 4 + r;
          e = e < ncol ? e : ncol - 1;  // past the tail: any valid row (masked in the softmax)
          r4[r] = __ldg(cib + e);
        }
      }
    };
    int pre0[4] = {0, 0, 0, 0}, pre1[4] = {0, 0, 0, 0};
    fetch(0, pre0);
    fetch(1, pre1);
    for (int j = 0; j < n && ok; ++j) {
      const bool col = j < ntc;
      const bool pooled = POOL && col && ncol - j * kKeys >= kKeys;
      int rows4[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        rows4[r] = b * p.L + pre0[r];
        pre0[r] = pre1[r];
      }
      fetch(j + 2, pre1);
      int off0 = 0, off1 = -1;  // row coordinates of the two 64-key halves
      if (pooled) {
        off0 = pool_row0 + j * kKeys;
        off1 = off0 + 64;
      } else if (!col) {
        const int m = j - ntc;
        off0 = b * p.L + __ldg(bo_row + 2 * m);
        off1 = 2 * m + 1 < nband ? b * p.L + __ldg(bo_row + 2 * m + 1) : off0;  // a missing half is masked
      }
      const int s = j % kStg;
      const uint32_t ph = (j / kStg) & 1;
      for (int kv = 0; kv < 2; ++kv) {
        uint64_t* full = kv ? &bar->vfull[s] : &bar->kfull[s];
        uint64_t* empty = kv ? &bar->vempty[s] : &bar->kempty[s];
        if (!mbar_wait(empty, ph ^ 1)) { set_error(p.err, WGKV_ERR_TIMEOUT); ok = false; break; }
        uint8_t* st = sm + (kv ? C::kOffV : C::kOffK) + s * C::kKV;
        if (lane == 0) mbar_arrive_expect_tx(full, C::kKV);
        if (lane == 0 && kv == 0) { WGKV_TRACE(0, j) }
        __syncwarp();
        if (col && !pooled) {
#pragma unroll
          for (int d = 0; d < C::kDB; ++d)
            tma_gather4(st + d * C::kBox + lane * 512, kv ? &tmVg : &tmKg, full, h * D + d * 64, rows4[0], rows4[1],
                        rows4[2], rows4[3]);
        } else if (lane == 0) {
          const CUtensorMap* m = pooled ? (kv ? &tmVp : &tmKp) : (kv ? &tmV : &tmK);
          const int x0 = pooled ? 0 : h * D;
          for (int d = 0; d < C::kDB; ++d) {
            tma_load_2d(st + d * C::kBox, m, full, x0 + d * 64, off0);
            tma_load_2d(st + d * C::kBox + 8192, m, full, x0 + d * 64, off1);
          }
        }
        __syncwarp();
      }
    }
  } else if (warp == 1) {
    // ============================ MMA issuer (1 thread) ============================
    if (lane == 0) {
      const uint32_t id_qk = umma_idesc_bf16(128, kKeys, 0, 0);
      const uint32_t id_pv = umma_idesc_bf16(128, D, 0, 1);
      if (!mbar_wait(&bar->qfull, 0)) { set_error(p.err, WGKV_ERR_TIMEOUT); ok = false; }
      for (int j = 0; j <= n && ok; ++j) {
        const int s = j % kStg, ps = (j - 1) % kStg;
        if (j < n && !mbar_wait(&bar->kfull[s], (j / kStg) & 1)) {
          set_error(p.err, WGKV_ERR_TIMEOUT);
          ok = false;
          break;
        }
        WGKV_TRACE(1, j)
        if (j > 0 && !mbar_wait(&bar->vfull[ps], ((j - 1) / kStg) & 1)) {
          set_error(p.err, WGKV_ERR_TIMEOUT);
          ok = false;
          break;
        }
        const uint32_t kst = smem_u32(sm + C::kOffK + s * C::kKV);
        const uint32_t vst = smem_u32(sm + C::kOffV + ps * C::kKV);
        for (int t = 0; t < NM; ++t) {
          const uint32_t tS = tmem + t * 256, tO = tS + 128;
          if (j > 0) {
            // O_t += P_t(j-1) V(j-1): P sits as packed bf16 pairs in S_t's first 64 columns
            if (!mbar_wait(&bar->pfull[t], (j - 1) & 1)) { set_error(p.err, WGKV_ERR_TIMEOUT); ok = false; break; }
            WGKV_TRACE(2 + t, j - 1)
            tc_fence_after();
#ifndef WGKV_EXPERIMENT_NO_PV  // timing experiment only: skips O += P V (wrong results)
#pragma unroll
            for (int k = 0; k < kKeys / 16; ++k) {
              const uint64_t bb = umma_desc_sw128(vst + k * 2048, C::kBox, 1024);
              umma_ts(tO, tS + k * 8, bb, id_pv, (j > 1 || k > 0) ? 1u : 0u);
            }
#endif
            umma_commit(&bar->odone[t]);
          }
          if (j < n) {
            // S_t = Q_t K(j)^T; issued after PV_t(j-1), which read P from these columns
            const uint32_t qt = smem_u32(sm + t * C::kQTile);
#pragma unroll
            for (int k = 0; k < D / 16; ++k) {
              const uint64_t a = umma_desc_sw128(qt + (k >> 2) * 16384 + (k & 3) * 32, 16, 1024);
              const uint64_t bb = umma_desc_sw128(kst + (k >> 2) * C::kBox + (k & 3) * 32, 16, 1024);
              umma_ss(tS, a, bb, id_qk, k > 0 ? 1u : 0u);
            }
            umma_commit(&bar->sfull[t]);
          }
        }
        if (!ok) break;
        if (j > 0) umma_commit(&bar->vempty[ps]);
        if (j < n) umma_commit(&bar->kempty[s]);
      }
    }
    __syncwarp();
  }  // warps 2, 3: idle until the final barrier
  } else {
    // ====================== softmax: HV threads per 128-key row ======================
    if constexpr (C::kRegSplit) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(C::kRegHi));
    constexpr int KPT = kKeys / HV;           // keys of a row this thread owns
    constexpr int kOC = D / HV;               // O columns this thread owns
    const int sw = warp - 4;
    const int t = sw / (4 * HV);
    const int hf = (sw >> 2) % HV;            // which KPT-key slice of every tile
    const int quad = warp & 3;                // TMEM lanes 32*quad.. are the ones this warp may access
    const int row = quad * 32 + lane;         // TMEM lane = row of M-tile t
    const int hh = 2 * t + (row >> 6);
    const int q = s0 + (row & 63);
    const int bar_id = 1 + t * 4 + quad;      // named barrier of the HV warps sharing these rows
    const uint32_t trow = tmem + (uint32_t(quad * 32) << 16) + t * 256;
    float* xm = reinterpret_cast<float*>(sm + C::kOffX);  // [slot][t][hf][row]
    auto xslot = [&](int slot, int h_) { return xm + ((slot * NM + t) * 2 + h_) * 128 + row; };
    const float sc = p.scale_log2;
    const int qlim = min(q, p.L - 1);
    float m_used = -INFINITY, l = 0.f;
#ifdef WGKV_PREFILL_PINGPONG
    if constexpr (NM == 2 && HV == 1) {
      if (t == 1 && n > 0) asm volatile("bar.arrive 9, 256;" ::: "memory");  // M-tile 0 goes first
    }
#endif
    for (int j = 0; j < n; ++j) {
      if (ok && !mbar_wait(&bar->sfull[t], j & 1)) { set_error(p.err, WGKV_ERR_TIMEOUT); ok = false; }
      if (quad == 0 && lane == 0 && hf == 0) { WGKV_TRACE(4 + t, j) }
      tc_fence_after();
      float sv[KPT];
#pragma unroll
      for (int c = 0; c < KPT; c += 32) tmem_ld32(trow + hf * KPT + c, sv + c);
      // limits of this thread's 64-key blocks (column tail / causal band / missing band block)
      int lim[KPT / 64];
#pragma unroll
      for (int u = 0; u < KPT / 64; ++u) {
        const int kb = hf * (KPT / 64) + u;   // 64-key block of the tile
        if (j < ntc) {
          lim[u] = ncol - j * kKeys - kb * 64 - 1;
        } else {
          const int blk = 2 * (j - ntc) + kb;
          lim[u] = blk < nband ? qlim - __ldg(bo_row + blk) : -1;
        }
      }
      tmem_wait_ld();
      if (quad == 0 && lane == 0 && t == 0 && hf == 0) { WGKV_TRACE(8, j) }
#pragma unroll
      for (int u = 0; u < KPT / 64; ++u) {
        if (lim[u] < 63) {
#pragma unroll
          for (int c = 0; c < 64; ++c) sv[u * 64 + c] = c <= lim[u] ? sv[u * 64 + c] : -INFINITY;
        }
      }
      // row max: three-input max over independent chains
      constexpr int kCh = KPT / 16;           // 8 chains (128 keys) or 4 (64 keys)
      float mx[kCh];
#pragma unroll
      for (int u = 0; u < kCh; ++u) mx[u] = fmaxf(sv[2 * u], sv[2 * u + 1]);
#pragma unroll
      for (int c = 2 * kCh; c < KPT; c += 2 * kCh) {
#pragma unroll
        for (int u = 0; u < kCh; ++u) mx[u] = max3(mx[u], sv[c + 2 * u], sv[c + 2 * u + 1]);
      }
      float mraw = mx[0];
#pragma unroll
      for (int u = 1; u < kCh; ++u) mraw = fmaxf(mraw, mx[u]);
      if constexpr (HV == 2) {
        *xslot(j & 1, hf) = mraw;
        asm volatile("bar.sync %0, 64;" ::"r"(bar_id) : "memory");  // both slices have their tile max
        mraw = fmaxf(mraw, *xslot(j & 1, hf ^ 1));
      }
      if (quad == 0 && lane == 0 && t == 0 && hf == 0) { WGKV_TRACE(11, j) }
      const float mt = mraw * sc;
      float alpha = 1.f;
      bool need = false;
      if (mt > m_used + kRescaleThreshold) {  // also true on the first visible key (m_used = -inf)
        need = true;
        alpha = exp2f(m_used - mt);  // 0 when m_used = -inf
        m_used = mt;
      }
      if (j > 0 && __any_sync(0xffffffff, need && alpha != 1.f)) {
        // O is rescaled only when the running max grew: then wait for PV(j-1) to have landed in O.
        // (Skipping the wait otherwise is safe: PV_t(j) is issued only after this iteration's P, so
        // odone[t] is never more than one phase ahead of the parity waited on here or at the end.)
        if (ok && !mbar_wait(&bar->odone[t], (j - 1) & 1)) { set_error(p.err, WGKV_ERR_TIMEOUT); ok = false; }
        tc_fence_after();
#pragma unroll 1
        for (int c0 = 0; c0 < kOC; c0 += 32) {
          float ov[32];
          tmem_ld32(trow + 128 + hf * kOC + c0, ov);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) ov[c] *= alpha;
          tmem_st32(trow + 128 + hf * kOC + c0, ov);
        }
      }
#ifdef WGKV_PREFILL_PINGPONG
      // the two M-tiles' exponential loops take turns (named barriers 9 / 10, 256 threads each), so
      // one tile's exponentials run while the other tile's MMAs do
      if constexpr (NM == 2 && HV == 1) asm volatile("bar.sync %0, 256;" ::"r"(9 + t) : "memory");
#endif
      const float nbase = m_used == -INFINITY ? 0.f : -m_used;
      // p = 2^(s * scale - m): the scale-and-shift as paired FMAs, the exponential on the SFU (part
      // on the FMA pipe), the row sum as paired adds; each 32-key chunk of P goes to TMEM (packed
      // bf16 pairs over the first S columns) as soon as it is computed
      const uint64_t sc2 = f2(sc, sc), nb2 = f2(nbase, nbase);
      uint64_t sa = f2(0.f, 0.f), sb = f2(0.f, 0.f);
#pragma unroll
      for (int cc = 0; cc < KPT; cc += 32) {
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 32; c += 4) {
          float x0, x1, x2, x3, p0, p1, p2, p3;
          const uint64_t xa = fma2(f2(sv[cc + c], sv[cc + c + 1]), sc2, nb2);
          const uint64_t xb = fma2(f2(sv[cc + c + 2], sv[cc + c + 3]), sc2, nb2);
          f2_split(xa, x0, x1);
          f2_split(xb, x2, x3);
          const int pi = (cc + c) >> 1;  // index of the pair (x0, x1); (x2, x3) is pi + 1
          exp2_pair(pi, xa, x0, x1, p0, p1, pk[c >> 1]);
          exp2_pair(pi + 1, xb, x2, x3, p2, p3, pk[(c >> 1) + 1]);
          sa = add2(sa, f2(p0, p1));
          sb = add2(sb, f2(p2, p3));
        }
        tmem_st16(trow + ((hf * KPT + cc) >> 1), pk);
      }
      float s0_, s1_, s2_, s3_;
      f2_split(sa, s0_, s1_);
      f2_split(sb, s2_, s3_);
      l = l * alpha + ((s0_ + s1_) + (s2_ + s3_));
#ifdef WGKV_PREFILL_PINGPONG
      if constexpr (NM == 2 && HV == 1) {
        if (t == 0 || j + 1 < n) asm volatile("bar.arrive %0, 256;" ::"r"(10 - t) : "memory");
      }
#endif
      if (quad == 0 && lane == 0 && t == 0 && hf == 0) { WGKV_TRACE(12, j) }
      // the P stores and any O rescale must land before the MMA reads them
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->pfull[t]);
      if (quad == 0 && lane == 0 && hf == 0) { WGKV_TRACE(6 + t, j) }
    }
    // ---- epilogue: O / l -> bf16 ----
    if (ok && n > 0) {
      if (!mbar_wait(&bar->odone[t], (n - 1) & 1)) { set_error(p.err, WGKV_ERR_TIMEOUT); ok = false; }
    }
    tc_fence_after();
    if constexpr (HV == 2) {
      *xslot(2, hf) = l;
      asm volatile("bar.sync %0, 64;" ::"r"(bar_id) : "memory");
      l += *xslot(2, hf ^ 1);
    }
    const bool any = l > 0.f;  // a row that saw no key (degenerate index sets only) writes zeros
    const float inv = any ? 1.f / l : 0.f;
    uint16_t* orow = p.out + b * p.o_sb + int64_t(q) * p.o_sl + int64_t(hq0 + hh) * p.o_sh + hf * kOC;
#pragma unroll 1
    for (int c0 = 0; c0 < kOC; c0 += 32) {
      float ov[32];
      tmem_ld32(trow + 128 + hf * kOC + c0, ov);
      tmem_wait_ld();
      if (ok && q < p.L) {
        if (!any) {
#pragma unroll
          for (int c = 0; c < 32; ++c) ov[c] = 0.f;
        }
#pragma unroll
        for (int c = 0; c < 32; c += 8) {
          uint4 v;
          v.x = pack_bf16x2(ov[c] * inv, ov[c + 1] * inv);
          v.y = pack_bf16x2(ov[c + 2] * inv, ov[c + 3] * inv);
          v.z = pack_bf16x2(ov[c + 4] * inv, ov[c + 5] * inv);
          v.w = pack_bf16x2(ov[c + 6] * inv, ov[c + 7] * inv);
          *reinterpret_cast<uint4*>(orow + c0 + c) = v;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<C::kTmemCols>(tmem);
  }
}

template <int D, int NM, bool POOL, int HV>
int launch_tc(const uint16_t* q, const uint16_t* k, const uint16_t* v, int64_t q_sl, int64_t k_sl, int64_t v_sl,
              int Hq, int Hk, const uint16_t* pool_k, const uint16_t* pool_v, int64_t pool_rows, const TcParams& p,
              cudaStream_t stream) {
  using C = Tc<D, NM, HV>;
  CUtensorMap mq, mk, mv, mkg, mvg;
  const uint64_t rows = uint64_t(p.B) * p.L;
  if (!encode_2d_bf16(&mq, q, uint64_t(Hq) * D, rows, q_sl, 64, 64, true)) return WGKV_ECUDA;
  if (!encode_2d_bf16(&mk, k, uint64_t(Hk) * D, rows, k_sl, 64, 64, true)) return WGKV_ECUDA;
  if (!encode_2d_bf16(&mv, v, uint64_t(Hk) * D, rows, v_sl, 64, 64, true)) return WGKV_ECUDA;
  if (!encode_2d_bf16(&mkg, k, uint64_t(Hk) * D, rows, k_sl, 64, 1, true)) return WGKV_ECUDA;
  if (!encode_2d_bf16(&mvg, v, uint64_t(Hk) * D, rows, v_sl, 64, 1, true)) return WGKV_ECUDA;
  CUtensorMap mkp = mkg, mvp = mvg;  // pool maps (only read in pooled mode)
  if (POOL) {
    if (!encode_2d_bf16(&mkp, pool_k, D, uint64_t(pool_rows), D, 64, 64, true)) return WGKV_ECUDA;
    if (!encode_2d_bf16(&mvp, pool_v, D, uint64_t(pool_rows), D, 64, 64, true)) return WGKV_ECUDA;
  }
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    if (cudaFuncSetAttribute(sparse_prefill_tc_kernel<D, NM, POOL, HV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::kSmem) != cudaSuccess)
      return WGKV_ECUDA;
    attr[dev] = true;
  }
  dim3 grid(p.R, p.Hk * p.n_hg, p.B);
  sparse_prefill_tc_kernel<D, NM, POOL, HV><<<grid, C::kThreads, C::kSmem, stream>>>(mq, mk, mv, mkg, mvg, mkp, mvp, p);
  return cudaGetLastError() == cudaSuccess ? WGKV_OK : WGKV_ECUDA;
}

}  // namespace

// Used by wgkv_sparse_prefill when the problem fits the tensor-core kernel
// (even GQA group, D in {64, 128}, each tensor a 2D [B*L, H*D] view with 16-byte rows).
// Returns 1 when it does not apply (the caller falls back), else a WGKV status.
int sparse_prefill_tc(const uint16_t* q, int64_t q_sb, int64_t q_sl, int64_t q_sh, const uint16_t* k, int64_t k_sb,
                      int64_t k_sl, int64_t k_sh, const uint16_t* v, int64_t v_sb, int64_t v_sl, int64_t v_sh, int B,
                      int L, int Hq, int Hk, int D, const int32_t* bc, const int32_t* bo, int64_t bo_stride,
                      const int32_t* cc, const int32_t* ci, int64_t ci_stride, float scale, uint16_t* out,
                      int64_t o_sb, int64_t o_sl, int64_t o_sh, int* err, cudaStream_t stream,
                      const uint16_t* pool_k, const uint16_t* pool_v, int64_t pool_rows, const int32_t* table,
                      int64_t t_stride, int t_first, int t_page) {
  const int G = Hq / Hk;
  if (G % 2 != 0 || (D != 64 && D != 128)) return 1;
  if (q_sh != D || k_sh != D || v_sh != D) return 1;
  if ((B > 1) && (q_sb != int64_t(L) * q_sl || k_sb != int64_t(L) * k_sl || v_sb != int64_t(L) * v_sl)) return 1;
  if (((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
        reinterpret_cast<uintptr_t>(out)) & 15) ||
      ((q_sl | k_sl | v_sl) % 8) || ((o_sb | o_sl | o_sh) % 8))
    return 1;
  if (int64_t(B) * L >= (int64_t(1) << 31)) return 1;
  TcParams p;
  p.B = B; p.L = L; p.Hk = Hk; p.G = G; p.R = (L + 63) / 64;
  p.bc = bc; p.bo = bo; p.cc = cc; p.ci = ci; p.bo_stride = bo_stride; p.ci_stride = ci_stride;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = out; p.o_sb = o_sb; p.o_sl = o_sl; p.o_sh = o_sh;
  p.err = err;
  p.table = table; p.t_stride = t_stride; p.t_first = t_first; p.t_page = t_page;
  const bool pool = pool_k != nullptr;
  if (pool && (!pool_v || !table || ((reinterpret_cast<uintptr_t>(pool_k) | reinterpret_cast<uintptr_t>(pool_v)) & 15)))
    return WGKV_EINVAL;
  // threads per 128-key row of the softmax: 1 (default; 8-10 % faster than 2 at the C3 shape) or
  // 2 (WGKV_PREFILL_SPLIT=2)
  static const int hv = [] {
    const char* e = getenv("WGKV_PREFILL_SPLIT");
    return (e && e[0] == '2') ? 2 : 1;
  }();
#define WGKV_TC_LAUNCH2(DD, NMM, HVV)                                                                            \
  (pool ? launch_tc<DD, NMM, true, HVV>(q, k, v, q_sl, k_sl, v_sl, Hq, Hk, pool_k, pool_v, pool_rows, p, stream) \
        : launch_tc<DD, NMM, false, HVV>(q, k, v, q_sl, k_sl, v_sl, Hq, Hk, pool_k, pool_v, pool_rows, p, stream))
#define WGKV_TC_LAUNCH(DD, NMM) (hv == 1 ? WGKV_TC_LAUNCH2(DD, NMM, 1) : WGKV_TC_LAUNCH2(DD, NMM, 2))
  if (G % 4 == 0) {
    p.n_hg = G / 4;
    return D == 128 ? WGKV_TC_LAUNCH(128, 2) : WGKV_TC_LAUNCH(64, 2);
  }
  p.n_hg = G / 2;
  return D == 128 ? WGKV_TC_LAUNCH(128, 1) : WGKV_TC_LAUNCH(64, 1);
#undef WGKV_TC_LAUNCH
#undef WGKV_TC_LAUNCH2
}

}  // namespace wgkv

#ifdef WGKV_EXPERIMENT_TRACE
extern "C" __attribute__((visibility("default"))) int wgkv_experiment_trace_copy(void* host) {
  return cudaMemcpyFromSymbol(host, wgkv::g_trace, sizeof(wgkv::g_trace)) == cudaSuccess ? 0 : -1;
}
#endif
