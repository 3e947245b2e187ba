// Ragged paged decode attention (GQA), sm_100a.
//
// Replaces the reference's split/reduce Triton pair
// (src/modeling_layers.py:834-1000) and its host-built chunk schedule
// (:1032-1055).  Design:
//
// * Work unit = 16 consecutive tokens of one (batch, kv-head) -- one 16-row
//   slice of a page.  The units of all heads are laid end to end (prefix sum
//   computed on the device by every CTA, no host sync) and the grid, a
//   multiple of the SM count, cuts that line into equal segments, so ragged
//   heads are balanced exactly ("stream-K" split).
// * Per CTA: one producer warp issues TMA tile loads (SWIZZLE_128B, no
//   multicast) of K and V units into a STAGES-deep shared-memory ring guarded
//   by mbarriers; NCW consumer warps each take one unit per stage.  Page ids
//   for the next 32 units are fetched by the producer lanes ahead of use.
// * Consumers compute S = Q K^T and O += P V with mma.sync m16n8k16 (bf16 in,
//   fp32 accumulate); the G query heads of a KV head share every K/V byte
//   read (rows >= G of the 16-row tile are zero).  Online softmax in fp32
//   with P rounded to bf16 before PV, as the reference kernel does (:930).
// * A head covered by several CTAs is merged by the last CTA to finish it
//   (per-head atomic counter, self-resetting); no spin waits.
#include <mutex>

#include "common.cuh"
#include "runtime.h"

namespace wgkv {
namespace {

constexpr int kNCW = 8;  // consumer warps (the kernel is consumer-bound below 8)
constexpr int kThreads = 32 * (kNCW + 1);
constexpr int kMaxBH = 4096;          // max batch * kv_heads handled in shared memory
constexpr int kCtasPerSM = 1;

struct DecodeParams {
  const uint16_t* q;
  uint16_t* out;
  const int32_t* seqlens;
  const int32_t* table;
  int64_t table_stride;
  int64_t num_pages;
  int page_size;
  int upp;  // units per page = page_size / 16
  int BH;
  int G;
  float scale_log2;
  float* part;
  int* counters;
  int* err;
};

// D: head dim; S: pipeline stages (3 for D=128 when shared memory allows, else fewer)
template <int D, int S>
struct Cfg {
  static constexpr int kUnitBytes = 16 * D * 2;         // one K (or V) unit
  static constexpr int kStageBytes = kNCW * 2 * kUnitBytes;
  static constexpr int kStages = S;
  static constexpr int kBoxes = D / 64;                 // 64-column TMA boxes per unit
};

template <int D, int S>
size_t smem_bytes(int BH, int G) {
  size_t s = 1024;  // alignment slack
  s += size_t(Cfg<D, S>::kStages) * Cfg<D, S>::kStageBytes;
  s += size_t(BH + 1 + kThreads) * 4;                   // prefix + scan scratch
  s += size_t(kNCW) * G * (D + 2) * 4;                  // cross-warp merge
  s += 2 * Cfg<D, S>::kStages * 8 + 64;                 // barriers + flags
  return s;
}

template <int D, int S>
__global__ void __launch_bounds__(kThreads, 1)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                        DecodeParams p) {
  using C = Cfg<D, S>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stage_base = smem;
  int* pre = reinterpret_cast<int*>(smem + C::kStages * C::kStageBytes);
  int* scan = pre + p.BH + 1;  // kThreads ints
  float* merge = reinterpret_cast<float*>(scan + kThreads);
  const int G = p.G;
  uint64_t* full = reinterpret_cast<uint64_t*>(merge + kNCW * G * (D + 2) + 1);
  full = reinterpret_cast<uint64_t*>((reinterpret_cast<uintptr_t>(full) + 7) & ~uintptr_t(7));
  uint64_t* empty = full + C::kStages;
  int* flag = reinterpret_cast<int*>(empty + C::kStages);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int BH = p.BH;

  // Inputs (lengths, tables, queries, ring rows) may be written by the kernel launched just before
  // this one (programmatic dependent launch lets this grid start early): wait for it before reading.
  if (tid == 0) {
    for (int st = 0; st < C::kStages; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], kNCW);
    }
    fence_barrier_init();
  }
  if (tid == 32) {
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  griddep_launch();  // the next kernel (e.g. the output projection) may start fetching its weights

  // ---- prefix sum of 16-token units per (b, h) ---------------------------
  {
    const int per = (BH + kThreads - 1) / kThreads;
    const int i0 = min(BH, tid * per), i1 = min(BH, i0 + per);
    int sum = 0;
    for (int i = i0; i < i1; ++i) sum += (max(p.seqlens[i], 0) + 15) >> 4;
    int total;
    int run = block_excl_scan<kThreads>(sum, scan, total);  // this thread's first unit
    if (tid == 0) pre[BH] = total;
    for (int i = i0; i < i1; ++i) {
      pre[i] = run;
      run += (max(p.seqlens[i], 0) + 15) >> 4;
    }
    __syncthreads();
  }

  // heads with no tokens: zero output (strided over CTAs)
  for (int bh = blockIdx.x; bh < BH; bh += gridDim.x) {
    if (pre[bh + 1] == pre[bh]) {
      for (int e = tid; e < G * D; e += kThreads) p.out[size_t(bh) * G * D + e] = 0;
    }
  }

  const int U = pre[BH];
  const int seg = (U + gridDim.x - 1) / gridDim.x;
  const int u0 = blockIdx.x * seg;
  const int u1 = min(U, u0 + seg);
  if (seg == 0 || u0 >= u1) return;

  // first head overlapping u0: last bh with pre[bh] <= u0
  int lo = 0, hi = BH;  // invariant: pre[lo] <= u0 < pre[hi]
  while (hi - lo > 1) {
    int mid = (lo + hi) >> 1;
    if (pre[mid] <= u0) lo = mid; else hi = mid;
  }
  const int bh0 = lo;

  if (warp == 0) {
    // ============================ producer ============================
    if (lane == 0) {
      prefetch_tensormap(&tmK);
      prefetch_tensormap(&tmV);
    }
    int it = 0;
    bool ok = true;
    for (int bh = bh0, rs = u0; ok && rs < u1; ++bh) {
      const int hs = pre[bh], he = pre[bh + 1];
      if (he <= rs) continue;
      const int re = min(u1, he);
      const int32_t* trow = p.table + int64_t(bh) * p.table_stride;
      // units [rs, re) of head bh, local unit index = u - hs
      for (int b0 = rs; ok && b0 < re; b0 += 32) {
        const int u = b0 + lane;
        int pid = 0;
        if (u < re) {
          const int ul = u - hs;
          pid = __ldg(trow + ul / p.upp);
          if (pid < 0 || pid >= p.num_pages) {
            set_error(p.err, WGKV_ERR_BAD_PAGE);
            pid = 0;
          }
          pid = pid * p.upp + ul % p.upp;  // 16-row slice index
        }
        const int nb = min(32, re - b0);
        for (int k0 = 0; k0 < nb; k0 += kNCW, ++it) {
          const int s = it % C::kStages;
          const uint32_t ph = (it / C::kStages) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1)) {
            set_error(p.err, WGKV_ERR_TIMEOUT);
            ok = false;
            break;
          }
          const int nv = min(kNCW, nb - k0);
          if (lane == 0) mbar_arrive_expect_tx(&full[s], nv * 2 * C::kUnitBytes);
          __syncwarp();
          if (lane >= k0 && lane < k0 + nv) {
            uint8_t* kb = stage_base + s * C::kStageBytes + (lane - k0) * 2 * C::kUnitBytes;
            uint8_t* vb = kb + C::kUnitBytes;
#pragma unroll
            for (int x = 0; x < C::kBoxes; ++x) {
              tma_load_2d(kb + x * 2048, &tmK, &full[s], x * 64, pid * 16);
              tma_load_2d(vb + x * 2048, &tmV, &full[s], x * 64, pid * 16);
            }
          }
          __syncwarp();
        }
      }
      rs = re;
    }
    // Leave only once every load this warp issued has landed: if a consumer gave up waiting
    // (WGKV_ERR_TIMEOUT) the CTA may otherwise retire with bulk copies still writing its shared
    // memory.  On the normal path these phases completed long ago and each wait returns at once.
    if (lane == 0) {
      for (int j = max(0, it - C::kStages); j < it; ++j) {
        if (!mbar_wait(&full[j % C::kStages], (j / C::kStages) & 1)) set_error(p.err, WGKV_ERR_TIMEOUT);
      }
    }
    return;
  }

  // ============================== consumers ==============================
  const int cw = warp - 1;
  const int g = lane >> 2;   // row within the 16-row tile (query head in group)
  const int t4 = lane & 3;
  const int ctid = tid - 32;  // 0 .. 32*kNCW-1
  int it = 0;
  bool ok = true;

  for (int bh = bh0, rs = u0; rs < u1; ++bh) {
    const int hs = pre[bh], he = pre[bh + 1];
    if (he <= rs) continue;
    const int re = min(u1, he);
    const int seqlen = p.seqlens[bh];

    // Q fragments (rows >= G are zero)
    uint32_t qa[D / 16][4];
    {
      const uint32_t* q32 = reinterpret_cast<const uint32_t*>(p.q + size_t(bh) * G * D);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int c0 = kk * 16 + 2 * t4;
        qa[kk][0] = g < G ? __ldg(q32 + (g * D + c0) / 2) : 0u;
        qa[kk][1] = g + 8 < G ? __ldg(q32 + ((g + 8) * D + c0) / 2) : 0u;
        qa[kk][2] = g < G ? __ldg(q32 + (g * D + c0 + 8) / 2) : 0u;
        qa[kk][3] = g + 8 < G ? __ldg(q32 + ((g + 8) * D + c0 + 8) / 2) : 0u;
      }
    }
    float acc[D / 8][4];
#pragma unroll
    for (int j = 0; j < D / 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    for (int b0 = rs; b0 < re; b0 += 32) {
      const int nb = min(32, re - b0);
      for (int k0 = 0; k0 < nb; k0 += kNCW, ++it) {
        const int s = it % C::kStages;
        const uint32_t ph = (it / C::kStages) & 1;
        if (ok && !mbar_wait(&full[s], ph)) {
          set_error(p.err, WGKV_ERR_TIMEOUT);
          ok = false;
        }
        const int uidx = k0 + cw;
        if (ok && uidx < nb) {
          const int ul = b0 + uidx - hs;  // unit index within the head
          const int nvalid = min(16, seqlen - ul * 16);
          uint8_t* kb = stage_base + s * C::kStageBytes + cw * 2 * C::kUnitBytes;
          uint8_t* vb = kb + C::kUnitBytes;
          if (nvalid < 16) {
            // rows past the head's length hold whatever the page holds: zero V there
            for (int e = lane; e < (16 - nvalid) * (D / 8); e += 32) {
              const int r = nvalid + e / (D / 8);
              const int c = e % (D / 8);
              *reinterpret_cast<uint4*>(vb + (c / 8) * 2048 + r * 128 + (c % 8) * 16) = make_uint4(0, 0, 0, 0);
            }
            __syncwarp();
          }
          // ---- S = Q K^T (16 x 16 tokens) ----
          float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
          const uint32_t kbase = smem_u32(kb);
          const int mi = lane >> 3, ri = lane & 7;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const int box = kk >> 2;
            const int chunk = (kk & 3) * 2 + (mi & 1);
            const int tok = (mi >> 1) * 8 + ri;
            uint32_t r0, r1, r2, r3;
            ldmatrix_x4(r0, r1, r2, r3, kbase + box * 2048 + swz128(tok, chunk));
            mma_bf16_16816(s0, qa[kk], r0, r1);
            mma_bf16_16816(s1, qa[kk], r2, r3);
          }
          // ---- online softmax (base 2) ----
          const int j0 = 2 * t4, j1 = 2 * t4 + 1, j2 = 8 + 2 * t4, j3 = 9 + 2 * t4;
          const float sc = p.scale_log2;
          float x00 = j0 < nvalid ? s0[0] * sc : -INFINITY;
          float x01 = j1 < nvalid ? s0[1] * sc : -INFINITY;
          float x02 = j2 < nvalid ? s1[0] * sc : -INFINITY;
          float x03 = j3 < nvalid ? s1[1] * sc : -INFINITY;
          float x10 = j0 < nvalid ? s0[2] * sc : -INFINITY;
          float x11 = j1 < nvalid ? s0[3] * sc : -INFINITY;
          float x12 = j2 < nvalid ? s1[2] * sc : -INFINITY;
          float x13 = j3 < nvalid ? s1[3] * sc : -INFINITY;
          float mx0 = fmaxf(fmaxf(x00, x01), fmaxf(x02, x03));
          float mx1 = fmaxf(fmaxf(x10, x11), fmaxf(x12, x13));
          mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffff, mx0, 1));
          mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffff, mx0, 2));
          mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffff, mx1, 1));
          mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffff, mx1, 2));
          const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);  // finite: >= 1 valid token
          const float a0 = exp2f(m0 - mn0), a1 = exp2f(m1 - mn1);  // exp2(-inf) = 0 on first unit
          m0 = mn0;
          m1 = mn1;
          const float p00 = exp2f(x00 - mn0), p01 = exp2f(x01 - mn0), p02 = exp2f(x02 - mn0), p03 = exp2f(x03 - mn0);
          const float p10 = exp2f(x10 - mn1), p11 = exp2f(x11 - mn1), p12 = exp2f(x12 - mn1), p13 = exp2f(x13 - mn1);
          l0 = l0 * a0 + (p00 + p01) + (p02 + p03);
          l1 = l1 * a1 + (p10 + p11) + (p12 + p13);
#pragma unroll
          for (int j = 0; j < D / 8; ++j) {
            acc[j][0] *= a0;
            acc[j][1] *= a0;
            acc[j][2] *= a1;
            acc[j][3] *= a1;
          }
          uint32_t pa[4];
          pa[0] = pack_bf16x2(p00, p01);
          pa[1] = pack_bf16x2(p10, p11);
          pa[2] = pack_bf16x2(p02, p03);
          pa[3] = pack_bf16x2(p12, p13);
          // ---- O += P V ----
          const uint32_t vbase = smem_u32(vb);
#pragma unroll
          for (int nd = 0; nd < D / 16; ++nd) {
            const int box = nd >> 2;
            const int chunk = (nd & 3) * 2 + (mi >> 1);
            const int tok = (mi & 1) * 8 + ri;
            uint32_t r0, r1, r2, r3;
            ldmatrix_x4_trans(r0, r1, r2, r3, vbase + box * 2048 + swz128(tok, chunk));
            mma_bf16_16816(acc[2 * nd], pa, r0, r1);
            mma_bf16_16816(acc[2 * nd + 1], pa, r2, r3);
          }
          if (nvalid < 16) fence_proxy_async_smem();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
    }

    // ---- merge the NCW warps' states for head bh ----
    l0 += __shfl_xor_sync(0xffffffff, l0, 1);
    l0 += __shfl_xor_sync(0xffffffff, l0, 2);
    l1 += __shfl_xor_sync(0xffffffff, l1, 1);
    l1 += __shfl_xor_sync(0xffffffff, l1, 2);
    float* mw = merge + cw * G * (D + 2);  // [G][D] acc, then m[G], l[G]
    if (t4 == 0) {
      if (g < G) { mw[G * D + g] = m0; mw[G * D + G + g] = l0; }
      if (g + 8 < G) { mw[G * D + g + 8] = m1; mw[G * D + G + g + 8] = l1; }
    }
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      const int d = j * 8 + 2 * t4;
      if (g < G) { mw[g * D + d] = acc[j][0]; mw[g * D + d + 1] = acc[j][1]; }
      if (g + 8 < G) { mw[(g + 8) * D + d] = acc[j][2]; mw[(g + 8) * D + d + 1] = acc[j][3]; }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(32 * kNCW));

    const bool whole = (rs == hs) && (re == he);
    float* slot = p.part + size_t(bh + blockIdx.x) * G * (D + 2);
    for (int e = ctid; e < G * D; e += 32 * kNCW) {
      const int r = e / D;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kNCW; ++w) M = fmaxf(M, merge[w * G * (D + 2) + G * D + r]);
      float L = 0.f, A = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int w = 0; w < kNCW; ++w) {
          const float* mwx = merge + w * G * (D + 2);
          const float f = exp2f(mwx[G * D + r] - M);
          L += mwx[G * D + G + r] * f;
          A += mwx[e] * f;
        }
      }
      if (whole) {
        p.out[size_t(bh) * G * D + e] = __bfloat16_as_ushort(__float2bfloat16_rn(L > 0.f ? A / L : 0.f));
      } else {
        slot[e] = A;
        if (e % D == 0) { slot[G * D + r] = M; slot[G * D + G + r] = L; }
      }
    }
    if (!whole) {
      __threadfence();
      asm volatile("bar.sync 1, %0;" ::"n"(32 * kNCW));
      const int c_first = hs / seg, c_last = (he - 1) / seg;
      if (ctid == 0) {
        const int old = atomicAdd(&p.counters[bh], 1);
        const int last = old == c_last - c_first;
        if (last) p.counters[bh] = 0;
        *flag = last;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(32 * kNCW));
      if (*flag) {
        __threadfence();
        const int np = c_last - c_first + 1;
        const float* p0 = p.part + size_t(bh + c_first) * G * (D + 2);
        // (m, l) of every partial, then its scale factor, staged in `merge`
        float* mm = merge;             // [np][G]
        float* ll = mm + np * G;       // [np][G]
        float* rowL = ll + np * G;     // [G]
        if (2 * np * G + G <= kNCW * G * (D + 2)) {
          for (int t = ctid; t < np * G; t += 32 * kNCW) {
            const float* sl = p0 + size_t(t / G) * G * (D + 2);
            mm[t] = __ldcg(sl + G * D + t % G);
            ll[t] = __ldcg(sl + G * D + G + t % G);
          }
          asm volatile("bar.sync 1, %0;" ::"n"(32 * kNCW));
          // row maxima and normalisers: one consumer warp per query head
          for (int r = cw; r < G; r += kNCW) {
            float M = -INFINITY;
            for (int c = lane; c < np; c += 32) M = fmaxf(M, mm[c * G + r]);
            for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffff, M, o));
            float L = 0.f;
            for (int c = lane; c < np; c += 32) {
              const float f = M == -INFINITY ? 0.f : exp2f(mm[c * G + r] - M);
              mm[c * G + r] = f;  // scale factor of partial c, row r
              L += ll[c * G + r] * f;
            }
            for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(0xffffffff, L, o);
            if (lane == 0) rowL[r] = L;
          }
          asm volatile("bar.sync 1, %0;" ::"n"(32 * kNCW));
          for (int e = ctid; e < G * D; e += 32 * kNCW) {
            const int r = e / D;
            float A0 = 0.f, A1 = 0.f, A2 = 0.f, A3 = 0.f;
            int c = 0;
            for (; c + 4 <= np; c += 4) {  // four independent L2 loads in flight
              const float v0 = __ldcg(p0 + size_t(c) * G * (D + 2) + e);
              const float v1 = __ldcg(p0 + size_t(c + 1) * G * (D + 2) + e);
              const float v2 = __ldcg(p0 + size_t(c + 2) * G * (D + 2) + e);
              const float v3 = __ldcg(p0 + size_t(c + 3) * G * (D + 2) + e);
              A0 = fmaf(v0, mm[c * G + r], A0);
              A1 = fmaf(v1, mm[(c + 1) * G + r], A1);
              A2 = fmaf(v2, mm[(c + 2) * G + r], A2);
              A3 = fmaf(v3, mm[(c + 3) * G + r], A3);
            }
            for (; c < np; ++c) A0 = fmaf(__ldcg(p0 + size_t(c) * G * (D + 2) + e), mm[c * G + r], A0);
            const float A = (A0 + A1) + (A2 + A3), L = rowL[r];
            p.out[size_t(bh) * G * D + e] = __bfloat16_as_ushort(__float2bfloat16_rn(L > 0.f ? A / L : 0.f));
          }
        } else {
          for (int e = ctid; e < G * D; e += 32 * kNCW) {
            const int r = e / D;
            float M = -INFINITY;
            for (int c = c_first; c <= c_last; ++c)
              M = fmaxf(M, __ldcg(p.part + size_t(bh + c) * G * (D + 2) + G * D + r));
            float L = 0.f, A = 0.f;
            if (M != -INFINITY) {
              for (int c = c_first; c <= c_last; ++c) {
                const float* sl = p.part + size_t(bh + c) * G * (D + 2);
                const float f = exp2f(__ldcg(sl + G * D + r) - M);
                L += __ldcg(sl + G * D + G + r) * f;
                A += __ldcg(sl + e) * f;
              }
            }
            p.out[size_t(bh) * G * D + e] = __bfloat16_as_ushort(__float2bfloat16_rn(L > 0.f ? A / L : 0.f));
          }
        }
      }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(32 * kNCW));  // merge buffer free for the next head
    rs = re;
  }
}

template <int D, int S>
int launch(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, int64_t num_pages, int page_size,
           const int32_t* seqlens, const int32_t* table, int64_t table_stride, int B, int Hq, int Hk, float scale,
           uint16_t* out, void* ws, size_t ws_bytes, int* err, cudaStream_t stream) {
  const int G = Hq / Hk;
  const int BH = B * Hk;
  const int sms = device_sms();
  if (sms <= 0) return WGKV_ECUDA;
  const int grid = sms * kCtasPerSM;
  const size_t need = size_t(BH) * 4 + 256 + size_t(BH + grid) * G * (D + 2) * 4;
  if (ws_bytes < need) return WGKV_ENOSPC;
  CUtensorMap tmK, tmV;
  const uint64_t rows = uint64_t(num_pages) * page_size;
  if (!encode_2d_bf16(&tmK, kc, D, rows, D, 64, 16, true)) return WGKV_ECUDA;
  if (!encode_2d_bf16(&tmV, vc, D, rows, D, 64, 16, true)) return WGKV_ECUDA;
  DecodeParams p;
  p.q = q;
  p.out = out;
  p.seqlens = seqlens;
  p.table = table;
  p.table_stride = table_stride;
  p.num_pages = num_pages;
  p.page_size = page_size;
  p.upp = page_size / 16;
  p.BH = BH;
  p.G = G;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.counters = reinterpret_cast<int*>(ws);
  p.part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + ((size_t(BH) * 4 + 255) & ~size_t(255)));
  p.err = err;
  const size_t smem = smem_bytes<D, S>(BH, G);
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(paged_decode_kernel<D, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) !=
        cudaSuccess)
      return WGKV_ECUDA;
    attr_set[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // overlap set-up with the prior kernel
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, paged_decode_kernel<D, S>, tmK, tmV, p) != cudaSuccess) return WGKV_ECUDA;
  return cudaGetLastError() == cudaSuccess ? WGKV_OK : WGKV_ECUDA;
}

// Argument checks shared by both decode entry points (run before anything is enqueued).
int check_decode_args(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, int64_t num_pages,
                      int page_size, const int32_t* cache_seqlens, const int32_t* block_table, int batch,
                      int num_q_heads, int num_kv_heads, int head_dim, const uint16_t* out) {
  if (!q || !k_cache || !v_cache || !cache_seqlens || !block_table || !out) return WGKV_EINVAL;
  if (batch <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0) return WGKV_EINVAL;
  if (num_q_heads / num_kv_heads > 16 || page_size <= 0 || page_size % 16 != 0 || num_pages <= 0) return WGKV_EINVAL;
  if (head_dim != 64 && head_dim != 128) return WGKV_EINVAL;
  if (batch * num_kv_heads > kMaxBH) return WGKV_EINVAL;
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15) return WGKV_EINVAL;
  return WGKV_OK;
}

}  // namespace
}  // namespace wgkv

extern "C" size_t wgkv_paged_decode_workspace_size(int batch, int num_q_heads, int num_kv_heads, int head_dim) {
  const int sms = wgkv::device_sms();
  const int grid = (sms > 0 ? sms : 148) * wgkv::kCtasPerSM;
  const size_t BH = size_t(batch) * num_kv_heads;
  const int G = num_kv_heads > 0 ? num_q_heads / num_kv_heads : 1;
  return ((BH * 4 + 255) & ~size_t(255)) + (BH + grid) * G * (head_dim + 2) * 4 + 256;
}

extern "C" int wgkv_paged_decode(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                 int64_t num_pages, int page_size, const int32_t* cache_seqlens,
                                 const int32_t* block_table, int64_t table_stride, int batch, int num_q_heads,
                                 int num_kv_heads, int head_dim, float softmax_scale, uint16_t* out, void* workspace,
                                 size_t workspace_bytes, int* err, void* stream) {
  using namespace wgkv;
  if (!workspace) return WGKV_EINVAL;
  const int chk = check_decode_args(q, k_cache, v_cache, num_pages, page_size, cache_seqlens, block_table, batch,
                                    num_q_heads, num_kv_heads, head_dim, out);
  if (chk != WGKV_OK) return chk;
  constexpr size_t kMaxSmem = 227 * 1024;
  const int BH = batch * num_kv_heads, G = num_q_heads / num_kv_heads;
  const cudaStream_t st = as_stream(stream);
#define WGKV_DEC_LAUNCH(DD, SS)                                                                                     \
  launch<DD, SS>(q, k_cache, v_cache, num_pages, page_size, cache_seqlens, block_table, table_stride, batch,         \
                 num_q_heads, num_kv_heads, softmax_scale, out, workspace, workspace_bytes, err, st)
  // deepest pipeline that fits next to the prefix and merge buffers
  switch (head_dim) {
    case 64:
      if (smem_bytes<64, 6>(BH, G) <= kMaxSmem) return WGKV_DEC_LAUNCH(64, 6);
      if (smem_bytes<64, 3>(BH, G) <= kMaxSmem) return WGKV_DEC_LAUNCH(64, 3);
      return WGKV_EINVAL;
    case 128:
      if (smem_bytes<128, 3>(BH, G) <= kMaxSmem) return WGKV_DEC_LAUNCH(128, 3);
      if (smem_bytes<128, 2>(BH, G) <= kMaxSmem) return WGKV_DEC_LAUNCH(128, 2);
      return WGKV_EINVAL;
#undef WGKV_DEC_LAUNCH
    default:
      return WGKV_EINVAL;
  }
}

// ---------------------------------------------------------------------------
// Allocation-free variant: split-K scratch in a file-scope device array.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_decode_scratch[WGKV_PAGED_DECODE_STATIC_SCRATCH_BYTES];

namespace {
std::mutex g_scratch_mu;
void* g_scratch_addr[64] = {nullptr};

// Device address of g_decode_scratch on the current device (resolved once per
// device; the symbol's host-side name is not a device address).
void* static_scratch(int dev) {
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_decode_scratch) != cudaSuccess) return nullptr;
    g_scratch_addr[dev] = p;
  }
  return g_scratch_addr[dev];
}
}  // namespace

extern "C" int wgkv_paged_decode_noalloc(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                         int64_t num_pages, int page_size, const int32_t* cache_seqlens,
                                         const int32_t* block_table, int64_t table_stride, int batch,
                                         int num_q_heads, int num_kv_heads, int head_dim, float softmax_scale,
                                         uint16_t* out, int* err, void* stream) {
  const int chk = wgkv::check_decode_args(q, k_cache, v_cache, num_pages, page_size, cache_seqlens, block_table,
                                          batch, num_q_heads, num_kv_heads, head_dim, out);
  if (chk != WGKV_OK) return chk;
  const size_t need = wgkv_paged_decode_workspace_size(batch, num_q_heads, num_kv_heads, head_dim);
  if (need > WGKV_PAGED_DECODE_STATIC_SCRATCH_BYTES) return WGKV_ENOSPC;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return WGKV_ECUDA;
  void* scratch = static_scratch(dev);
  if (!scratch) return WGKV_ECUDA;
  // the per-head counters must start at zero (the array keeps the last call's contents)
  const size_t counter_bytes = size_t(batch) * num_kv_heads * 4;
  if (cudaMemsetAsync(scratch, 0, counter_bytes, wgkv::as_stream(stream)) != cudaSuccess) return WGKV_ECUDA;
  return wgkv_paged_decode(q, k_cache, v_cache, num_pages, page_size, cache_seqlens, block_table, table_stride, batch,
                           num_q_heads, num_kv_heads, head_dim, softmax_scale, out, scratch,
                           WGKV_PAGED_DECODE_STATIC_SCRATCH_BYTES, err, stream);
}
