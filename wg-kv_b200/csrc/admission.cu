// Write gate, admission compaction, ring append and lazy promotion (sm_100a).
//
// Reference: src/modeling_layers.py -- GatingPredictor.forward fast path
// (:170-196), the threshold (:1465), prefill_wrapper's ring fill and per-head
// compaction (:1290-1331, a host loop with torch.where + .item() syncs),
// migrate_local_kv_to_global (:674-763, nonzero + .item()), and
// decode_wrapper's ring append (:1390-1413).  Here every step is a device
// kernel with no host synchronisation: counts are reduced per 2048-token
// chunk with warp ballots, scanned on the device, and pages are handed out by
// a device-side bump allocator in the reference's (layer, batch, head) order
// so the page tables come out identical.  Also here: the QUEST page key
// bounds kept by compaction and promotion (:744-761, :1333-1347), promotion
// drawing on the SnapKV free list first (:694-709), the decode prologue fused
// in front of the gate (q/k norm + RoPE, modeling_llama.py:265-271,
// modeling_qwen3.py:236-239) and the device copy of the ring position that
// lets a decode step replay as a CUDA graph.
#include <math.h>
#include <string.h>

#include "common.cuh"
#include "runtime.h"

namespace wgkv {

// Mask counting per 2048-token chunk (declared in common.cuh; also launched by the sparse-index builder).
__global__ void __launch_bounds__(kScanThreads) chunk_count_kernel(MaskView mv, int Hk, int limit, int nch,
                                                                   int* counts) {
  const int bh = blockIdx.y, b = bh / Hk, h = bh - b * Hk, c = blockIdx.x;
  const int t0 = c * kChunk + threadIdx.x * 8;
  int n = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) n += (t0 + j < limit) && mv.at(b, h, t0 + j) ? 1 : 0;
  for (int o = 16; o; o >>= 1) n += __shfl_xor_sync(0xffffffff, n, o);
  __shared__ int wsum[kScanThreads / 32];
  if ((threadIdx.x & 31) == 0) wsum[threadIdx.x >> 5] = n;
  __syncthreads();
  if (threadIdx.x == 0) {
    int s = 0;
    for (int w = 0; w < kScanThreads / 32; ++w) s += wsum[w];
    counts[bh * nch + c] = s;
  }
}

namespace {

// ============================================================================
// gate: bf16 2-layer MLP per (b, h, t) on mma.sync tensor cores
// ============================================================================
constexpr int kGateRows = 128;   // rows (tokens) per CTA
constexpr int kGateThreads = 256;  // 8 warps x 16 rows
constexpr int kGateChunk = 64;   // W1 rows (hidden neurons) per shared-memory chunk

struct GateParams {
  const uint16_t* in[3];
  int64_t sb[3], sh[3], st[3];
  const uint16_t* norm[3];
  int n_in;
  int B, Hk, L, D, I, inner, act;  // act: WGKV_GATE_SILU | WGKV_GATE_CONV bits
  const uint16_t *w1, *b1, *w2, *b2;
  float eps, thr, floor;             // floor: bf16 score floor of the conv path (-inf on the fast path)
  uint16_t* scores;
  int64_t ssb, ssh, sst;
  uint8_t* mask;
  int64_t msb, msh, mst;
};


WGKV_DEV float act_fn(float x, int act) {
  if (act & WGKV_GATE_SILU) return x / (1.f + expf(-x));       // nn.SiLU
  return 0.5f * x * (1.f + erff(x * 0.70710678118654752440f));  // nn.GELU() (erf form)
}

// Hidden pre-activation from the fp32 dot product: the conv path (g_fast_path=False, :198-201)
// rounds once after the bias; the einsum fast path (:185-187) rounds the product, then the sum.
WGKV_DEV float gate_hidden(float dot, float bias, int act) {
  return (act & WGKV_GATE_CONV) ? bf16_round(dot + bias) : bf16_round(bf16_round(dot) + bias);
}

// Score from the fp32 output dot product: bias (same rounding rule), sigmoid in bf16, then the
// conv path's torch.clamp(min=g_epsilon) (:205; NaN stays NaN as in torch).
WGKV_DEV float gate_score(float dot, float bias, int act, float floor) {
  const float o = (act & WGKV_GATE_CONV) ? bf16_round(dot + bias) : bf16_round(bf16_round(dot) + bias);
  const float s = bf16_round(1.f / (1.f + expf(-o)));
  return s < floor ? floor : s;
}

__global__ void __launch_bounds__(kGateThreads) gate_kernel(GateParams p) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int I = p.I, RS = I + 8;  // padded row stride (elements): conflict-free ldmatrix
  uint16_t* xs = reinterpret_cast<uint16_t*>(sm);
  uint16_t* ws = xs + kGateRows * RS;
  float* b1s = reinterpret_cast<float*>(ws + kGateChunk * RS);
  float* w2s = b1s + kGateChunk;
  const int h = blockIdx.y;
  const int row0 = blockIdx.x * kGateRows;
  const int nrows = p.B * p.L;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // ---- stage the input rows (concat + optional RMS norm) as bf16 ----------
  // Each warp owns rows warp, warp + 8, ...: all of its rows' loads for one input are issued before
  // any is used (kRowsPerWarp independent 8-byte loads per lane in flight), so the staging runs at
  // memory throughput rather than one row latency after another.
  constexpr int kRowsPerWarp = kGateRows / (kGateThreads / 32);
  const int per = p.D / 32;  // elements per lane per input (2 or 4)
  for (int s = 0; s < p.n_in; ++s) {
    uint32_t raw[kRowsPerWarp][2];
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
      const int gr = row0 + warp + i * (kGateThreads / 32);
      raw[i][0] = raw[i][1] = 0u;
      if (gr < nrows) {
        const int b = gr / p.L, t = gr - b * p.L;
        const uint16_t* src = p.in[s] + b * p.sb[s] + h * p.sh[s] + int64_t(t) * p.st[s] + lane * per;
        if (per == 4) {
          const uint2 w = __ldg(reinterpret_cast<const uint2*>(src));
          raw[i][0] = w.x;
          raw[i][1] = w.y;
        } else {
          raw[i][0] = __ldg(reinterpret_cast<const uint32_t*>(src));
        }
      }
    }
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
      const int r = warp + i * (kGateThreads / 32);
      float x[4] = {__uint_as_float(raw[i][0] << 16), __uint_as_float(raw[i][0] & 0xffff0000u),
                    __uint_as_float(raw[i][1] << 16), __uint_as_float(raw[i][1] & 0xffff0000u)};
      if (p.norm[s]) {
        // GatingRMSNorm.forward (:123-128): fp32 variance, x * rsqrt(var + eps) -> bf16, * weight -> bf16
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) ss += x[j] * x[j];  // x[j] = 0 past `per`
        for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffff, ss, o);
        const float inv = 1.f / sqrtf(ss / float(p.D) + p.eps);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (j < per) {
            const float y = bf16_round(x[j] * inv);
            x[j] = bf16_round(bf2f(p.norm[s][lane * per + j]) * y);
          }
        }
      }
      // rows past the end stay zero (their loads were skipped, and the norm of zeros is zero)
      uint16_t* dst = xs + r * RS + s * p.D + lane * per;
      *reinterpret_cast<uint32_t*>(dst) = pack_bf16x2(x[0], x[1]);
      if (per == 4) *reinterpret_cast<uint32_t*>(dst + 2) = pack_bf16x2(x[2], x[3]);
    }
  }

  const int g = lane >> 2, t4 = lane & 3, mi = lane >> 3, ri = lane & 7;
  float part0 = 0.f, part1 = 0.f;
  const uint16_t* w1h = p.w1 + int64_t(h) * p.inner * I;
  for (int n0 = 0; n0 < p.inner; n0 += kGateChunk) {
    __syncthreads();
    // W1 rows n0 .. n0+63 (zero past inner), 16-byte vectors
    const int vec_per_row = I / 8;
    for (int e = tid; e < kGateChunk * vec_per_row; e += kGateThreads) {
      const int j = e / vec_per_row, c = e - j * vec_per_row;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (n0 + j < p.inner) v = *reinterpret_cast<const uint4*>(w1h + int64_t(n0 + j) * I + c * 8);
      *reinterpret_cast<uint4*>(ws + j * RS + c * 8) = v;
    }
    if (tid < kGateChunk) {
      const bool ok = n0 + tid < p.inner;
      b1s[tid] = ok ? bf2f(p.b1[h * p.inner + n0 + tid]) : 0.f;
      w2s[tid] = ok ? bf2f(p.w2[h * p.inner + n0 + tid]) : 0.f;
    }
    __syncthreads();
    float acc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    const uint32_t xbase = smem_u32(xs + (warp * 16 + (mi & 1) * 8 + ri) * RS + (mi >> 1) * 8);
    const uint32_t wbase = smem_u32(ws + ((mi >> 1) * 8 + ri) * RS + (mi & 1) * 8);
    for (int kk = 0; kk < I / 16; ++kk) {
      uint32_t a[4];
      ldmatrix_x4(a[0], a[1], a[2], a[3], xbase + kk * 32);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t r0, r1, r2, r3;
        ldmatrix_x4(r0, r1, r2, r3, wbase + (np * 16 * RS) * 2 + kk * 32);
        mma_bf16_16816(acc[2 * np], a, r0, r1);
        mma_bf16_16816(acc[2 * np + 1], a, r2, r3);
      }
    }
    // epilogue: bf16(h) -> bf16(h + b1) -> bf16(act) -> fp32 dot with w2
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int n = j * 8 + 2 * t4 + e;
        const float bb = b1s[n], ww = w2s[n];
        float h0 = gate_hidden(acc[j][e], bb, p.act);
        float h1 = gate_hidden(acc[j][2 + e], bb, p.act);
        part0 += bf16_round(act_fn(h0, p.act)) * ww;
        part1 += bf16_round(act_fn(h1, p.act)) * ww;
      }
    }
  }
  part0 += __shfl_xor_sync(0xffffffff, part0, 1);
  part0 += __shfl_xor_sync(0xffffffff, part0, 2);
  part1 += __shfl_xor_sync(0xffffffff, part1, 1);
  part1 += __shfl_xor_sync(0xffffffff, part1, 2);
  if (t4 == 0) {
    const float b2 = bf2f(p.b2[h]);
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int gr = row0 + warp * 16 + g + rr * 8;
      if (gr >= nrows) continue;
      const int b = gr / p.L, t = gr - b * p.L;
      const float s = gate_score(rr ? part1 : part0, b2, p.act, p.floor);
      if (p.scores) p.scores[b * p.ssb + h * p.ssh + int64_t(t) * p.sst] = f2bf(s);
      if (p.mask) p.mask[b * p.msb + h * p.msh + int64_t(t) * p.mst] = s > p.thr ? 1 : 0;
    }
  }
}

// ============================================================================
// prefill compaction
// ============================================================================
struct PoolArgs {
  wgkv_pool P;
};

// Single CTA: per-head chunk scans, page allocation in (b, h) order, table writes.
__global__ void __launch_bounds__(1024) prefill_alloc_kernel(PoolArgs pa, int layer, int nch, int n_loc,
                                                             int* counts, int* totals, int* first, int* okflag) {
  const wgkv_pool& P = pa.P;
  const int BH = P.batch * P.kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int bh = warp; bh < BH; bh += 32) {
    int carry = 0;
    for (int c0 = 0; c0 < nch; c0 += 32) {
      const int c = c0 + lane;
      const int v = c < nch ? counts[bh * nch + c] : 0;
      int x = v;
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffff, x, o);
        if (lane >= o) x += y;
      }
      if (c < nch) counts[bh * nch + c] = carry + x - v;
      carry += __shfl_sync(0xffffffff, x, 31);
    }
    if (lane == 0) totals[bh] = carry;
  }
  __syncthreads();
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    const int nf = *P.next_free_block;
    int64_t run = 0;
    int ok = 1;
    for (int bh = 0; bh < BH; ++bh) {
      const int n = totals[bh];
      if (n > 0 && n_loc + n > P.max_tokens_per_head) {
        set_error(P.err, WGKV_ERR_HEAD_CAPACITY);
        ok = 0;
      }
      first[bh] = int(nf + run);
      run += (n + P.page - 1) / P.page;
    }
    if (nf + run > P.total_blocks) {
      set_error(P.err, WGKV_ERR_POOL_EXHAUSTED);
      ok = 0;
    }
    if (ok) *P.next_free_block = int(nf + run);
    *okflag = ok;
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  const int lp = P.window / P.page;
  for (int bh = warp; bh < BH; bh += 32) {
    const int n = totals[bh];
    const int need = (n + P.page - 1) / P.page;
    int32_t* trow = P.block_table + (int64_t(layer) * BH + bh) * P.max_blocks_per_head + lp;
    for (int j = lane; j < need; j += 32) trow[j] = first[bh] + j;
    if (lane == 0) P.global_lengths[layer * BH + bh] = n;
  }
}

struct RowSrc {
  const uint16_t* p;
  int64_t sb, sh, st;
};

template <bool kVec16>
WGKV_DEV void copy_row(uint16_t* dst, const uint16_t* src, int D, int lane_in_group, int group_size) {
  if (kVec16) {
    for (int c = lane_in_group; c < D / 8; c += group_size)
      reinterpret_cast<uint4*>(dst)[c] = *reinterpret_cast<const uint4*>(src + c * 8);
  } else {
    for (int c = lane_in_group; c < D / 2; c += group_size)
      reinterpret_cast<uint32_t*>(dst)[c] = *reinterpret_cast<const uint32_t*>(src + c * 2);
  }
}

template <bool kVec16>
__global__ void __launch_bounds__(kScanThreads) prefill_scatter_kernel(PoolArgs pa, int layer, int L, int n_early,
                                                                       int n_loc, int nch, MaskView mv, RowSrc K,
                                                                       RowSrc V, RowSrc PK, const int* counts,
                                                                       const int* first, const int* okflag) {
  if (!*okflag) return;
  const wgkv_pool& P = pa.P;
  const int Hk = P.kv_heads, BH = P.batch * Hk, D = P.head_dim;
  const int bh = blockIdx.y, b = bh / Hk, h = bh - b * Hk, c = blockIdx.x;
  __shared__ int2 list[kChunk];  // (token, -2 - ring slot for ring rows)
  __shared__ int wsum[kScanThreads / 32];
  __shared__ int s_n;
  const int t0 = c * kChunk + threadIdx.x * 8;
  const int ring_start = L - n_loc;  // first token that goes to the ring
  const int64_t ring_row0 = (int64_t(layer) * BH + bh) * P.window;
  uint8_t mk[8];
  int ng = 0, nr = 0;
  {
    // the thread's 8 mask bytes: one 8-byte load when they are contiguous and aligned
    const uint8_t* mp = mv.m + b * mv.sb + h * mv.sh + int64_t(t0) * mv.st;
    if (mv.st == 1 && t0 + 8 <= L && (reinterpret_cast<uintptr_t>(mp) & 7) == 0) {
      const uint2 w = *reinterpret_cast<const uint2*>(mp);
#pragma unroll
      for (int j = 0; j < 8; ++j) mk[j] = uint8_t(((j < 4 ? w.x : w.y) >> (8 * (j & 3))) & 0xff);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) mk[j] = t0 + j < L ? mv.at(b, h, t0 + j) : 0;
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int t = t0 + j;
    ng += (t < n_early && mk[j]) ? 1 : 0;
    nr += (t < L && t >= ring_start) ? 1 : 0;
  }
  int tot;
  const int gbase = block_excl_scan<kScanThreads>(ng, wsum, tot);
  int rtot;
  const int rbase = block_excl_scan<kScanThreads>(nr, wsum, rtot);
  const int chunk_off = (c < nch) ? counts[bh * nch + c] : 0;
  const int64_t gdst0 = int64_t(first[bh]) * P.page + chunk_off;
  int gi = gbase, ri = rbase;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int t = t0 + j;
    if (t < n_early && mk[j]) {
      list[gi] = make_int2(t, 0);  // destination = gdst0 + list index
      ++gi;
    } else if (t < L && t >= ring_start) {
      const int slot = t - ring_start;
      list[tot + ri] = make_int2(t, -2 - slot);  // ring rows encoded as -2 - slot
      P.local_is_global[ring_row0 + slot] = mk[j];
      ++ri;
    }
  }
  if (threadIdx.x == 0) s_n = tot + rtot;
  __syncthreads();
  const int n = s_n;
  // copy rows: one warp-quarter (8 lanes) per row
  const int grp = threadIdx.x >> 3, gl = threadIdx.x & 7;
  if (kVec16 && D <= 128 && !(P.local_pre_key && PK.p)) {
    // two rows per group per pass, every load issued before any store: 8 x 16 B in flight per lane
    constexpr int kG = kScanThreads / 8;
    const int nv = D / 8;  // 16-byte vectors per row (8 or 16)
    for (int e0 = grp; e0 < n; e0 += 2 * kG) {
      uint4 kr[2][2], vr[2][2];
      int64_t dst[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int e = e0 + u * kG;
        if (e >= n) continue;
        const int t = list[e].x;
        dst[u] = e >= tot ? ring_row0 + (-2 - list[e].y) : gdst0 + e;
        const uint16_t* ks = K.p + b * K.sb + h * K.sh + int64_t(t) * K.st;
        const uint16_t* vs = V.p + b * V.sb + h * V.sh + int64_t(t) * V.st;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int c = gl + 8 * i;
          if (c < nv) {
            kr[u][i] = __ldg(reinterpret_cast<const uint4*>(ks) + c);
            vr[u][i] = __ldg(reinterpret_cast<const uint4*>(vs) + c);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (e0 + u * kG >= n) continue;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int c = gl + 8 * i;
          if (c < nv) {
            reinterpret_cast<uint4*>(P.k + dst[u] * D)[c] = kr[u][i];
            reinterpret_cast<uint4*>(P.v + dst[u] * D)[c] = vr[u][i];
          }
        }
      }
    }
    return;
  }
  for (int e = grp; e < n; e += kScanThreads / 8) {
    const int t = list[e].x;
    int64_t dst;
    const bool ring = e >= tot;
    if (ring) dst = ring_row0 + (-2 - list[e].y);
    else dst = gdst0 + e;
    const int64_t so_k = b * K.sb + h * K.sh + int64_t(t) * K.st;
    const int64_t so_v = b * V.sb + h * V.sh + int64_t(t) * V.st;
    copy_row<kVec16>(P.k + dst * D, K.p + so_k, D, gl, 8);
    copy_row<kVec16>(P.v + dst * D, V.p + so_v, D, gl, 8);
    if (ring && P.local_pre_key && PK.p) {
      const int64_t so_p = b * PK.sb + h * PK.sh + int64_t(t) * PK.st;
      copy_row<kVec16>(P.local_pre_key + dst * D, PK.p + so_p, D, gl, 8);
    }
  }
}

// QUEST key bounds of the global pages a prefill just filled (:1333-1347): one warp per page,
// lanes over the head dimension.
__global__ void __launch_bounds__(256) quest_bounds_kernel(PoolArgs pa, int layer, const int* okflag) {
  const wgkv_pool& P = pa.P;
  if (!*okflag) return;
  const int BH = P.batch * P.kv_heads, bh = blockIdx.y;
  const int T = P.page, D = P.head_dim;
  const int glen = P.global_lengths[int64_t(layer) * BH + bh];
  const int pg = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (pg * T >= glen) return;
  const int64_t pid = P.block_table[(int64_t(layer) * BH + bh) * P.max_blocks_per_head + P.window / T + pg];
  const int rows = min(T, glen - pg * T);
  for (int c = lane; c < D; c += 32) {
    uint16_t lo = P.k[pid * T * D + c], hi = lo;
    for (int r = 1; r < rows; ++r) {
      const uint16_t kb = P.k[(pid * T + r) * D + c];
      if (bf2f(kb) < bf2f(lo)) lo = kb;
      if (bf2f(kb) > bf2f(hi)) hi = kb;
    }
    P.quest_min[pid * D + c] = lo;
    P.quest_max[pid * D + c] = hi;
  }
}

// ============================================================================
// decode: ring append + cache_seqlens
// ============================================================================
// ins < 0: the position lives in pool.ring_state = {local_length, local_ptr} (decode_wrapper :1390-1396)
__device__ __forceinline__ void ring_position(const wgkv_pool& P, int& ins, int& cur) {
  if (ins >= 0) return;
  const int len = P.ring_state[0];
  if (len < P.window) {
    ins = len;
    cur = len + 1;
  } else {
    ins = P.ring_state[1];
    cur = P.window;
  }
}

__global__ void __launch_bounds__(256) decode_append_kernel(PoolArgs pa, int layer, int ins, int cur, RowSrc K,
                                                            RowSrc V, RowSrc PK, int32_t* cache_seqlens) {
  const wgkv_pool& P = pa.P;
  const int Hk = P.kv_heads, BH = P.batch * Hk, D = P.head_dim;
  const int i = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (i >= BH) return;
  ring_position(P, ins, cur);
  const int b = i / Hk, h = i - b * Hk;
  const int64_t row = (int64_t(layer) * BH + i) * P.window + ins;
  copy_row<false>(P.k + row * D, K.p + b * K.sb + h * K.sh, D, lane, 32);
  copy_row<false>(P.v + row * D, V.p + b * V.sb + h * V.sh, D, lane, 32);
  if (PK.p && P.local_pre_key) copy_row<false>(P.local_pre_key + row * D, PK.p + b * PK.sb + h * PK.sh, D, lane, 32);
  if (lane == 0 && cache_seqlens) cache_seqlens[i] = cur + P.global_lengths[layer * BH + i];
}

// ============================================================================
// lazy promotion (migrate_local_kv_to_global)
// ============================================================================
constexpr int kPromoteThreads = 1024;
constexpr int kPromoteMaxPer = 32;  // (layer, b, h) entries per thread: up to 32768 heads per pool

__global__ void __launch_bounds__(kPromoteThreads) promote_kernel(PoolArgs pa, int ptr) {
  const wgkv_pool& P = pa.P;
  const int N = P.layers * P.batch * P.kv_heads;
  const int W = P.window, T = P.page;
  if (ptr < 0) {  // position on the device: promote only once the ring is full (:1470)
    if (P.ring_state[0] < W) return;
    ptr = P.ring_state[1];
  }
  // a capacity error already flagged (and not yet read by the host) stops promotions: the
  // reference has aborted at that point, and the copy kernel relies on it
  if (P.err && (*P.err & (WGKV_ERR_HEAD_CAPACITY | WGKV_ERR_POOL_EXHAUSTED))) return;
  const int per = (N + kPromoteThreads - 1) / kPromoteThreads;
  const int i0 = threadIdx.x * per;  // contiguous entries keep the (layer, b, h) allocation order
  __shared__ int wsum[kPromoteThreads / 32];
  __shared__ int s_ovf, s_nf, s_ok, s_fc, s_nff;
  if (threadIdx.x == 0) s_ovf = 0;
  // all loads of this thread's entries are issued together; admission bits kept as a bitmask
  uint32_t fmask = 0;
#pragma unroll
  for (int k = 0; k < kPromoteMaxPer; ++k)
    if (k < per && i0 + k < N && P.local_is_global[int64_t(i0 + k) * W + ptr]) fmask |= 1u << k;
  int need = 0, ovf = 0;
#pragma unroll
  for (int k = 0; k < kPromoteMaxPer; ++k) {
    if (fmask & (1u << k)) {
      const int gl = P.global_lengths[i0 + k];
      need += (gl % T) == 0;
      ovf |= (W + gl + 1 > P.max_tokens_per_head);
    }
  }
  // block-wide exclusive scan of `need` (thread order = entry order)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = need;
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffff, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[warp] = x;
  if (ovf) atomicOr(&s_ovf, 1);
  __syncthreads();
  int wb = 0, tot = 0;
  for (int w = 0; w < kPromoteThreads / 32; ++w) {
    if (w < warp) wb += wsum[w];
    tot += wsum[w];
  }
  if (threadIdx.x == 0) {
    const int nf = *P.next_free_block;
    // pages freed by eviction are reused first, the free list's tail in list order (:694-709)
    const int fc = P.free_count ? *P.free_count : 0;
    const int nff = tot < fc ? tot : fc;
    s_nf = nf;
    s_fc = fc;
    s_nff = nff;
    s_ok = 0;
    if (s_ovf) {
      set_error(P.err, WGKV_ERR_HEAD_CAPACITY);
    } else if (int64_t(nf) + tot - nff > P.total_blocks) {
      set_error(P.err, WGKV_ERR_POOL_EXHAUSTED);
    } else {
      *P.next_free_block = nf + tot - nff;
      if (nff) *P.free_count = fc - nff;
      s_ok = 1;
    }
  }
  __syncthreads();
  if (!s_ok) return;
  int next = wb + x - need;  // allocation rank of this thread's first new page
#pragma unroll 1
  for (int k = 0; k < kPromoteMaxPer; ++k) {
    if (!(fmask & (1u << k))) continue;
    const int i = i0 + k;
    const int gl = P.global_lengths[i];
    int32_t* trow = P.block_table + int64_t(i) * P.max_blocks_per_head + W / T;
    if (gl % T == 0) {  // a new page for this token
      const int r = next++;
      trow[gl / T] = r < s_nff ? P.free_ids[s_fc - s_nff + r] : s_nf + (r - s_nff);
    }
    P.global_lengths[i] = gl + 1;
  }
}

// The row copies of a promotion, after promote_kernel wrote the tables and lengths: 8 lanes per
// promoted (layer, b, h), 32 of them per CTA, every load of a row issued before its stores; the
// page's key bounds (:744-761) are updated from the same loads.  Nothing is copied when the pool's
// error word holds a capacity error (promote_kernel then changed nothing either).
__global__ void __launch_bounds__(256) promote_copy_kernel(PoolArgs pa, int ptr) {
  const wgkv_pool& P = pa.P;
  const int N = P.layers * P.batch * P.kv_heads;
  const int W = P.window, T = P.page, D = P.head_dim;
  if (ptr < 0) {
    if (P.ring_state[0] < W) return;
    ptr = P.ring_state[1];
  }
  if (P.err && (*P.err & (WGKV_ERR_HEAD_CAPACITY | WGKV_ERR_POOL_EXHAUSTED))) return;
  const int gl8 = threadIdx.x & 7;
  const int nv = D / 8;  // 16-byte vectors per row (8 or 16)
  const int i = blockIdx.x * 32 + (threadIdx.x >> 3);
  if (i >= N || !P.local_is_global[int64_t(i) * W + ptr]) return;
  {
    const int gl = P.global_lengths[i] - 1;  // the length before this promotion
    const int pid = P.block_table[int64_t(i) * P.max_blocks_per_head + W / T + gl / T];
    const int64_t dst = int64_t(pid) * T + gl % T;
    const int64_t src = int64_t(i) * W + ptr;
    const uint4* ks = reinterpret_cast<const uint4*>(P.k + src * D);
    const uint4* vs = reinterpret_cast<const uint4*>(P.v + src * D);
    uint4 kr[2], vr[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int c = gl8 + 8 * u;
      if (c < nv) {
        kr[u] = ks[c];
        vr[u] = vs[c];
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int c = gl8 + 8 * u;
      if (c >= nv) continue;
      reinterpret_cast<uint4*>(P.k + dst * D)[c] = kr[u];
      reinterpret_cast<uint4*>(P.v + dst * D)[c] = vr[u];
      if (P.quest_min) {  // page key bounds: a new page starts at the key
        uint4* mn = reinterpret_cast<uint4*>(P.quest_min + int64_t(pid) * D) + c;
        uint4* mx = reinterpret_cast<uint4*>(P.quest_max + int64_t(pid) * D) + c;
        const uint4 kv = kr[u];
        if (gl % T == 0) {
          *mn = kv;
          *mx = kv;
        } else {
          const uint4 a = *mn, z = *mx;
          const uint32_t kw[4] = {kv.x, kv.y, kv.z, kv.w}, aw[4] = {a.x, a.y, a.z, a.w}, zw[4] = {z.x, z.y, z.z, z.w};
          uint32_t lo[4], hi[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {  // two bf16 per word: keep each half's min / max bits
            uint32_t l = 0, h2 = 0;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              const uint32_t sh = 16 * half;
              const uint16_t kb = uint16_t(kw[e] >> sh), ab = uint16_t(aw[e] >> sh), zb = uint16_t(zw[e] >> sh);
              l |= uint32_t(bf2f(kb) < bf2f(ab) ? kb : ab) << sh;
              h2 |= uint32_t(bf2f(kb) > bf2f(zb) ? kb : zb) << sh;
            }
            lo[e] = l;
            hi[e] = h2;
          }
          *mn = make_uint4(lo[0], lo[1], lo[2], lo[3]);
          *mx = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        }
      }
    }
  }
}

// local_length / local_ptr update after the last layer of a decode step (:1408-1413)
__global__ void ring_advance_kernel(int32_t* rs, int W) {
  if (rs[0] < W) rs[0] += 1;
  else rs[1] = rs[1] + 1 == W ? 0 : rs[1] + 1;
}

// ============================================================================
// decode: gate on the new key + ring append + cache_seqlens, one CTA per (b, h)
// ============================================================================
constexpr int kDgaThreads = 128;

struct DecodeGateParams {
  RowSrc in[3];  // selected gate inputs (concat order), token stride unused
  const uint16_t* norm[3];
  int n_in, I, inner, act;  // act: WGKV_GATE_SILU | WGKV_GATE_CONV bits
  const uint16_t *w1, *b1, *w2, *b2;
  float eps, thr, floor;
};

// Optional decode prologue fused in front of the gate (modeling_llama.py:265-271, modeling_qwen3.py:
// 236-239): the q/k/v projection row of each sequence, [q heads | k heads | v heads] x D, gets the
// optional per-head RMS norm (q_norm / k_norm), then RoPE at the device-side position; the k row
// before RoPE is the gate's pre_k.  Element-wise roundings follow the bf16 torch expressions
// x * cos + rotate_half(x) * sin and (x * rsqrt(mean(x^2) + eps)).to(bf16) * w.
struct RopeParams {
  const uint16_t* qkv;  // NULL: no prologue (inputs come from DecodeGateParams / K / V)
  int64_t sb;           // elements between sequences
  int Hq;
  const uint16_t *q_norm, *k_norm;
  float eps;
  const uint16_t *cos, *sin;  // (n_pos, D) bf16
  const int64_t* pos;
  int64_t n_pos;
  uint16_t* q_out;  // (B, Hq, D) contiguous
  int sel[3];       // gate input -> staged row (0 pre_k, 1 rotated k, 2 v)
};

// RMS-norm (optional) + RoPE of one D-row by the whole block (thread t owns element t).
WGKV_DEV void norm_rope_row(const uint16_t* src, const uint16_t* norm, float eps, float c, float s, int D,
                            float* xbuf, float* red, uint16_t* pre_out, uint16_t* rot_out) {
  const int tid = threadIdx.x;
  float x = tid < D ? bf2f(src[tid]) : 0.f;
  if (norm) {
    float ss = x * x;
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffff, ss, o);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < kDgaThreads / 32; ++w) tot += red[w];
    const float inv = rsqrtf(tot / float(D) + eps);
    if (tid < D) x = bf16_round(bf16_round(x * inv) * bf2f(norm[tid]));
  }
  if (tid < D) {
    xbuf[tid] = x;
    if (pre_out) pre_out[tid] = f2bf(x);
  }
  __syncthreads();
  if (tid < D) {
    const int hd = D / 2;
    const float xr = tid < hd ? -xbuf[tid + hd] : xbuf[tid - hd];
    rot_out[tid] = f2bf(bf16_round(x * c) + bf16_round(xr * s));
  }
  __syncthreads();  // xbuf / red are reused by the next row
}

__global__ void __launch_bounds__(kDgaThreads) decode_gate_append_kernel(PoolArgs pa, DecodeGateParams g, RopeParams R,
                                                                          int layer, int ins, int cur, RowSrc K,
                                                                          RowSrc V, int32_t* cache_seqlens) {
  const wgkv_pool& P = pa.P;
  const int Hk = P.kv_heads, BH = P.batch * Hk, D = P.head_dim;
  const int i = blockIdx.x, b = i / Hk, h = i - b * Hk;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // launched early behind the previous kernel (programmatic dependent launch): wait for its results
  griddep_wait();
  ring_position(P, ins, cur);
  // the paged-decode launch that follows may start its set-up now (it waits for this grid's results)
  griddep_launch();
  __shared__ float xs[384];
  __shared__ float part[kDgaThreads / 32];
  __shared__ __align__(16) uint16_t stage[3][128];
  const int64_t row = (int64_t(layer) * BH + i) * P.window + ins;
  const uint16_t* k_src = K.p + b * K.sb + h * K.sh;
  const uint16_t* v_src = V.p + b * V.sb + h * V.sh;
  if (R.qkv) {
    int64_t pos = *R.pos;
    if (pos < 0 || pos >= R.n_pos) {
      if (tid == 0) set_error(P.err, WGKV_ERR_BAD_POSITION);
      pos = pos < 0 ? 0 : R.n_pos - 1;
    }
    const float c = tid < D ? bf2f(R.cos[pos * D + tid]) : 0.f;
    const float sn = tid < D ? bf2f(R.sin[pos * D + tid]) : 0.f;
    const uint16_t* qkv = R.qkv + b * R.sb;
    const int G = R.Hq / Hk;
    if (blockIdx.y > 0) {  // CTAs 1..G of the head: one query row each
      const int hq = h * G + blockIdx.y - 1;
      norm_rope_row(qkv + int64_t(hq) * D, R.q_norm, R.eps, c, sn, D, xs, part, nullptr,
                    R.q_out + (int64_t(b) * R.Hq + hq) * D);
      return;
    }
    if (tid < D) stage[2][tid] = qkv[int64_t(R.Hq + Hk + h) * D + tid];
    norm_rope_row(qkv + int64_t(R.Hq + h) * D, R.k_norm, R.eps, c, sn, D, xs, part, stage[0], stage[1]);
    k_src = stage[1];
    v_src = stage[2];
    if (!g.w1 && P.local_pre_key) copy_row<false>(P.local_pre_key + row * D, stage[0], D, tid, kDgaThreads);
  }
  // ---- gate input row(s): one warp per input, optional RMS norm, rounded to bf16 ----
  if (g.w1 && warp < g.n_in) {
    const uint16_t* src = R.qkv ? stage[R.sel[warp]] : g.in[warp].p + b * g.in[warp].sb + h * g.in[warp].sh;
    const int per = D / 32;
    float x[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (j < per) x[j] = bf2f(src[lane * per + j]);
    if (g.norm[warp]) {
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) ss += x[j] * x[j];
      for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffff, ss, o);
      const float inv = 1.f / sqrtf(ss / float(D) + g.eps);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (j < per) x[j] = bf16_round(bf2f(g.norm[warp][lane * per + j]) * bf16_round(x[j] * inv));
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (j < per) xs[warp * D + lane * per + j] = x[j];
  }
  // ---- ring append (independent of the gate) ----
  copy_row<false>(P.k + row * D, k_src, D, tid, kDgaThreads);
  copy_row<false>(P.v + row * D, v_src, D, tid, kDgaThreads);
  if (tid == 0 && cache_seqlens) cache_seqlens[i] = cur + P.global_lengths[layer * BH + i];
  if (!g.w1) return;  // deferred gating: the ring is rescored as a whole later
  __syncthreads();
  // ---- hidden layer: a thread per neuron (W1 row read as 16-byte vectors), fp32 dot products ----
  const uint16_t* w1h = g.w1 + int64_t(h) * g.inner * g.I;
  float acc_out = 0.f;
  for (int j = tid; j < g.inner; j += kDgaThreads) {
    const uint4* wr = reinterpret_cast<const uint4*>(w1h + int64_t(j) * g.I);
    const float b1j = bf2f(__ldg(g.b1 + h * g.inner + j)), w2j = bf2f(__ldg(g.w2 + h * g.inner + j));
    float s = 0.f;
    // the row's 16-byte chunks in batches of 8, each batch's loads issued before its FMAs (the
    // products are still summed in element order)
    constexpr int kWB = 8;
    for (int c0 = 0; c0 < g.I / 8; c0 += kWB) {
      uint4 wb[kWB];
#pragma unroll
      for (int u = 0; u < kWB; ++u) wb[u] = c0 + u < g.I / 8 ? __ldg(wr + c0 + u) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int u = 0; u < kWB; ++u) {
        if (c0 + u >= g.I / 8) break;
        const int c = c0 + u;
        const uint32_t ww[4] = {wb[u].x, wb[u].y, wb[u].z, wb[u].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          s = fmaf(xs[c * 8 + 2 * e], __uint_as_float(ww[e] << 16), s);
          s = fmaf(xs[c * 8 + 2 * e + 1], __uint_as_float(ww[e] & 0xffff0000u), s);
        }
      }
    }
    const float hb = gate_hidden(s, b1j, g.act);
    acc_out += bf16_round(act_fn(hb, g.act)) * w2j;
  }
  for (int o = 16; o; o >>= 1) acc_out += __shfl_xor_sync(0xffffffff, acc_out, o);
  if (lane == 0) part[warp] = acc_out;
  __syncthreads();
  if (tid == 0) {
    float o = 0.f;
    for (int w = 0; w < kDgaThreads / 32; ++w) o += part[w];
    const float sc = gate_score(o, bf2f(g.b2[h]), g.act, g.floor);
    P.local_is_global[row] = sc > g.thr ? 1 : 0;  // ring slot `ins` of (layer, b, h)
  }
}

bool pool_ok(const wgkv_pool* P) {
  return P && P->k && P->v && P->block_table && P->global_lengths && P->local_is_global && P->next_free_block &&
         P->layers > 0 && P->batch > 0 && P->kv_heads > 0 && (P->head_dim == 64 || P->head_dim == 128) &&
         P->page > 0 && P->window > 0 && P->window % P->page == 0 && P->total_blocks > 0;
}

// a host ring position, or WGKV_RING_ON_DEVICE with the pool's device copy present
bool ring_pos_ok(const wgkv_pool* P, int pos) {
  return pos == WGKV_RING_ON_DEVICE ? P->ring_state != nullptr : (pos >= 0 && pos < P->window);
}

}  // namespace
}  // namespace wgkv

using namespace wgkv;

// The conv path's clamp floor as torch applies it to a bf16 tensor: g_epsilon rounded to bf16
// (round to nearest even); the fast path has no floor.
static float gate_floor(int act, float score_floor) {
  if (!(act & WGKV_GATE_CONV)) return -INFINITY;
  uint32_t u;
  memcpy(&u, &score_floor, 4);
  if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0x7fffu + ((u >> 16) & 1u)) & 0xffff0000u;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

extern "C" int wgkv_gate_scores(const uint16_t* pre_k, int64_t pk_sb, int64_t pk_sh, int64_t pk_st,
                                const uint16_t* post_k, int64_t k_sb, int64_t k_sh, int64_t k_st,
                                const uint16_t* value, int64_t v_sb, int64_t v_sh, int64_t v_st, int batch,
                                int kv_heads, int seq_len, int head_dim, int input_mask, const uint16_t* w1,
                                const uint16_t* b1, const uint16_t* w2, const uint16_t* b2, const uint16_t* norm_w,
                                float rms_eps, int inner, int act, float score_floor, float threshold,
                                uint16_t* scores, int64_t s_sb,
                                int64_t s_sh, int64_t s_st, uint8_t* mask, int64_t m_sb, int64_t m_sh, int64_t m_st,
                                void* stream) {
  if (batch <= 0 || kv_heads <= 0 || seq_len < 0 || (head_dim != 64 && head_dim != 128)) return WGKV_EINVAL;
  if (inner <= 0 || inner % 8 != 0 || !w1 || !b1 || !w2 || !b2 || (act & ~(WGKV_GATE_SILU | WGKV_GATE_CONV))) return WGKV_EINVAL;
  if (seq_len == 0) return WGKV_OK;
  GateParams p = {};
  const uint16_t* ins[3] = {pre_k, post_k, value};
  const int64_t sbs[3] = {pk_sb, k_sb, v_sb}, shs[3] = {pk_sh, k_sh, v_sh}, sts[3] = {pk_st, k_st, v_st};
  int n = 0;
  for (int s = 0; s < 3; ++s) {
    if (!(input_mask & (1 << s))) continue;
    if (!ins[s] || (reinterpret_cast<uintptr_t>(ins[s]) & 3) || (sbs[s] | shs[s] | sts[s]) & 1) return WGKV_EINVAL;
    p.in[n] = ins[s];
    p.sb[n] = sbs[s];
    p.sh[n] = shs[s];
    p.st[n] = sts[s];
    p.norm[n] = norm_w ? norm_w + s * head_dim : nullptr;
    ++n;
  }
  if (n == 0 || n * head_dim > 384) return WGKV_EINVAL;
  if (reinterpret_cast<uintptr_t>(w1) & 15) return WGKV_EINVAL;
  p.n_in = n;
  p.B = batch;
  p.Hk = kv_heads;
  p.L = seq_len;
  p.D = head_dim;
  p.I = n * head_dim;
  p.inner = inner;
  p.act = act;
  p.w1 = w1;
  p.b1 = b1;
  p.w2 = w2;
  p.b2 = b2;
  p.eps = rms_eps;
  p.thr = threshold;
  p.floor = gate_floor(act, score_floor);
  p.scores = scores;
  p.ssb = s_sb;
  p.ssh = s_sh;
  p.sst = s_st;
  p.mask = mask;
  p.msb = m_sb;
  p.msh = m_sh;
  p.mst = m_st;
  const int RS = p.I + 8;
  const size_t smem = size_t(kGateRows + kGateChunk) * RS * 2 + 2 * kGateChunk * 4;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    if (cudaFuncSetAttribute(gate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) != cudaSuccess)
      return WGKV_ECUDA;
    attr[dev] = true;
  }
  dim3 grid((int64_t(batch) * seq_len + kGateRows - 1) / kGateRows, kv_heads);
  gate_kernel<<<grid, kGateThreads, smem, as_stream(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? WGKV_OK : WGKV_ECUDA;
}

static int nchunks(int n) { return n > 0 ? (n + kChunk - 1) / kChunk : 0; }

extern "C" size_t wgkv_prefill_admit_workspace_size(int batch, int kv_heads, int seq_len) {
  const size_t BH = size_t(batch) * kv_heads;
  return (BH * (nchunks(seq_len) + 2) + 64) * 4;
}

extern "C" int wgkv_prefill_admit(const wgkv_pool* pool, int layer, int seq_len, const uint16_t* k, int64_t k_sb,
                                  int64_t k_sh, int64_t k_st, const uint16_t* v, int64_t v_sb, int64_t v_sh,
                                  int64_t v_st, const uint16_t* pre_k, int64_t pk_sb, int64_t pk_sh, int64_t pk_st,
                                  const uint8_t* g_mask, int64_t m_sb, int64_t m_sh, int64_t m_st, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  if (!pool_ok(pool) || layer < 0 || layer >= pool->layers || seq_len <= 0 || !k || !v || !g_mask || !workspace)
    return WGKV_EINVAL;
  const int BH = pool->batch * pool->kv_heads;
  const int W = pool->window;
  const int n_loc = seq_len < W ? seq_len : W;
  const int n_early = seq_len - W;  // tokens eligible for the global cache
  const int nch = nchunks(n_early);
  if (workspace_bytes < wgkv_prefill_admit_workspace_size(pool->batch, pool->kv_heads, n_early > 0 ? n_early : 0))
    return WGKV_ENOSPC;
  int* counts = reinterpret_cast<int*>(workspace);
  int* totals = counts + size_t(BH) * nch;
  int* first = totals + BH;
  int* okflag = first + BH;
  cudaStream_t s = as_stream(stream);
  MaskView mv{g_mask, m_sb, m_sh, m_st};
  if (nch > 0) {
    chunk_count_kernel<<<dim3(nch, BH), kScanThreads, 0, s>>>(mv, pool->kv_heads, n_early, nch, counts);
  }
  PoolArgs pa{*pool};
  prefill_alloc_kernel<<<1, 1024, 0, s>>>(pa, layer, nch, n_loc, counts, totals, first, okflag);
  const int D = pool->head_dim;
  const bool vec16 = ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
                       reinterpret_cast<uintptr_t>(pre_k)) & 15) == 0 &&
                     ((k_sb | k_sh | k_st | v_sb | v_sh | v_st) % 8 == 0) &&
                     (!pre_k || (pk_sb | pk_sh | pk_st) % 8 == 0);
  if (((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 3) || ((k_sb | k_sh | k_st | v_sb | v_sh | v_st) & 1))
    return WGKV_EINVAL;
  (void)D;
  RowSrc K{k, k_sb, k_sh, k_st}, V{v, v_sb, v_sh, v_st}, PK{pre_k, pk_sb, pk_sh, pk_st};
  dim3 grid(nchunks(seq_len), BH);
  if (vec16)
    prefill_scatter_kernel<true><<<grid, kScanThreads, 0, s>>>(pa, layer, seq_len, n_early, n_loc, nch, mv, K, V, PK,
                                                               counts, first, okflag);
  else
    prefill_scatter_kernel<false><<<grid, kScanThreads, 0, s>>>(pa, layer, seq_len, n_early, n_loc, nch, mv, K, V, PK,
                                                                counts, first, okflag);
  if (pool->quest_min && pool->quest_max && n_early > 0) {
    const int max_pages = (n_early + pool->page - 1) / pool->page;
    quest_bounds_kernel<<<dim3((max_pages + 7) / 8, BH), 256, 0, s>>>(pa, layer, okflag);
  }
  return cudaGetLastError() == cudaSuccess ? WGKV_OK : WGKV_ECUDA;
}

extern "C" int wgkv_promote(const wgkv_pool* pool, int local_ptr, void* stream) {
  if (!pool_ok(pool) || !ring_pos_ok(pool, local_ptr)) return WGKV_EINVAL;
  PoolArgs pa{*pool};
  if (pool->layers * pool->batch * pool->kv_heads > kPromoteThreads * kPromoteMaxPer) return WGKV_EINVAL;
  promote_kernel<<<1, kPromoteThreads, 0, as_stream(stream)>>>(pa, local_ptr);
  if (cudaGetLastError() != cudaSuccess) return WGKV_ECUDA;
  const int N = pool->layers * pool->batch * pool->kv_heads;
  promote_copy_kernel<<<(N + 31) / 32, 256, 0, as_stream(stream)>>>(pa, local_ptr);
  return cudaGetLastError() == cudaSuccess ? WGKV_OK : WGKV_ECUDA;
}

extern "C" int wgkv_ring_advance(const wgkv_pool* pool, void* stream) {
  if (!pool_ok(pool) || !pool->ring_state) return WGKV_EINVAL;
  ring_advance_kernel<<<1, 1, 0, as_stream(stream)>>>(pool->ring_state, pool->window);
  return cudaGetLastError() == cudaSuccess ? WGKV_OK : WGKV_ECUDA;
}

extern "C" int wgkv_decode_append(const wgkv_pool* pool, int layer, int insert_pos, int cur_local_len,
                                  const uint16_t* k_new, int64_t k_sb, int64_t k_sh, const uint16_t* v_new,
                                  int64_t v_sb, int64_t v_sh, const uint16_t* pre_k_new, int64_t pk_sb, int64_t pk_sh,
                                  int32_t* cache_seqlens, void* stream) {
  if (!pool_ok(pool) || layer < 0 || layer >= pool->layers || !ring_pos_ok(pool, insert_pos) || !k_new || !v_new)
    return WGKV_EINVAL;
  if (((reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new) |
        reinterpret_cast<uintptr_t>(pre_k_new)) & 3) || ((k_sb | k_sh | v_sb | v_sh | pk_sb | pk_sh) & 1))
    return WGKV_EINVAL;
  PoolArgs pa{*pool};
  const int BH = pool->batch * pool->kv_heads;
  RowSrc K{k_new, k_sb, k_sh, 0}, V{v_new, v_sb, v_sh, 0}, PK{pre_k_new, pk_sb, pk_sh, 0};
  decode_append_kernel<<<(BH + 7) / 8, 256, 0, as_stream(stream)>>>(pa, layer, insert_pos, cur_local_len, K, V, PK,
                                                                    cache_seqlens);
  return cudaGetLastError() == cudaSuccess ? WGKV_OK : WGKV_ECUDA;
}

extern "C" int wgkv_decode_gate_append(const wgkv_pool* pool, int layer, int insert_pos, int cur_local_len,
                                       const uint16_t* pre_k_new, int64_t pk_sb, int64_t pk_sh,
                                       const uint16_t* k_new, int64_t k_sb, int64_t k_sh, const uint16_t* v_new,
                                       int64_t v_sb, int64_t v_sh, int input_mask, const uint16_t* w1,
                                       const uint16_t* b1, const uint16_t* w2, const uint16_t* b2,
                                       const uint16_t* norm_w, float rms_eps, int inner, int act, float score_floor,
                                       float threshold, int32_t* cache_seqlens, void* stream) {
  if (!pool_ok(pool) || layer < 0 || layer >= pool->layers || !ring_pos_ok(pool, insert_pos) ||
      !k_new || !v_new || !w1 || !b1 || !w2 || !b2 || inner <= 0 ||
      (act & ~(WGKV_GATE_SILU | WGKV_GATE_CONV)))
    return WGKV_EINVAL;
  if (((reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new) |
        reinterpret_cast<uintptr_t>(pre_k_new) | reinterpret_cast<uintptr_t>(w1)) & 3) ||
      ((k_sb | k_sh | v_sb | v_sh | pk_sb | pk_sh) & 1))
    return WGKV_EINVAL;
  const int D = pool->head_dim;
  DecodeGateParams g = {};
  const uint16_t* src[3] = {pre_k_new, k_new, v_new};
  const int64_t sbs[3] = {pk_sb, k_sb, v_sb}, shs[3] = {pk_sh, k_sh, v_sh};
  int n = 0;
  for (int s = 0; s < 3; ++s) {
    if (!(input_mask & (1 << s))) continue;
    if (!src[s]) return WGKV_EINVAL;
    g.in[n] = RowSrc{src[s], sbs[s], shs[s], 0};
    g.norm[n] = norm_w ? norm_w + s * D : nullptr;
    ++n;
  }
  if (n == 0 || n * D > 384 || (n * D) % 8 || (reinterpret_cast<uintptr_t>(w1) & 15)) return WGKV_EINVAL;
  g.n_in = n;
  g.I = n * D;
  g.inner = inner;
  g.act = act;
  g.w1 = w1; g.b1 = b1; g.w2 = w2; g.b2 = b2;
  g.eps = rms_eps;
  g.thr = threshold;
  g.floor = gate_floor(act, score_floor);
  PoolArgs pa{*pool};
  RowSrc K{k_new, k_sb, k_sh, 0}, V{v_new, v_sb, v_sh, 0};
  const int BH = pool->batch * pool->kv_heads;
  if (launch_pdl(decode_gate_append_kernel, dim3(BH), dim3(kDgaThreads), 0, as_stream(stream), pa, g, RopeParams{},
                 layer, insert_pos, cur_local_len, K, V, cache_seqlens) != cudaSuccess)
    return WGKV_ECUDA;
  return WGKV_OK;
}

extern "C" int wgkv_decode_prologue(const wgkv_pool* pool, int layer, int insert_pos, int cur_local_len,
                                    const uint16_t* qkv, int64_t qkv_sb, int q_heads, const uint16_t* q_norm,
                                    const uint16_t* k_norm, float qk_eps, const uint16_t* rope_cos,
                                    const uint16_t* rope_sin, const int64_t* position, int64_t n_positions,
                                    uint16_t* q_out, int input_mask, const uint16_t* w1, const uint16_t* b1,
                                    const uint16_t* w2, const uint16_t* b2, const uint16_t* norm_w, float rms_eps,
                                    int inner, int act, float score_floor, float threshold, int32_t* cache_seqlens,
                                    void* stream) {
  if (!pool_ok(pool) || layer < 0 || layer >= pool->layers || !ring_pos_ok(pool, insert_pos) || !qkv || !rope_cos ||
      !rope_sin || !position || n_positions <= 0 || !q_out || q_heads <= 0 || q_heads % pool->kv_heads)
    return WGKV_EINVAL;
  const int D = pool->head_dim;
  if (qkv_sb < int64_t(q_heads + 2 * pool->kv_heads) * D) return WGKV_EINVAL;
  DecodeGateParams g = {};
  RopeParams R = {};
  R.qkv = qkv;
  R.sb = qkv_sb;
  R.Hq = q_heads;
  R.q_norm = q_norm;
  R.k_norm = k_norm;
  R.eps = qk_eps;
  R.cos = rope_cos;
  R.sin = rope_sin;
  R.pos = position;
  R.n_pos = n_positions;
  R.q_out = q_out;
  if (w1) {
    if (!b1 || !w2 || !b2 || inner <= 0 || (act & ~(WGKV_GATE_SILU | WGKV_GATE_CONV)) ||
        (reinterpret_cast<uintptr_t>(w1) & 15))
      return WGKV_EINVAL;
    int n = 0;
    for (int s = 0; s < 3; ++s) {
      if (!(input_mask & (1 << s))) continue;
      R.sel[n] = s;
      g.norm[n] = norm_w ? norm_w + s * D : nullptr;
      ++n;
    }
    if (n == 0 || n * D > 384 || (n * D) % 8) return WGKV_EINVAL;
    g.n_in = n;
    g.I = n * D;
    g.inner = inner;
    g.act = act;
    g.w1 = w1; g.b1 = b1; g.w2 = w2; g.b2 = b2;
    g.eps = rms_eps;
    g.thr = threshold;
    g.floor = gate_floor(act, score_floor);
  }
  PoolArgs pa{*pool};
  const int BH = pool->batch * pool->kv_heads;
  // one CTA per (b, h) for the key, gate and append, plus one per query head of the group
  if (launch_pdl(decode_gate_append_kernel, dim3(BH, 1 + q_heads / pool->kv_heads), dim3(kDgaThreads), 0,
                 as_stream(stream), pa, g, R, layer, insert_pos, cur_local_len, RowSrc{}, RowSrc{},
                 cache_seqlens) != cudaSuccess)
    return WGKV_ECUDA;
  return WGKV_OK;
}
