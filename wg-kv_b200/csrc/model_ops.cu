// Plumbing of the decoder around the WG-KV attention path (the end-to-end driver):
// * RMSNorm and SiLU(gate) * up, one launch each, with the bf16 roundings of the torch expressions
//     (x.float() * rsqrt(mean(x^2) + eps)).to(bf16) * w        (LlamaRMSNorm / Qwen3RMSNorm)
//     silu(gate).to(bf16) * up                                  (LlamaMLP / Qwen3MLP act_fn(gate) * up)
//   HBM-bound streams over rows; 16-byte vector loads, one CTA per row.
// * Skinny GEMM y = x W^T (+ residual) for the decode step's few rows (m <= 8): a weight-streaming
//   kernel (every weight byte read once, 16-byte loads, several in flight per lane) that the
//   library GEMMs do not reach at m = 1 on these shapes.
#include "common.cuh"
#include "runtime.h"

namespace wgkv {
namespace {

constexpr int kRowThreads = 256;

WGKV_DEV uint4 pack8(const float* f) {
  uint4 u;
  u.x = pack_bf16x2(f[0], f[1]);
  u.y = pack_bf16x2(f[2], f[3]);
  u.z = pack_bf16x2(f[4], f[5]);
  u.w = pack_bf16x2(f[6], f[7]);
  return u;
}

// cols % 8 == 0, cols <= 8 * kRowThreads * kMaxVec
constexpr int kMaxVec = 4;

__global__ void __launch_bounds__(kRowThreads) rms_norm_kernel(const uint16_t* x, int64_t xs, const uint16_t* w,
                                                               int cols, float eps, uint16_t* out, int64_t os) {
  const int r = blockIdx.x, tid = threadIdx.x;
  griddep_launch();
  griddep_wait();
  const uint4* src = reinterpret_cast<const uint4*>(x + int64_t(r) * xs);
  const int nv = cols / 8;
  float v[kMaxVec][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxVec; ++k) {
    const int c = tid + k * kRowThreads;
    if (c < nv) {
      unpack8(src[c], v[k]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[k][e] * v[k][e];
    }
  }
  __shared__ float red[kRowThreads / 32];
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffff, ss, o);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kRowThreads / 32; ++i) tot += red[i];
  const float inv = rsqrtf(tot / float(cols) + eps);
  uint4* dst = reinterpret_cast<uint4*>(out + int64_t(r) * os);
  const uint4* wv = reinterpret_cast<const uint4*>(w);
#pragma unroll
  for (int k = 0; k < kMaxVec; ++k) {
    const int c = tid + k * kRowThreads;
    if (c < nv) {
      float g[8], y[8];
      unpack8(__ldg(wv + c), g);
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = bf16_round(v[k][e] * inv) * g[e];
      dst[c] = pack8(y);
    }
  }
}

// gu row = [gate (inter) | up (inter)]
__global__ void __launch_bounds__(kRowThreads) silu_mul_kernel(const uint16_t* gu, int64_t gs, int rows,
                                                               int inter, uint16_t* out, int64_t os) {
  const int c = blockIdx.x * kRowThreads + threadIdx.x;
  griddep_launch();
  griddep_wait();
  if (c >= inter / 8) return;
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    const uint4* g4 = reinterpret_cast<const uint4*>(gu + r * gs);
    float g[8], u[8], y[8];
    unpack8(g4[c], g);
    unpack8(g4[inter / 8 + c], u);
#pragma unroll
    for (int e = 0; e < 8; ++e) y[e] = bf16_round(g[e] / (1.f + expf(-g[e]))) * u[e];
    reinterpret_cast<uint4*>(out + r * os)[c] = pack8(y);
  }
}

// ---------------------------------------------------------------------------------------------
// skinny GEMM: block = 8 warps over `rpb` weight rows; the 8 / rpb warps of a row split K.
// Every lane issues all the 16-byte weight loads of one pass (kSgUnroll, predicated) before using
// them, so short rows cost one memory round trip.
constexpr int kSgWarps = 8;
constexpr int kSgUnroll = 8;

// x rows as the GEMM sees them: plain, or RMS-normalised on the fly (norm_w != NULL) with the
// roundings of rms_norm_kernel, bf16(bf16(x * inv) * w)
template <int M>
struct XRows {
  const uint16_t* x;
  int64_t xs;
  const uint16_t* norm_w;
  const float* inv;  // [M] in shared memory when norm_w is set

  WGKV_DEV void load(int m, int c, float* xf) const {
    unpack8(__ldg(reinterpret_cast<const uint4*>(x + m * xs) + c), xf);
    if (norm_w) {
      float g[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(norm_w) + c), g);
#pragma unroll
      for (int e = 0; e < 8; ++e) xf[e] = bf16_round(bf16_round(xf[e] * inv[m]) * g[e]);
    }
  }
};

// inv[m] = rsqrt(mean(x[m]^2) + eps) of the M rows, block-wide (every thread of the block calls it)
template <int M>
WGKV_DEV void block_rms_inv(const uint16_t* x, int64_t xs, int k, float eps, float* inv) {
  __shared__ float red[kSgWarps][M];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int m = 0; m < M; ++m) {
    float ss = 0.f;
    for (int c = threadIdx.x; c < k / 8; c += kSgWarps * 32) {
      float f[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(x + m * xs) + c), f);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
    }
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffff, ss, o);
    if (lane == 0) red[warp][m] = ss;
  }
  __syncthreads();
  if (threadIdx.x < M) {
    float t = 0.f;
    for (int w = 0; w < kSgWarps; ++w) t += red[w][threadIdx.x];
    inv[threadIdx.x] = rsqrtf(t / float(k) + eps);
  }
  __syncthreads();
}

// acc[m] += sum over chunks [c, c1) of this lane (stride 32) of x[m] . w_row; wv holds the first pass
template <int M>
WGKV_DEV void dot_rows(const uint4* wr, int cfirst, int c1, const XRows<M>& X, uint4 (&wv)[kSgUnroll],
                       bool preloaded, float (&acc)[M]) {
  for (int cb = cfirst; cb < c1; cb += 32 * kSgUnroll) {
    if (!preloaded || cb != cfirst) {
#pragma unroll
      for (int u = 0; u < kSgUnroll; ++u)
        wv[u] = cb + 32 * u < c1 ? __ldcs(wr + cb + 32 * u) : make_uint4(0, 0, 0, 0);  // streamed once
    }
#pragma unroll
    for (int u = 0; u < kSgUnroll; ++u) {
      const int c = cb + 32 * u;
      if (c >= c1) break;
      float wf[8];
      unpack8(wv[u], wf);
#pragma unroll
      for (int m = 0; m < M; ++m) {
        float xf[8];
        X.load(m, c, xf);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[m] = fmaf(xf[e], wf[e], acc[m]);
      }
    }
  }
}

template <int M>
__global__ void __launch_bounds__(kSgWarps * 32) skinny_gemm_kernel(const uint16_t* __restrict__ x, int64_t xs,
                                                                    const uint16_t* __restrict__ w, int n, int k,
                                                                    int rpb, void* y, int64_t ys, int out_f32,
                                                                    const uint16_t* res, int64_t rs,
                                                                    const uint16_t* norm_w, float eps) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ks = kSgWarps / rpb;          // warps per row
  const int row_in = warp % rpb, slice = warp / rpb;
  const int row = blockIdx.x * rpb + row_in;
  const int kc = k / 8;                   // 16-byte chunks per row
  const int per = (kc + ks - 1) / ks;     // chunks per slice
  const int c0 = slice * per, c1 = min(kc, c0 + per);
  __shared__ float inv[M];
  float acc[M];
#pragma unroll
  for (int m = 0; m < M; ++m) acc[m] = 0.f;
  griddep_launch();
  const uint4* wr = reinterpret_cast<const uint4*>(w + int64_t(min(row, n - 1)) * k);
  // the first pass of weight loads does not depend on the previous kernel: issue it before waiting
  uint4 wv[kSgUnroll];
#pragma unroll
  for (int u = 0; u < kSgUnroll; ++u) {
    const int c = c0 + lane + 32 * u;
    wv[u] = row < n && c < c1 ? __ldcs(wr + c) : make_uint4(0, 0, 0, 0);
  }
  griddep_wait();
  if (norm_w) block_rms_inv<M>(x, xs, k, eps, inv);
  const XRows<M> X{x, xs, norm_w, inv};
  if (row < n) dot_rows<M>(wr, c0 + lane, c1, X, wv, true, acc);
#pragma unroll
  for (int m = 0; m < M; ++m)
    for (int o = 16; o; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffff, acc[m], o);
  __shared__ float part[kSgWarps][M];
  if (lane == 0) {
#pragma unroll
    for (int m = 0; m < M; ++m) part[warp][m] = acc[m];
  }
  __syncthreads();
  // one thread per (row, m) sums the K slices of its row
  const int t = threadIdx.x;
  if (t < rpb * M) {
    const int ri = t % rpb, m = t / rpb;
    const int r = blockIdx.x * rpb + ri;
    if (r < n) {
      float v = 0.f;
      for (int s2 = 0; s2 < ks; ++s2) v += part[s2 * rpb + ri][m];
      if (res) v += bf2f(res[m * rs + r]);
      if (out_f32) reinterpret_cast<float*>(y)[m * ys + r] = v;
      else reinterpret_cast<uint16_t*>(y)[m * ys + r] = f2bf(v);
    }
  }
}

// Many rows (n >= 8 * 4 * SMs, or paired): persistent warps, one output row at a time, grid-stride;
// no block barrier after the optional RMS prologue.  paired: w holds [gate (n/2 rows) | up (n/2
// rows)] and output j = bf16(bf16(silu(bf16(g_j))) * bf16(u_j)) -- the MLP activation of
// silu_mul_kernel fused into its projection.
template <int M>
__global__ void __launch_bounds__(kSgWarps * 32) skinny_rows_kernel(const uint16_t* __restrict__ x, int64_t xs,
                                                                    const uint16_t* __restrict__ w, int n, int k,
                                                                    void* y, int64_t ys, int out_f32,
                                                                    const uint16_t* res, int64_t rs,
                                                                    const uint16_t* norm_w, float eps, int paired) {
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * kSgWarps + (threadIdx.x >> 5), nw = gridDim.x * kSgWarps;
  const int kc = k / 8;
  const int n_out = paired ? n / 2 : n;
  __shared__ float inv[M];
  griddep_launch();
  uint4 wv[kSgUnroll];
  {  // the first row's first pass of weight loads goes out before waiting for the previous kernel
    const uint4* wr = reinterpret_cast<const uint4*>(w + int64_t(min(gw, n_out - 1)) * k);
#pragma unroll
    for (int u = 0; u < kSgUnroll; ++u) {
      const int c = lane + 32 * u;
      wv[u] = gw < n_out && c < kc ? __ldcs(wr + c) : make_uint4(0, 0, 0, 0);
    }
  }
  griddep_wait();
  if (norm_w) block_rms_inv<M>(x, xs, k, eps, inv);
  const XRows<M> X{x, xs, norm_w, inv};
  for (int row = gw; row < n_out; row += nw) {
    float acc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = 0.f;
    dot_rows<M>(reinterpret_cast<const uint4*>(w + int64_t(row) * k), lane, kc, X, wv, row == gw, acc);
#pragma unroll
    for (int m = 0; m < M; ++m)
      for (int o = 16; o; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffff, acc[m], o);
    if (paired) {
      float up[M];
#pragma unroll
      for (int m = 0; m < M; ++m) up[m] = 0.f;
      dot_rows<M>(reinterpret_cast<const uint4*>(w + int64_t(row + n_out) * k), lane, kc, X, wv, false, up);
#pragma unroll
      for (int m = 0; m < M; ++m) {
        float u = up[m];
        for (int o = 16; o; o >>= 1) u += __shfl_xor_sync(0xffffffff, u, o);
        const float g = bf16_round(acc[m]);
        acc[m] = bf16_round(g / (1.f + expf(-g))) * bf16_round(u);
      }
    }
#pragma unroll
    for (int m = 0; m < M; ++m) {
      if (lane == m) {
        float v = acc[m];
        if (res) v += bf2f(res[m * rs + row]);
        if (out_f32) reinterpret_cast<float*>(y)[m * ys + row] = v;
        else reinterpret_cast<uint16_t*>(y)[m * ys + row] = f2bf(v);
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------
// greedy token: argmax of each fp32 logits row (first index on ties, as torch.argmax); one launch,
// chunk partials per CTA, the last CTA of a row (atomic ticket, reset for the next call) finishes.
constexpr int kAmThreads = 256;
constexpr int kAmChunk = 4096;

WGKV_DEV void am_better(float& v, int& i, float v2, int i2) {
  if (v2 > v || (v2 == v && i2 < i)) { v = v2; i = i2; }
}

__global__ void __launch_bounds__(kAmThreads) argmax_kernel(const float* x, int64_t xs, int n, float* pv, int* pi,
                                                           int* ticket, int64_t* out, int64_t os) {
  const int r = blockIdx.y, c = blockIdx.x, nc = gridDim.x, tid = threadIdx.x;
  griddep_launch();
  griddep_wait();
  const float* row = x + int64_t(r) * xs;
  float v = -INFINITY;
  int i = 0x7fffffff;
  for (int j = c * kAmChunk + tid; j < min(n, (c + 1) * kAmChunk); j += kAmThreads) am_better(v, i, row[j], j);
  for (int o = 16; o; o >>= 1) am_better(v, i, __shfl_xor_sync(0xffffffff, v, o), __shfl_xor_sync(0xffffffff, i, o));
  __shared__ float sv[kAmThreads / 32];
  __shared__ int si[kAmThreads / 32];
  __shared__ int s_last;
  if ((tid & 31) == 0) { sv[tid >> 5] = v; si[tid >> 5] = i; }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < kAmThreads / 32; ++w) am_better(v, i, sv[w], si[w]);
    pv[int64_t(r) * nc + c] = v;
    pi[int64_t(r) * nc + c] = i;
    __threadfence();
    const int t = atomicAdd(&ticket[r], 1);
    s_last = t == nc - 1;
    if (s_last) ticket[r] = 0;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  v = -INFINITY;
  i = 0x7fffffff;
  for (int k = tid; k < nc; k += kAmThreads) am_better(v, i, __ldcg(pv + int64_t(r) * nc + k), __ldcg(pi + int64_t(r) * nc + k));
  for (int o = 16; o; o >>= 1) am_better(v, i, __shfl_xor_sync(0xffffffff, v, o), __shfl_xor_sync(0xffffffff, i, o));
  if ((tid & 31) == 0) { sv[tid >> 5] = v; si[tid >> 5] = i; }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < kAmThreads / 32; ++w) am_better(v, i, sv[w], si[w]);
    out[int64_t(r) * os] = i;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace wgkv

using namespace wgkv;

extern "C" int wgkv_rms_norm(const uint16_t* x, int64_t x_stride, const uint16_t* weight, int rows, int cols,
                             float eps, uint16_t* out, int64_t out_stride, void* stream) {
  if (!x || !weight || !out || rows < 0 || cols <= 0 || cols % 8 || cols > 8 * kRowThreads * kMaxVec ||
      x_stride % 8 || out_stride % 8 || !aligned16(x) || !aligned16(weight) || !aligned16(out))
    return WGKV_EINVAL;
  if (rows == 0) return WGKV_OK;
  if (launch_pdl(rms_norm_kernel, dim3(rows), dim3(kRowThreads), 0, static_cast<cudaStream_t>(stream), x, x_stride,
                 weight, cols, eps, out, out_stride) != cudaSuccess)
    return WGKV_ECUDA;
  return WGKV_OK;
}

extern "C" int wgkv_silu_mul(const uint16_t* gate_up, int64_t gu_stride, int rows, int inter, uint16_t* out,
                             int64_t out_stride, void* stream) {
  if (!gate_up || !out || rows < 0 || inter <= 0 || inter % 8 || gu_stride % 8 || out_stride % 8 ||
      !aligned16(gate_up) || !aligned16(out))
    return WGKV_EINVAL;
  if (rows == 0) return WGKV_OK;
  dim3 grid((inter / 8 + kRowThreads - 1) / kRowThreads, rows < 65535 ? rows : 65535);
  if (launch_pdl(silu_mul_kernel, grid, dim3(kRowThreads), 0, static_cast<cudaStream_t>(stream), gate_up, gu_stride,
                 rows, inter, out, out_stride) != cudaSuccess)
    return WGKV_ECUDA;
  return WGKV_OK;
}

extern "C" int wgkv_skinny_gemm(const uint16_t* x, int64_t x_stride, int m, const uint16_t* w, int n, int k, void* y,
                                int64_t y_stride, int out_f32, const uint16_t* residual, int64_t r_stride,
                                const uint16_t* rms_weight, float rms_eps, int paired, void* stream) {
  if (!x || !w || !y || m <= 0 || m > 8 || n <= 0 || k <= 0 || k % 8 || x_stride % 8 || !aligned16(x) ||
      !aligned16(w) || (residual && out_f32) || (rms_weight && !aligned16(rms_weight)))
    return WGKV_EINVAL;
  if (paired && (n % 2 || out_f32 || residual)) return WGKV_EINVAL;
  const int sms = device_sms();
  if (sms <= 0) return WGKV_ECUDA;
  // rows per block: as many as keep >= 4 blocks per SM; the block's other warps split K
  int rpb = 1;
  while (rpb < kSgWarps && int64_t(n) / (rpb * 2) >= 4 * sms) rpb *= 2;
  const bool rows = paired || (rpb == kSgWarps && int64_t(n) >= int64_t(kSgWarps) * 8 * sms);
  const int blocks = rows ? 8 * sms : (n + rpb - 1) / rpb;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
#define WGKV_SG(MM)                                                                                            \
  e = rows ? launch_pdl(skinny_rows_kernel<MM>, dim3(blocks), dim3(kSgWarps * 32), 0, s, x, x_stride, w, n, k, y,  \
                        y_stride, out_f32, residual, r_stride, rms_weight, rms_eps, paired)                     \
           : launch_pdl(skinny_gemm_kernel<MM>, dim3(blocks), dim3(kSgWarps * 32), 0, s, x, x_stride, w, n, k,     \
                        rpb, y, y_stride, out_f32, residual, r_stride, rms_weight, rms_eps)
  switch (m) {
    case 1: WGKV_SG(1); break;
    case 2: WGKV_SG(2); break;
    case 3: WGKV_SG(3); break;
    case 4: WGKV_SG(4); break;
    case 5: WGKV_SG(5); break;
    case 6: WGKV_SG(6); break;
    case 7: WGKV_SG(7); break;
    default: WGKV_SG(8); break;
  }
#undef WGKV_SG
  return e == cudaSuccess ? WGKV_OK : WGKV_ECUDA;
}

extern "C" size_t wgkv_argmax_workspace_size(int rows, int n) {
  const size_t nc = (size_t(n) + kAmChunk - 1) / kAmChunk;
  return size_t(rows) * (nc * 8 + 4) + 256;
}

extern "C" int wgkv_argmax(const float* logits, int64_t row_stride, int rows, int n, int64_t* out, int64_t out_stride,
                           void* workspace, size_t workspace_bytes, void* stream) {
  if (!logits || !out || !workspace || rows <= 0 || n <= 0 || rows > 65535) return WGKV_EINVAL;
  if (workspace_bytes < wgkv_argmax_workspace_size(rows, n)) return WGKV_ENOSPC;
  const int nc = (n + kAmChunk - 1) / kAmChunk;
  int* ticket = static_cast<int*>(workspace);  // rows ints, zero before the first call, left zero
  float* pv = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + ((size_t(rows) * 4 + 255) & ~size_t(255)));
  int* pi = reinterpret_cast<int*>(pv + size_t(rows) * nc);
  if (launch_pdl(argmax_kernel, dim3(nc, rows), dim3(kAmThreads), 0, static_cast<cudaStream_t>(stream), logits,
                 row_stride, n, pv, pi, ticket, out, out_stride) != cudaSuccess)
    return WGKV_ECUDA;
  return WGKV_OK;
}
