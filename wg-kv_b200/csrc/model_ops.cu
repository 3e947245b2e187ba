// Element-wise plumbing of the decoder around the WG-KV attention path (the end-to-end driver):
// RMSNorm and SiLU(gate) * up, one launch each, with the bf16 roundings of the torch expressions
//   (x.float() * rsqrt(mean(x^2) + eps)).to(bf16) * w          (LlamaRMSNorm / Qwen3RMSNorm)
//   silu(gate).to(bf16) * up                                    (LlamaMLP / Qwen3MLP act_fn(gate) * up)
// Both are HBM-bound streams over rows; 16-byte vector loads, one CTA per row.
#include "common.cuh"

namespace wgkv {
namespace {

constexpr int kRowThreads = 256;

WGKV_DEV void unpack8(const uint4& u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    f[2 * e] = __uint_as_float(w[e] << 16);
    f[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
  }
}

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
  rms_norm_kernel<<<rows, kRowThreads, 0, static_cast<cudaStream_t>(stream)>>>(x, x_stride, weight, cols, eps, out,
                                                                                out_stride);
  return cudaGetLastError() == cudaSuccess ? WGKV_OK : WGKV_ECUDA;
}

extern "C" int wgkv_silu_mul(const uint16_t* gate_up, int64_t gu_stride, int rows, int inter, uint16_t* out,
                             int64_t out_stride, void* stream) {
  if (!gate_up || !out || rows < 0 || inter <= 0 || inter % 8 || gu_stride % 8 || out_stride % 8 ||
      !aligned16(gate_up) || !aligned16(out))
    return WGKV_EINVAL;
  if (rows == 0) return WGKV_OK;
  dim3 grid((inter / 8 + kRowThreads - 1) / kRowThreads, rows < 65535 ? rows : 65535);
  silu_mul_kernel<<<grid, kRowThreads, 0, static_cast<cudaStream_t>(stream)>>>(gate_up, gu_stride, rows, inter, out,
                                                                                out_stride);
  return cudaGetLastError() == cudaSuccess ? WGKV_OK : WGKV_ECUDA;
}
