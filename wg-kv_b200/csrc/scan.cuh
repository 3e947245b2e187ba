// Chunked mask counting and block scans shared by the compaction kernels.
#pragma once
#include "common.cuh"

namespace wgkv {
namespace {

constexpr int kChunk = 2048;       // tokens per counting / scatter CTA
constexpr int kScanThreads = 256;  // 8 tokens per thread

struct MaskView {
  const uint8_t* m;
  int64_t sb, sh, st;
  WGKV_DEV uint8_t at(int b, int h, int t) const { return m[b * sb + h * sh + int64_t(t) * st]; }
};

// counts[bh * nch + c] = #admitted tokens of (b, h) in chunk c of [0, limit)
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


}  // namespace
}  // namespace wgkv
