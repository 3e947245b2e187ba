// Vertical-slash sparse indices on the device (sm_100a).
//
// Reference: generate_sparse_indices (src/modeling_layers.py:385-409),
// generate_block_offset (:321-349) and generate_column_index (:352-381).  The
// reference builds column_index with a per-(b, h) torch.nonzero loop and a
// .item() sync for Gmax; here the admitted positions are stream-compacted
// per 2048-token chunk (count -> per-head scan -> scatter) with no host sync,
// and Gmax is reduced with an atomicMax into a device word.
#include "common.cuh"
#include "runtime.h"

namespace wgkv {
namespace {

// exclusive scan of each head's chunk counts, in place
__global__ void __launch_bounds__(32) idx_scan_kernel(int nch, int* counts) {
  const int bh = blockIdx.x, lane = threadIdx.x;
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
}

struct IdxOut {
  int32_t* bc;
  int32_t* bo;
  int32_t* cc;
  int32_t* ci;
  int64_t ci_stride;
  int32_t* max_count;
};

__global__ void __launch_bounds__(kScanThreads) idx_scatter_kernel(MaskView mv, int Hk, int L, int W, int blk, int nch,
                                                                   const int* counts, IdxOut o) {
  const int bh = blockIdx.y, b = bh / Hk, h = bh - b * Hk, c = blockIdx.x;
  const int R = (L + blk - 1) / blk;
  const int P = min(W / blk, R);
  __shared__ int wsum[kScanThreads / 32];

  // band tables (shared by every head): written by the bh == 0 row of CTAs
  if (bh == 0) {
    const int M = P + 1;
    for (int e = c * kScanThreads + threadIdx.x; e < R * M; e += nch * kScanThreads) {
      const int i = e / M, col = e - i * M;
      o.bo[e] = i < P ? (col < P ? blk * col : 0) : 1 + blk * (i - P + col);
      if (col == 0) {
        int cnt = i < P ? i + 1 : P + 1;
        if (i == R - 1) {
          const int start = max(0, (R - 1) * blk - W + 1);
          cnt = (L - start + blk - 1) / blk;  // len(range(start, L, blk))
        }
        o.bc[i] = cnt;
      }
    }
  }
  if (c == 0)
    for (int i = threadIdx.x; i < P; i += kScanThreads) o.cc[int64_t(bh) * R + i] = 0;

  const int t0 = c * kChunk + threadIdx.x * 8;
  uint8_t mk[8];
  int n = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    mk[j] = (t0 + j < L) ? mv.at(b, h, t0 + j) : 0;
    n += mk[j] ? 1 : 0;
  }
  int tot;
  const int excl = block_excl_scan<kScanThreads>(n, wsum, tot);
  const int base = counts[bh * nch + c] + excl;  // #admitted < t0
  int32_t* ci = o.ci + int64_t(bh) * o.ci_stride;
  int r = base;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (mk[j]) ci[r++] = t0 + j;
  // column_count[i] = #admitted < blk*(i-P) + 1, for the block starts x = blk*(i-P) in this thread's tokens
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int x = t0 + j;
    if (x < L && x % blk == 0) {
      int before = base;
      for (int q = 0; q < j; ++q) before += mk[q] ? 1 : 0;
      const int val = before + (mk[j] ? 1 : 0);
      const int i = x / blk + P;
      if (i < R) o.cc[int64_t(bh) * R + i] = val;
      if (x == blk * ((L - 1) / blk) && o.max_count) atomicMax(o.max_count, val);
    }
  }
}

}  // namespace
}  // namespace wgkv

using namespace wgkv;

extern "C" size_t wgkv_sparse_indices_workspace_size(int batch, int kv_heads, int seq_len) {
  return (size_t(batch) * kv_heads * ((seq_len + kChunk - 1) / kChunk) + 64) * 4;
}

extern "C" int wgkv_sparse_indices(const uint8_t* g_mask, int64_t m_sb, int64_t m_sh, int64_t m_st, int batch,
                                   int kv_heads, int seq_len, int window, int block, int32_t* block_count,
                                   int32_t* block_offset, int32_t* column_count, int32_t* column_index,
                                   int64_t ci_stride, int32_t* max_count, void* workspace, size_t workspace_bytes,
                                   void* stream) {
  if (!g_mask || batch <= 0 || kv_heads <= 0 || seq_len <= 0 || block <= 0 || block % 8 != 0 ||
      kChunk % block != 0 || window < 0 || window % block != 0 || ci_stride < seq_len || !block_count ||
      !block_offset || !column_count || !column_index || !workspace)
    return WGKV_EINVAL;
  if (workspace_bytes < wgkv_sparse_indices_workspace_size(batch, kv_heads, seq_len)) return WGKV_ENOSPC;
  const int BH = batch * kv_heads;
  const int nch = (seq_len + kChunk - 1) / kChunk;
  int* counts = reinterpret_cast<int*>(workspace);
  cudaStream_t s = as_stream(stream);
  MaskView mv{g_mask, m_sb, m_sh, m_st};
  chunk_count_kernel<<<dim3(nch, BH), kScanThreads, 0, s>>>(mv, kv_heads, seq_len, nch, counts);
  idx_scan_kernel<<<BH, 32, 0, s>>>(nch, counts);
  IdxOut o{block_count, block_offset, column_count, column_index, ci_stride, max_count};
  idx_scatter_kernel<<<dim3(nch, BH), kScanThreads, 0, s>>>(mv, kv_heads, seq_len, window, block, nch, counts, o);
  return cudaGetLastError() == cudaSuccess ? WGKV_OK : WGKV_ECUDA;
}
