// Shared device helpers for the WG-KV sm_100a kernels: mbarriers, TMA
// (cp.async.bulk.tensor, never with .multicast), ldmatrix, mma.sync, bf16.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include "../../include/wgkv.h"

#define WGKV_DEV __device__ __forceinline__

namespace wgkv {

WGKV_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

WGKV_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

WGKV_DEV void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

WGKV_DEV void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

WGKV_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

WGKV_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

WGKV_DEV uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait on the phase with the given parity: gives up (returns false)
// after about kWaitLimitNs of wall time, so a broken pipeline ends the kernel
// with an error status instead of hanging the GPU.
constexpr uint64_t kWaitLimitNs = 2000000000ull;
WGKV_DEV bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  uint64_t t0 = 0;
  for (long long i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 255) == 0) {
      const uint64_t now = global_ns();
      if (i == 0) t0 = now;
      else if (now - t0 > kWaitLimitNs) return false;
    }
  }
}

// 2D tiled TMA load (no multicast) of box {x, y} into shared memory.
WGKV_DEV void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 3D tiled TMA load (no multicast) of box {x, y, z} into shared memory.
WGKV_DEV void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

WGKV_DEV void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Untiled bulk copy global -> shared (both 16-byte aligned, size % 16 == 0).
WGKV_DEV void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

WGKV_DEV void ldmatrix_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

WGKV_DEV void ldmatrix_x4_trans(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D = A(16x16, row) * B(16x8, col) + D, bf16 inputs, fp32 accumulate.
WGKV_DEV void mma_bf16_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

WGKV_DEV uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

WGKV_DEV float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

WGKV_DEV float bf2f(uint16_t v) { return __uint_as_float(uint32_t(v) << 16); }

// the 8 bf16 values of a 16-byte vector as floats
WGKV_DEV void unpack8(const uint4& u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    f[2 * e] = __uint_as_float(w[e] << 16);
    f[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
  }
}

// bf16 bit pattern of x (round to nearest even)
WGKV_DEV uint16_t f2bf(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }

// Byte offset of 16-byte chunk `chunk` (0..7) of row `row` inside a tile
// written by TMA with CU_TENSOR_MAP_SWIZZLE_128B (128-byte rows, tile base
// 1024-byte aligned): the chunk index is XORed with row % 8.
WGKV_DEV uint32_t swz128(uint32_t row, uint32_t chunk) { return row * 128u + ((chunk ^ (row & 7u)) << 4); }

// Programmatic dependent launch: a kernel launched with launch_pdl may start while the previous
// kernel of the stream finishes; it must call griddep_wait() before touching anything that kernel
// writes (or reads and it overwrites).  griddep_launch() lets the next kernel start early.
WGKV_DEV void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
WGKV_DEV void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Programmatic dependent launch is opt-in (WGKV_PDL=1 in the environment): it won little at batch 1
// on the Llama-3.2-1B decoder step and cost 13 % on the Llama-3.1-8B step (4.10 -> 4.70 ms), whose
// projections run many waves.  Without it griddepcontrol is a no-op and the kernels run in stream order.
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("WGKV_PDL");
    return e && e[0] == '1';
  }();
  return on;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Exclusive block-wide prefix sum of one int per thread of a kThreads-thread block (warp shuffles,
// then the warp totals); the block total comes back in `total`.  Every thread must call it; wsum
// holds kThreads / 32 ints of shared memory and is free again on return.
template <int kThreads>
WGKV_DEV int block_excl_scan(int v, int* wsum, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffff, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[warp] = x;
  __syncthreads();
  int base = 0;
  total = 0;
  for (int w = 0; w < kThreads / 32; ++w) {
    if (w < warp) base += wsum[w];
    total += wsum[w];
  }
  __syncthreads();
  return base + x - v;
}

// Radix-select step, run by one whole warp: walking the 256 bins of `hist` from the top (kDesc) or
// the bottom, the bin that holds the need-th key and how many keys of it are still to take
// (*take = need - keys in the bins before it).  Lane l sums 8 consecutive bins of the walk, a warp
// scan finds the lane, that lane walks its 8 bins.  Past the end it stops at the last bin.
template <bool kDesc>
WGKV_DEV void warp_pick_bin(const int* hist, int need, int* bin_out, int* take_out) {
  const int lane = threadIdx.x & 31;
  int c[8], sum = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    c[i] = hist[kDesc ? 255 - (lane * 8 + i) : lane * 8 + i];
    sum += c[i];
  }
  int incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffff, incl, o);
    if (lane >= o) incl += y;
  }
  const unsigned hit = __ballot_sync(0xffffffff, incl >= need);
  const int L = hit ? __ffs(hit) - 1 : 31;
  if (lane == L) {
    int acc = incl - sum, i = 0;
    for (; i < 7; ++i) {
      if (acc + c[i] >= need) break;
      acc += c[i];
    }
    *bin_out = kDesc ? 255 - (lane * 8 + i) : lane * 8 + i;
    *take_out = need - acc;
  }
}

WGKV_DEV void set_error(int* err, int code) {
  if (err) atomicOr(err, code);
}

// ---- chunked mask counting shared by the compaction kernels (admission, sparse indices) ----
constexpr int kChunk = 2048;       // tokens per counting / scatter CTA
constexpr int kScanThreads = 256;  // 8 tokens per thread

struct MaskView {
  const uint8_t* m;
  int64_t sb, sh, st;
  WGKV_DEV uint8_t at(int b, int h, int t) const { return m[b * sb + h * sh + int64_t(t) * st]; }
};

// counts[bh * nch + c] = #admitted tokens of (b, h) in chunk c of [0, limit); defined in admission.cu,
// launched there and by the sparse-index builder.
__global__ void chunk_count_kernel(MaskView mv, int Hk, int limit, int nch, int* counts);

}  // namespace wgkv
