// Row-parallel attention output projection fused with the sum over ranks, sm_100a.
//
// A KV-head-sharded layer (each GPU holds whole GQA groups and its own pool) ends in o_proj
// (src/modeling_llama.py:286) applied to that GPU's heads only: y_r = a_r W_r^T with W_r the
// columns of W_o that multiply its query heads, and the layer output is sum_r y_r.  Instead of a
// GEMM followed by a separate all-reduce, one kernel per GPU does both over NVLink peer memory:
//
// * CTA j owns output columns [32 j, 32 j + 32) for every row.  It computes its tile of y_r with
//   mma.sync (bf16 in, fp32 accumulate; the operands are a few MB, so the GEMM is a short
//   latency-bound prologue, not a tensor-core throughput problem), rounds it to bf16 like the
//   unfused GEMM's output, and stores it into this GPU's partial buffer.
// * It then publishes the tile: a system-scope release store of the call's epoch into tile j's
//   flag on every peer.  The transfer of a tile thus starts as soon as that tile is computed.
// * It waits (bounded) for tile j's flag from every peer, reads the N partial tiles -- its own
//   and N-1 over NVLink, plain 16-byte peer loads, no TMA, no multicast -- sums them in fp32 in
//   rank order (so every GPU gets the same bits) and writes y.
//
// Partial buffers and flags are double-buffered by epoch parity.  A GPU reuses a parity two
// calls later only after every peer has published a tile of the call in between, i.e. after every
// peer finished reading this buffer.  The epoch is a device counter advanced by the last CTA of
// each call, so consecutive launches (and graph replays) need no host bookkeeping.
#include <string.h>

#include <mutex>

#include "common.cuh"
#include "runtime.h"

namespace wgkv {
namespace {

constexpr int kTpCols = 32;          // output columns per CTA
constexpr int kTpRows = 64;          // rows per m-block (4 warps x 16)
constexpr int kTpK = 128;            // K per pipeline stage
constexpr int kTpStages = 4;
constexpr int kTpThreads = 128;
constexpr int kTpRS = kTpK + 8;      // padded smem row (elements): conflict-free ldmatrix
constexpr int kTpStageElems = (kTpRows + kTpCols) * kTpRS;
constexpr size_t kTpSmem = size_t(kTpStages) * kTpStageElems * 2;  // 104 KB, dynamic

struct TpArgs {
  const uint16_t* a;
  int64_t lda;
  int rows, k;
  const uint16_t* w;
  int n_out;
  uint16_t* y;
  int64_t ldy;
  wgkv_peer_group g;
  int* err;
};

WGKV_DEV void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
WGKV_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
WGKV_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

WGKV_DEV void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
WGKV_DEV uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
WGKV_DEV uint4 ld_volatile16(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// flags of a GPU: [parity][source rank][tile], `stride` = the group's tile capacity
WGKV_DEV uint32_t* flag_at(uint32_t* base, int parity, int src, int tile, int stride) {
  return base + (size_t(parity) * WGKV_TP_MAX_WORLD + src) * stride + tile;
}

__global__ void __launch_bounds__(kTpThreads) oproj_allreduce_kernel(TpArgs p) {
  extern __shared__ __align__(128) uint16_t tp_smem[];
  auto as = [&](int st) { return tp_smem + st * kTpStageElems; };
  auto ws = [&](int st) { return tp_smem + st * kTpStageElems + kTpRows * kTpRS; };
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, n_tiles = gridDim.x;
  const int fstride = p.g.max_cols / kTpCols + 1;
  const int c0 = tile * kTpCols;
  const int rank = p.g.rank, world = p.g.world;
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(p.g.ctr) + 1u;  // this call
  const int parity = epoch & 1u;
  uint16_t* mine = world > 1 ? reinterpret_cast<uint16_t*>(p.g.partial[rank]) +
                                   size_t(parity) * p.g.max_rows * p.g.max_cols
                             : nullptr;
  const int g = lane >> 2, t4 = lane & 3, mi = lane >> 3, ri = lane & 7;
  const int nk = p.k / kTpK;

  for (int m0 = 0; m0 < p.rows; m0 += kTpRows) {
    float acc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    auto load = [&](int kc, int st) {
      // A: 64 rows x 128 k = 1024 vectors of 16 B; W: 32 rows x 128 k = 512 vectors
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int v = tid + i * kTpThreads, r = v >> 4, c = (v & 15) * 8;
        const bool ok = m0 + r < p.rows;
        const uint16_t* src = p.a + int64_t(ok ? m0 + r : 0) * p.lda + kc * kTpK + c;
        cp_async16(smem_u32(as(st) + r * kTpRS + c), src, ok);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int v = tid + i * kTpThreads, r = v >> 4, c = (v & 15) * 8;
        cp_async16(smem_u32(ws(st) + r * kTpRS + c), p.w + int64_t(c0 + r) * p.k + kc * kTpK + c, true);
      }
    };
#pragma unroll
    for (int s = 0; s < kTpStages - 1; ++s) {
      if (s < nk) load(s, s);
      cp_async_commit();
    }
    for (int kc = 0; kc < nk; ++kc) {
      cp_async_wait<kTpStages - 2>();
      __syncthreads();
      if (kc + kTpStages - 1 < nk) load(kc + kTpStages - 1, (kc + kTpStages - 1) % kTpStages);
      cp_async_commit();
      const int st = kc % kTpStages;
      const uint32_t abase = smem_u32(as(st) + (warp * 16 + (mi & 1) * 8 + ri) * kTpRS + (mi >> 1) * 8);
      const uint32_t wbase = smem_u32(ws(st) + ((mi >> 1) * 8 + ri) * kTpRS + (mi & 1) * 8);
#pragma unroll
      for (int kk = 0; kk < kTpK / 16; ++kk) {
        uint32_t a[4];
        ldmatrix_x4(a[0], a[1], a[2], a[3], abase + kk * 32);
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          uint32_t r0, r1, r2, r3;
          ldmatrix_x4(r0, r1, r2, r3, wbase + (np * 16 * kTpRS) * 2 + kk * 32);
          mma_bf16_16816(acc[2 * np], a, r0, r1);
          mma_bf16_16816(acc[2 * np + 1], a, r2, r3);
        }
      }
    }
    cp_async_wait<0>();
    __syncthreads();  // the stages are reloaded by the next m-block
    // epilogue: bf16 tile -> y (single GPU) or this GPU's partial buffer
    uint16_t* dst = world > 1 ? mine : p.y;
    const int64_t ld = world > 1 ? p.g.max_cols : p.ldy;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const int col = c0 + nt * 8 + 2 * t4;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int row = m0 + warp * 16 + g + hf * 8;
        if (row < p.rows)
          *reinterpret_cast<uint32_t*>(dst + int64_t(row) * ld + col) =
              pack_bf16x2(acc[nt][2 * hf], acc[nt][2 * hf + 1]);
      }
    }
  }
  if (world > 1) {
    // ---- publish tile `tile` of this GPU's partial to every peer ----
    __syncthreads();
    if (tid == 0) {
      __threadfence_system();
      for (int r = 0; r < world; ++r)
        if (r != rank) st_release_sys(flag_at(p.g.flags[r], parity, rank, tile, fstride), epoch);
    }
    // ---- wait for the peers' tiles (bounded), then sum in rank order ----
    if (tid < world && tid != rank) {
      const uint32_t* f = flag_at(p.g.flags[rank], parity, tid, tile, fstride);
      uint64_t t0 = 0;
      for (long long it = 0;; ++it) {
        if (int32_t(ld_acquire_sys(f) - epoch) >= 0) break;
        if ((it & 1023) == 0) {
          const uint64_t now = global_ns();
          if (it == 0) {
            t0 = now;
          } else if (now - t0 > kWaitLimitNs) {
            set_error(p.err, WGKV_ERR_TIMEOUT);
            break;
          }
        }
      }
    }
    __syncthreads();
    const size_t slot = size_t(parity) * p.g.max_rows * p.g.max_cols;
    // 16-byte vectors of the tile: rows x 4
    for (int v = tid; v < p.rows * (kTpCols / 8); v += kTpThreads) {
      const int row = v >> 2, col = c0 + (v & 3) * 8;
      float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int r = 0; r < world; ++r) {
        const uint16_t* src = reinterpret_cast<const uint16_t*>(p.g.partial[r]) + slot +
                              size_t(row) * p.g.max_cols + col;
        const uint4 x = ld_volatile16(src);
        const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          s[2 * e] += __uint_as_float(xs[e] << 16);
          s[2 * e + 1] += __uint_as_float(xs[e] & 0xffff0000u);
        }
      }
      uint4 o;
      o.x = pack_bf16x2(s[0], s[1]);
      o.y = pack_bf16x2(s[2], s[3]);
      o.z = pack_bf16x2(s[4], s[5]);
      o.w = pack_bf16x2(s[6], s[7]);
      *reinterpret_cast<uint4*>(p.y + int64_t(row) * p.ldy + col) = o;
    }
  }
  // ---- the last CTA advances the epoch for the next call ----
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(p.g.ctr + 1, 1u) == unsigned(n_tiles) - 1u) {
      p.g.ctr[1] = 0u;
      __threadfence();
      p.g.ctr[0] = epoch;
    }
  }
}

// cuMemGetAddressRange through the runtime's driver entry point (no libcuda link)
typedef CUresult (*PFN_addr_range)(CUdeviceptr*, size_t*, CUdeviceptr);
PFN_addr_range g_range = nullptr;
std::once_flag g_range_once;

}  // namespace
}  // namespace wgkv

using namespace wgkv;

extern "C" size_t wgkv_tp_partial_bytes(int max_rows, int max_cols) {
  if (max_rows <= 0 || max_cols <= 0) return 0;
  return 2 * size_t(max_rows) * max_cols * 2;
}

extern "C" size_t wgkv_tp_flag_bytes(int max_cols) {
  if (max_cols <= 0) return 0;
  return 2 * size_t(WGKV_TP_MAX_WORLD) * (max_cols / kTpCols + 1) * 4;
}

extern "C" int wgkv_ipc_handle(const void* ptr, void* handle_out, size_t* offset_out) {
  if (!ptr || !handle_out || !offset_out) return WGKV_EINVAL;
  std::call_once(g_range_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_range = reinterpret_cast<PFN_addr_range>(fn);
  });
  if (!g_range) return WGKV_ECUDA;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (g_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return WGKV_ECUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return WGKV_ECUDA;
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = reinterpret_cast<uintptr_t>(ptr) - uintptr_t(base);
  return WGKV_OK;
}

extern "C" int wgkv_ipc_open(const void* handle, void** base_out) {
  if (!handle || !base_out) return WGKV_EINVAL;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? WGKV_OK : WGKV_ECUDA;
}

extern "C" int wgkv_ipc_close(void* base) {
  if (!base) return WGKV_EINVAL;
  return cudaIpcCloseMemHandle(base) == cudaSuccess ? WGKV_OK : WGKV_ECUDA;
}

extern "C" int wgkv_oproj_allreduce(const uint16_t* a, int64_t lda, int rows, int k, const uint16_t* w, int n_out,
                                    uint16_t* y, int64_t ldy, const wgkv_peer_group* group, int* err,
                                    void* stream) {
  if (!a || !w || !y || !group || !group->ctr || rows <= 0 || k <= 0 || n_out <= 0) return WGKV_EINVAL;
  const wgkv_peer_group& g = *group;
  if (g.world < 1 || g.world > WGKV_TP_MAX_WORLD || g.rank < 0 || g.rank >= g.world) return WGKV_EINVAL;
  if (k % kTpK || n_out % kTpCols || lda < k || ldy < n_out || lda % 8 || ldy % 8) return WGKV_EINVAL;
  static bool attr[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return WGKV_ECUDA;
  if (dev < 64 && !attr[dev]) {
    if (cudaFuncSetAttribute(oproj_allreduce_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kTpSmem)) !=
        cudaSuccess)
      return WGKV_ECUDA;
    attr[dev] = true;
  }
  if (((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(y)) & 15))
    return WGKV_EINVAL;
  const int sms = device_sms();
  if (g.world > 1) {
    // every CTA of the grid waits for the peers' copy of its tile: the grid must be co-resident
    if (sms <= 0 || n_out / kTpCols > sms) return WGKV_EINVAL;
    if (rows > g.max_rows || n_out > g.max_cols || g.max_cols % kTpCols) return WGKV_EINVAL;
    for (int r = 0; r < g.world; ++r)
      if (!g.partial[r] || !g.flags[r] || (reinterpret_cast<uintptr_t>(g.partial[r]) & 15)) return WGKV_EINVAL;
  }
  TpArgs p{a, lda, rows, k, w, n_out, y, ldy, g, err};
  oproj_allreduce_kernel<<<n_out / kTpCols, kTpThreads, kTpSmem, as_stream(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? WGKV_OK : WGKV_ECUDA;
}
