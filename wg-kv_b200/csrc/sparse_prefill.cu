// Block-sparse (vertical-slash) causal prefill attention, sm_100a.
//
// Replaces the vLLM-fork sparse_attn_func called at src/modeling_layers.py:1366-1374
// (semantics pinned by utils/test_sparse_attn.py:34-93): for query row block
// i (64 queries) of kv head h, the keys are the admitted columns
// column_index[0 : column_count[i]] (all strictly before the band) followed
// by the band blocks block_offset[i, 0 : block_count[i]] (64 keys each,
// causally masked).  One CTA owns (row block, kv head, batch, head group):
// 64 queries x HPC query heads of the GQA group share every K/V tile it loads.
// K/V tiles of 64 keys are gathered row by row with cp.async (zero-filled
// past the ends) into a double-buffered, padded shared-memory ring; QK^T and
// PV run on mma.sync m16n8k16 (bf16 in, fp32 accumulate) with an fp32 online
// softmax and P rounded to bf16 for PV.
#include "common.cuh"
#include "runtime.h"

namespace wgkv {
int sparse_prefill_tc(const uint16_t* q, int64_t q_sb, int64_t q_sl, int64_t q_sh, const uint16_t* k, int64_t k_sb,
                      int64_t k_sl, int64_t k_sh, const uint16_t* v, int64_t v_sb, int64_t v_sl, int64_t v_sh, int B,
                      int L, int Hq, int Hk, int D, const int32_t* bc, const int32_t* bo, int64_t bo_stride,
                      const int32_t* cc, const int32_t* ci, int64_t ci_stride, float scale, uint16_t* out,
                      int64_t o_sb, int64_t o_sl, int64_t o_sh, int* err, cudaStream_t stream,
                      const uint16_t* pool_k, const uint16_t* pool_v, int64_t pool_rows, const int32_t* table,
                      int64_t t_stride, int t_first, int t_page);
namespace {

constexpr int kBlk = 64;  // query rows per block = keys per tile

struct PrefillParams {
  const uint16_t *q, *k, *v;
  uint16_t* out;
  int64_t q_sb, q_sl, q_sh, k_sb, k_sl, k_sh, v_sb, v_sl, v_sh, o_sb, o_sl, o_sh;
  int B, L, Hq, Hk, G, R, n_hg;
  const int32_t *bc, *bo, *cc, *ci;
  int64_t bo_stride, ci_stride;
  float scale_log2;
};

WGKV_DEV void cp_async16(uint32_t saddr, const void* g, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(saddr), "l"(g), "r"(valid ? 16 : 0)
               : "memory");
}
WGKV_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
WGKV_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int D, int HPC>
__global__ void __launch_bounds__(128 * HPC, 1) sparse_prefill_kernel(PrefillParams p) {
  constexpr int NT = 128 * HPC;
  constexpr int RS = D + 8;  // padded smem row (elements)
  extern __shared__ __align__(16) uint8_t smem_raw[];
  auto Ks = reinterpret_cast<uint16_t(*)[kBlk * RS]>(smem_raw);
  auto Vs = reinterpret_cast<uint16_t(*)[kBlk * RS]>(smem_raw + 2 * kBlk * RS * 2);
  auto rows = reinterpret_cast<int(*)[kBlk]>(smem_raw + 4 * kBlk * RS * 2);

  const int i = p.R - 1 - blockIdx.x;  // heaviest row blocks first
  const int hg = blockIdx.y % p.n_hg;
  const int h = blockIdx.y / p.n_hg;
  const int b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3, mi = lane >> 3, ri = lane & 7;
  const int hl = warp >> 2;                   // head within this CTA
  const int hq = h * p.G + hg * HPC + hl;     // query head
  const bool head_ok = hg * HPC + hl < p.G;
  const int qrow0 = i * kBlk + (warp & 3) * 16;

  const int ncol = p.cc[(int64_t(b) * p.Hk + h) * p.R + i];
  const int nband = p.bc[i];
  const int ntc = (ncol + kBlk - 1) / kBlk;
  const int ntiles = ntc + nband;
  const int32_t* cidx = p.ci + (int64_t(b) * p.Hk + h) * p.ci_stride;
  const uint16_t* kb = p.k + b * p.k_sb + h * p.k_sh;
  const uint16_t* vb = p.v + b * p.v_sb + h * p.v_sh;

  auto load_tile = [&](int j, int s) {
    const bool col = j < ntc;
    const int off = col ? j * kBlk : p.bo[int64_t(i) * p.bo_stride + (j - ntc)];
    for (int e = tid; e < kBlk * (D / 8); e += NT) {
      const int r = e / (D / 8), ch = e - r * (D / 8);
      int tk;
      if (col) tk = (off + r < ncol) ? cidx[off + r] : -1;
      else tk = off + r;
      const bool valid = tk >= 0 && tk < p.L;
      const int tks = valid ? tk : 0;
      cp_async16(smem_u32(&Ks[s][r * RS + ch * 8]), kb + int64_t(tks) * p.k_sl + ch * 8, valid);
      cp_async16(smem_u32(&Vs[s][r * RS + ch * 8]), vb + int64_t(tks) * p.v_sl + ch * 8, valid);
      if (ch == 0) rows[s][r] = valid ? tk : -1;
    }
  };

  // Q fragments for this warp's 16 rows of head hq
  uint32_t qa[D / 16][4];
  {
    const int r0 = qrow0 + g, r1 = qrow0 + g + 8;
    const uint16_t* qb = p.q + b * p.q_sb + int64_t(hq) * p.q_sh;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const int c0 = kk * 16 + 2 * t4;
      const bool ok0 = head_ok && r0 < p.L, ok1 = head_ok && r1 < p.L;
      qa[kk][0] = ok0 ? *reinterpret_cast<const uint32_t*>(qb + int64_t(r0) * p.q_sl + c0) : 0u;
      qa[kk][1] = ok1 ? *reinterpret_cast<const uint32_t*>(qb + int64_t(r1) * p.q_sl + c0) : 0u;
      qa[kk][2] = ok0 ? *reinterpret_cast<const uint32_t*>(qb + int64_t(r0) * p.q_sl + c0 + 8) : 0u;
      qa[kk][3] = ok1 ? *reinterpret_cast<const uint32_t*>(qb + int64_t(r1) * p.q_sl + c0 + 8) : 0u;
    }
  }
  float acc[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int qi0 = qrow0 + g, qi1 = qrow0 + g + 8;

  if (ntiles > 0) {
    load_tile(0, 0);
    cp_async_commit();
  }
  for (int j = 0; j < ntiles; ++j) {
    const int s = j & 1;
    if (j + 1 < ntiles) {
      load_tile(j + 1, s ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const bool band = j >= ntc;
    // ---- S = Q K^T : 16 rows x 64 keys ----
    float sc[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
    const uint32_t kbase = smem_u32(&Ks[s][((mi >> 1) * 8 + ri) * RS + (mi & 1) * 8]);
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t r0, r1, r2, r3;
        ldmatrix_x4(r0, r1, r2, r3, kbase + (np * 16 * RS + kk * 16) * 2);
        mma_bf16_16816(sc[2 * np], qa[kk], r0, r1);
        mma_bf16_16816(sc[2 * np + 1], qa[kk], r2, r3);
      }
    }
    // ---- mask + online softmax ----
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int tk = rows[s][n * 8 + 2 * t4 + e];
        const bool v0 = tk >= 0 && (!band || tk <= qi0);
        const bool v1 = tk >= 0 && (!band || tk <= qi1);
        sc[n][e] = v0 ? sc[n][e] * p.scale_log2 : -INFINITY;
        sc[n][2 + e] = v1 ? sc[n][2 + e] * p.scale_log2 : -INFINITY;
        mx0 = fmaxf(mx0, sc[n][e]);
        mx1 = fmaxf(mx1, sc[n][2 + e]);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffff, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffff, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffff, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffff, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    // rows that have seen no key yet keep a -inf max: use 0 as the exponent base
    const float base0 = mn0 == -INFINITY ? 0.f : mn0, base1 = mn1 == -INFINITY ? 0.f : mn1;
    const float a0 = exp2f(m0 - base0), a1 = exp2f(m1 - base1);
    m0 = mn0;
    m1 = mn1;
    float ps0 = 0.f, ps1 = 0.f;
    uint32_t pa[4][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const float p00 = exp2f(sc[n][0] - base0), p01 = exp2f(sc[n][1] - base0);
      const float p10 = exp2f(sc[n][2] - base1), p11 = exp2f(sc[n][3] - base1);
      ps0 += p00 + p01;
      ps1 += p10 + p11;
      const int ks = n >> 1, hi = n & 1;
      pa[ks][hi * 2 + 0] = pack_bf16x2(p00, p01);
      pa[ks][hi * 2 + 1] = pack_bf16x2(p10, p11);
    }
    l0 = l0 * a0 + ps0;
    l1 = l1 * a1 + ps1;
#pragma unroll
    for (int d = 0; d < D / 8; ++d) {
      acc[d][0] *= a0;
      acc[d][1] *= a0;
      acc[d][2] *= a1;
      acc[d][3] *= a1;
    }
    // ---- O += P V ----
    const uint32_t vbase = smem_u32(&Vs[s][((mi & 1) * 8 + ri) * RS + (mi >> 1) * 8]);
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
      for (int nd = 0; nd < D / 16; ++nd) {
        uint32_t r0, r1, r2, r3;
        ldmatrix_x4_trans(r0, r1, r2, r3, vbase + (ks * 16 * RS + nd * 16) * 2);
        mma_bf16_16816(acc[2 * nd], pa[ks], r0, r1);
        mma_bf16_16816(acc[2 * nd + 1], pa[ks], r2, r3);
      }
    }
    __syncthreads();
  }

  l0 += __shfl_xor_sync(0xffffffff, l0, 1);
  l0 += __shfl_xor_sync(0xffffffff, l0, 2);
  l1 += __shfl_xor_sync(0xffffffff, l1, 1);
  l1 += __shfl_xor_sync(0xffffffff, l1, 2);
  if (!head_ok) return;
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  uint16_t* ob = p.out + b * p.o_sb + int64_t(hq) * p.o_sh;
#pragma unroll
  for (int d = 0; d < D / 8; ++d) {
    const int c = d * 8 + 2 * t4;
    if (qi0 < p.L)
      *reinterpret_cast<uint32_t*>(ob + int64_t(qi0) * p.o_sl + c) = pack_bf16x2(acc[d][0] * inv0, acc[d][1] * inv0);
    if (qi1 < p.L)
      *reinterpret_cast<uint32_t*>(ob + int64_t(qi1) * p.o_sl + c) = pack_bf16x2(acc[d][2] * inv1, acc[d][3] * inv1);
  }
}

template <int D, int HPC>
int launch(const PrefillParams& p, cudaStream_t s) {
  dim3 grid(p.R, p.Hk * p.n_hg, p.B);
  const size_t smem = size_t(4) * kBlk * (D + 8) * 2 + 2 * kBlk * 4;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    if (cudaFuncSetAttribute(sparse_prefill_kernel<D, HPC>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) !=
        cudaSuccess)
      return WGKV_ECUDA;
    attr[dev] = true;
  }
  sparse_prefill_kernel<D, HPC><<<grid, 128 * HPC, smem, s>>>(p);
  return cudaGetLastError() == cudaSuccess ? WGKV_OK : WGKV_ECUDA;
}

}  // namespace
}  // namespace wgkv

using namespace wgkv;

extern "C" int wgkv_sparse_prefill(const uint16_t* q, int64_t q_sb, int64_t q_sl, int64_t q_sh, const uint16_t* k,
                                   int64_t k_sb, int64_t k_sl, int64_t k_sh, const uint16_t* v, int64_t v_sb,
                                   int64_t v_sl, int64_t v_sh, int batch, int seq_len, int num_q_heads,
                                   int num_kv_heads, int head_dim, const int32_t* block_count,
                                   const int32_t* block_offset, int64_t bo_stride, const int32_t* column_count,
                                   const int32_t* column_index, int64_t ci_stride, float softmax_scale, uint16_t* out,
                                   int64_t o_sb, int64_t o_sl, int64_t o_sh, int* err, void* stream) {
  if (!q || !k || !v || !out || !block_count || !block_offset || !column_count || !column_index) return WGKV_EINVAL;
  if (batch <= 0 || seq_len <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0) return WGKV_EINVAL;
  // 16-byte row gathers and 4-byte q/out accesses
  if (((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15) ||
      ((k_sb | k_sl | k_sh | v_sb | v_sl | v_sh) % 8) || (reinterpret_cast<uintptr_t>(q) & 3) ||
      (reinterpret_cast<uintptr_t>(out) & 3) || ((q_sb | q_sl | q_sh | o_sb | o_sl | o_sh) & 1))
    return WGKV_EINVAL;
  {
    const int rc = sparse_prefill_tc(q, q_sb, q_sl, q_sh, k, k_sb, k_sl, k_sh, v, v_sb, v_sl, v_sh, batch, seq_len,
                                     num_q_heads, num_kv_heads, head_dim, block_count, block_offset, bo_stride,
                                     column_count, column_index, ci_stride, softmax_scale, out, o_sb, o_sl, o_sh, err,
                                     as_stream(stream), nullptr, nullptr, 0, nullptr, 0, 0, 0);
    if (rc != 1) return rc;  // handled by the tensor-core kernel
  }
  PrefillParams p;
  p.q = q; p.k = k; p.v = v; p.out = out;
  p.q_sb = q_sb; p.q_sl = q_sl; p.q_sh = q_sh;
  p.k_sb = k_sb; p.k_sl = k_sl; p.k_sh = k_sh;
  p.v_sb = v_sb; p.v_sl = v_sl; p.v_sh = v_sh;
  p.o_sb = o_sb; p.o_sl = o_sl; p.o_sh = o_sh;
  p.B = batch; p.L = seq_len; p.Hq = num_q_heads; p.Hk = num_kv_heads;
  p.G = num_q_heads / num_kv_heads;
  p.R = (seq_len + kBlk - 1) / kBlk;
  p.bc = block_count; p.bo = block_offset; p.cc = column_count; p.ci = column_index;
  p.bo_stride = bo_stride; p.ci_stride = ci_stride;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  cudaStream_t s = as_stream(stream);
  const int hpc = p.G >= 2 ? 2 : 1;
  p.n_hg = (p.G + hpc - 1) / hpc;
  if (head_dim == 128) return hpc == 2 ? launch<128, 2>(p, s) : launch<128, 1>(p, s);
  if (head_dim == 64) return hpc == 2 ? launch<64, 2>(p, s) : launch<64, 1>(p, s);
  return WGKV_EINVAL;
}

extern "C" int wgkv_sparse_prefill_pooled(const uint16_t* q, int64_t q_sb, int64_t q_sl, int64_t q_sh,
                                          const uint16_t* k, int64_t k_sb, int64_t k_sl, int64_t k_sh,
                                          const uint16_t* v, int64_t v_sb, int64_t v_sl, int64_t v_sh, int batch,
                                          int seq_len, int num_q_heads, int num_kv_heads, int head_dim,
                                          const int32_t* block_count, const int32_t* block_offset, int64_t bo_stride,
                                          const int32_t* column_count, const int32_t* column_index,
                                          int64_t ci_stride, float softmax_scale, uint16_t* out, int64_t o_sb,
                                          int64_t o_sl, int64_t o_sh, const uint16_t* pool_k, const uint16_t* pool_v,
                                          int64_t pool_rows, const int32_t* table, int64_t table_stride,
                                          int table_first, int page_size, int* err, void* stream) {
  if (!q || !k || !v || !out || !block_count || !block_offset || !column_count || !column_index) return WGKV_EINVAL;
  if (batch <= 0 || seq_len <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0) return WGKV_EINVAL;
  if (!pool_k || !pool_v || !table || pool_rows <= 0 || pool_rows >= (int64_t(1) << 31) || page_size <= 0)
    return WGKV_EINVAL;
  const int rc = sparse_prefill_tc(q, q_sb, q_sl, q_sh, k, k_sb, k_sl, k_sh, v, v_sb, v_sl, v_sh, batch, seq_len,
                                   num_q_heads, num_kv_heads, head_dim, block_count, block_offset, bo_stride,
                                   column_count, column_index, ci_stride, softmax_scale, out, o_sb, o_sl, o_sh, err,
                                   as_stream(stream), pool_k, pool_v, pool_rows, table, table_stride, table_first,
                                   page_size);
  if (rc != 1) return rc;
  // shapes the tensor-core kernel does not take: the gathering path reads the same columns from k / v
  return wgkv_sparse_prefill(q, q_sb, q_sl, q_sh, k, k_sb, k_sl, k_sh, v, v_sb, v_sl, v_sh, batch, seq_len,
                             num_q_heads, num_kv_heads, head_dim, block_count, block_offset, bo_stride, column_count,
                             column_index, ci_stride, softmax_scale, out, o_sb, o_sl, o_sh, err, stream);
}

// ----------------------------------------------------------------------------
// Admitted-column compaction for the generic sparse_attn_func path: copies the
// K/V rows column_index[b, h, 0 : column_count[b, h, R-1]) of every (b, h) into
// contiguous scratch rows (b*Hk + h) * cap + c, so the tensor-core kernel reads
// them as plain 2D TMA tiles (the same layout the paged pool has after prefill
// compaction).  HBM-bound: one read and one write per admitted row.
// ----------------------------------------------------------------------------
namespace wgkv {
namespace {
constexpr int kGatherRows = 32;  // rows per CTA (256 threads, 8 lanes per row)

__global__ void __launch_bounds__(256) gather_columns_kernel(const uint16_t* k, int64_t k_sb, int64_t k_sl,
                                                             int64_t k_sh, const uint16_t* v, int64_t v_sb,
                                                             int64_t v_sl, int64_t v_sh, int Hk, int D, int R,
                                                             const int32_t* cc, const int32_t* ci,
                                                             int64_t ci_stride, int64_t cap, uint16_t* dk,
                                                             uint16_t* dv) {
  const int bh = blockIdx.y, b = bh / Hk, h = bh - b * Hk;
  const int64_t last = cc[int64_t(bh) * R + R - 1];
  const int count = int(last < cap ? last : cap);
  const int r = blockIdx.x * kGatherRows + (threadIdx.x >> 3);
  const int lane8 = threadIdx.x & 7;
  if (r >= count) return;
  const int t = ci[int64_t(bh) * ci_stride + r];
  const uint4* sk = reinterpret_cast<const uint4*>(k + b * k_sb + int64_t(t) * k_sl + h * k_sh);
  const uint4* sv = reinterpret_cast<const uint4*>(v + b * v_sb + int64_t(t) * v_sl + h * v_sh);
  uint4* ok = reinterpret_cast<uint4*>(dk + (int64_t(bh) * cap + r) * D);
  uint4* ov = reinterpret_cast<uint4*>(dv + (int64_t(bh) * cap + r) * D);
  for (int c = lane8; c < D / 8; c += 8) {
    ok[c] = __ldg(sk + c);
    ov[c] = __ldg(sv + c);
  }
}
}  // namespace
}  // namespace wgkv

extern "C" int wgkv_gather_columns(const uint16_t* k, int64_t k_sb, int64_t k_sl, int64_t k_sh, const uint16_t* v,
                                   int64_t v_sb, int64_t v_sl, int64_t v_sh, int batch, int num_kv_heads,
                                   int head_dim, int seq_len, const int32_t* column_count,
                                   const int32_t* column_index, int64_t ci_stride, int64_t cap, uint16_t* out_k,
                                   uint16_t* out_v, void* stream) {
  using namespace wgkv;
  if (!k || !v || !column_count || !column_index || !out_k || !out_v || batch <= 0 || num_kv_heads <= 0 ||
      seq_len <= 0 || cap <= 0 || (head_dim != 64 && head_dim != 128))
    return WGKV_EINVAL;
  if (((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out_k) |
        reinterpret_cast<uintptr_t>(out_v)) & 15) || ((k_sb | k_sl | k_sh | v_sb | v_sl | v_sh) % 8))
    return WGKV_EINVAL;
  const int R = (seq_len + 63) / 64;
  dim3 grid((cap + kGatherRows - 1) / kGatherRows, batch * num_kv_heads);
  gather_columns_kernel<<<grid, 256, 0, as_stream(stream)>>>(k, k_sb, k_sl, k_sh, v, v_sb, v_sl, v_sh, num_kv_heads,
                                                             head_dim, R, column_count, column_index, ci_stride, cap,
                                                             out_k, out_v);
  return cudaGetLastError() == cudaSuccess ? WGKV_OK : WGKV_ECUDA;
}
