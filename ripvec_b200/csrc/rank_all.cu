// SearchIndex::rank in full (crates/ripvec-core/src/index.rs:172-186): every row whose score
// reaches the threshold, best first.  MCP `find_similar` calls rank(&emb, 0.0) and pages through
// the whole result (ripvec-mcp/src/tools.rs:563-570), so no row may be dropped.
//
// Three steps on the index's stream:
//   1. filter: every row's f32 dot product with the bf16-rounded query (one warp per row, any
//      summation order); rows whose f32 score reaches threshold - eps are candidates.  eps bounds
//      the f32 accumulation error (dim * 2^-22 * |q| * max|row|; the products of two bf16 values
//      are exact in f32, and an f32 sum of dim terms is off by at most dim * 2^-24 * sum |p_d|),
//      so no row whose exact score reaches the threshold is missed.  With threshold = -inf every
//      row is a candidate and the pass is skipped.
//   2. exact: each candidate's score is the sequential f64 sum over d = 0..dim-1 of the exact
//      bf16 x bf16 products (the definition of every other search entry point); rows with exact
//      score >= threshold are kept as (score, row) pairs.
//   3. sort: a radix sort of the pairs by score, descending.  The pairs arrive in no fixed order,
//      so equal scores are put in row order on the host, which receives every pair anyway.
#include <cub/device/device_radix_sort.cuh>

#include "common.cuh"
#include "rank_all.h"
#include "tmap.h"

namespace rv {

namespace {

constexpr int kFilterThreads = 256;

// Each warp takes groups of 32 consecutive rows; lane j of the warp records whether row j of the
// group passed, then the warp claims slots for its passing rows with one atomic.
__global__ void __launch_bounds__(kFilterThreads) rank_filter_kernel(const __nv_bfloat16* __restrict__ db,
                                                                     int64_t n, int dim,
                                                                     const __nv_bfloat16* __restrict__ qb,
                                                                     float lo, int* __restrict__ cand,
                                                                     unsigned long long* __restrict__ count) {
  extern __shared__ __align__(16) float qs[];
  for (int d = threadIdx.x; d < dim; d += blockDim.x) qs[d] = __bfloat162float(qb[d]);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t groups = (n + 31) >> 5;
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); g < groups;
       g += warps) {
    const int64_t r0 = g << 5;
    const int rows = static_cast<int>(n - r0 < 32 ? n - r0 : 32);
    bool pass = false;
    for (int j = 0; j < rows; ++j) {
      const __nv_bfloat16* p = db + static_cast<size_t>(r0 + j) * dim;
      float s = 0.f;
      for (int d = lane * 8; d < dim; d += 256) {
        float f[8];
        unpack8<__nv_bfloat16>(*reinterpret_cast<const uint4*>(p + d), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) s = fmaf(f[e], qs[d + e], s);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == j) pass = s >= lo;
    }
    const unsigned mask = __ballot_sync(0xffffffffu, pass);
    if (mask == 0u) continue;
    unsigned long long off = 0;
    if (lane == 0) off = atomicAdd(count, static_cast<unsigned long long>(__popc(mask)));
    off = __shfl_sync(0xffffffffu, off, 0);
    if (pass) cand[off + __popc(mask & ((1u << lane) - 1u))] = static_cast<int>(r0 + lane);
  }
}

// One thread per candidate (cand == nullptr: candidate i is row i): the sequential f64 sum, and
// the (score, base + row) pair when the score reaches the threshold.
__global__ void __launch_bounds__(256) rank_exact_kernel(const __nv_bfloat16* __restrict__ db, int dim,
                                                         const __nv_bfloat16* __restrict__ qb,
                                                         const int* __restrict__ cand, int64_t m, int64_t base,
                                                         double threshold, double* __restrict__ out_s,
                                                         int64_t* __restrict__ out_i,
                                                         unsigned long long* __restrict__ count) {
  extern __shared__ __align__(16) float qs[];
  for (int d = threadIdx.x; d < dim; d += blockDim.x) qs[d] = __bfloat162float(qb[d]);
  __syncthreads();
  const int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  bool keep = false;
  double acc = 0.0;
  int64_t row = 0;
  if (c < m) {
    row = cand ? cand[c] : c;
    const __nv_bfloat16* p = db + static_cast<size_t>(row) * dim;
#pragma unroll 4
    for (int d = 0; d < dim; d += 8) {
      float f[8];
      unpack8<__nv_bfloat16>(*reinterpret_cast<const uint4*>(p + d), f);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc = fma(double(f[e]), double(qs[d + e]), acc);
    }
    keep = acc >= threshold;
  }
  const unsigned mask = __ballot_sync(0xffffffffu, keep);
  if (mask == 0u) return;
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(mask) - 1;
  unsigned long long off = 0;
  if (lane == leader) off = atomicAdd(count, static_cast<unsigned long long>(__popc(mask)));
  off = __shfl_sync(0xffffffffu, off, leader);
  if (keep) {
    const unsigned long long o = off + __popc(mask & ((1u << lane) - 1u));
    out_s[o] = acc;
    out_i[o] = base + row;
  }
}

}  // namespace

cudaError_t rank_filter(const __nv_bfloat16* db, int64_t n, int dim, const __nv_bfloat16* qb, float lo,
                        int* cand, unsigned long long* count, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  const int64_t groups = (n + 31) / 32;
  const int64_t per_cta = kFilterThreads / 32;
  const int64_t want = (groups + per_cta - 1) / per_cta;
  const int grid = static_cast<int>(std::min<int64_t>(want, int64_t(device_sm_count()) * 8));
  rank_filter_kernel<<<grid, kFilterThreads, size_t(dim) * 4, st>>>(db, n, dim, qb, lo, cand, count);
  return cudaGetLastError();
}

cudaError_t rank_exact(const __nv_bfloat16* db, int dim, const __nv_bfloat16* qb, const int* cand, int64_t m,
                       int64_t base, double threshold, double* out_s, int64_t* out_i,
                       unsigned long long* count, cudaStream_t st) {
  if (m <= 0) return cudaSuccess;
  const int64_t grid = (m + 255) / 256;
  rank_exact_kernel<<<static_cast<unsigned>(grid), 256, size_t(dim) * 4, st>>>(db, dim, qb, cand, m, base,
                                                                                threshold, out_s, out_i, count);
  return cudaGetLastError();
}

cudaError_t rank_sort_desc(void* temp, size_t* temp_bytes, const double* keys_in, double* keys_out,
                           const int64_t* vals_in, int64_t* vals_out, int64_t m, cudaStream_t st) {
  if (m > INT32_MAX) return cudaErrorInvalidValue;
  return cub::DeviceRadixSort::SortPairsDescending(temp, *temp_bytes, keys_in, keys_out, vals_in, vals_out,
                                                   static_cast<int>(m), 0, 64, st);
}

}  // namespace rv
