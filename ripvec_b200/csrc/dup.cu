// All-pairs near-duplicate search: SearchIndex::find_duplicates
// (crates/ripvec-core/src/index.rs:325-348), which forms the full n x n similarity matrix with one
// BLAS GEMM and keeps the upper-triangle pairs scoring at least the threshold.
//
// Here the same products come from the tcgen05 GEMM in strips of rows (A = rows [r0, r0 + R),
// B = rows [r0, n), so only the upper triangle and its diagonal blocks are computed; tiles are
// walked column block by column block, so the strip stays in L2 and B streams once), and the
// epilogue keeps a pair (i, j > i) whose f32 score is at least threshold - eps, eps a bound on
// the f32 accumulation error (dim * 2^-22 * max row norm^2).  No matrix leaves the SM: a kept
// pair is a {i, j, f32 score} record at a slot from one global counter per warp.  Each record is
// then re-scored exactly (sequential f64 sum of the bf16 products, the exact scan's definition),
// and the host keeps the pairs at or above the threshold.  Every pair whose exact score reaches
// the threshold has an f32 score of at least threshold - eps, so none is missed.
#include "dup.h"
#include "gemm_tc.cuh"

namespace rv {

namespace {

// Writes the records of the set bits of (m0, m1): pair (i, j0 + bit) with its f32 score.
// Slots past cap are dropped (the counter still counts them).  Out of line, like the scan
// filter's writer, to keep the GEMM's instruction footprint small.
__device__ __noinline__ void write_pairs(int4* rec, long long cap, unsigned long long p0, const float* vals,
                                         uint32_t m0, uint32_t m1, int i, int j0) {
  unsigned long long p = p0;
  while (m0) {
    const int b = __ffs(m0) - 1;
    m0 &= m0 - 1;
    if (p < static_cast<unsigned long long>(cap)) rec[p] = make_int4(i, j0 + b, __float_as_int(vals[b]), 0);
    ++p;
  }
  while (m1) {
    const int b = __ffs(m1) - 1;
    m1 &= m1 - 1;
    if (p < static_cast<unsigned long long>(cap))
      rec[p] = make_int4(i, j0 + 32 + b, __float_as_int(vals[32 + b]), 0);
    ++p;
  }
}

// GEMM epilogue: row = strip row (global i = r0 + row), col = B column (global j = r0 + col).
struct EpiPairFilter {
  int4* rec;
  unsigned long long* counter;
  long long cap;
  float thr_lo;
  int r0;
  int n;
  using Pre = NoPre;
  using Tile = NoTile;
  // B (the rows from r0 on, up to n x 1536 bytes) outgrows L2 while A (one strip) fits: walk the
  // tiles column block by column block so that each B tile comes from HBM once.
  static constexpr bool kColumnMajorTiles = true;
  __device__ __forceinline__ void stage(float*, int, int) const {}
  __device__ __forceinline__ void tile_load(Tile&, int, int) const {}
  __device__ __forceinline__ void load(Pre&, int, int) const {}
  // Called by the lanes whose row is inside the strip (a prefix of the warp's lanes).
  __device__ __forceinline__ void apply(const Pre&, Tile&, int row, int col, const float (&v0)[32],
                                        const float (&v1)[32]) const {
    const unsigned am = __activemask();
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < 32; ++k) mx = fmax3(mx, v0[k], v1[k]);
    const bool maybe = mx >= thr_lo;
    if (!__any_sync(am, maybe)) return;  // common case: no score near the threshold
    const int i = r0 + row;
    const int j0 = r0 + col;
    uint32_t m0 = 0u, m1 = 0u;
    if (maybe) {
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const int ja = j0 + k, jb = j0 + 32 + k;
        m0 |= ((v0[k] >= thr_lo && ja > i && ja < n) ? 1u : 0u) << k;
        m1 |= ((v1[k] >= thr_lo && jb > i && jb < n) ? 1u : 0u) << k;
      }
    }
    const int cnt = __popc(m0) + __popc(m1);
    const int lane = threadIdx.x & 31;
    const int last = 31 - __clz(am);
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(am, incl, o);
      if (lane >= o) incl += y;
    }
    unsigned long long base = 0ull;
    if (lane == last && incl > 0) base = atomicAdd(counter, static_cast<unsigned long long>(incl));
    base = __shfl_sync(am, base, last);
    if (cnt == 0) return;
    float vals[64];
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      vals[k] = v0[k];
      vals[32 + k] = v1[k];
    }
    write_pairs(rec, cap, base + static_cast<unsigned long long>(incl - cnt), vals, m0, m1, i, j0);
  }
};

// One thread per record: the exact score of pair (i, j), the sequential f64 sum over d of the
// bf16 products (each exact in f64).
__global__ void __launch_bounds__(256) pair_rescore_kernel(const __nv_bfloat16* __restrict__ db, int dim,
                                                           const int4* __restrict__ rec, long long m,
                                                           double* __restrict__ s64) {
  for (long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; t < m;
       t += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int4 r = rec[t];
    const __nv_bfloat16* a = db + static_cast<size_t>(r.x) * dim;
    const __nv_bfloat16* b = db + static_cast<size_t>(r.y) * dim;
    double acc = 0.0;
#pragma unroll 4
    for (int d = 0; d < dim; d += 8) {
      float fa[8], fb[8];
      unpack8<__nv_bfloat16>(*reinterpret_cast<const uint4*>(a + d), fa);
      unpack8<__nv_bfloat16>(*reinterpret_cast<const uint4*>(b + d), fb);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc = fma(double(fa[k]), double(fb[k]), acc);
    }
    s64[t] = acc;
  }
}

}  // namespace

cudaError_t dup_candidates(const CUtensorMap& tm_strip, const CUtensorMap& tm_rows, int rows, int cols, int dim,
                           int r0, int n, float thr_lo, int4* rec, unsigned long long* counter, long long cap,
                           unsigned int* err, cudaStream_t st) {
  if (rows <= 0 || cols <= 0) return cudaSuccess;
  if (cols % 256 != 0 || dim % 64 != 0) return cudaErrorInvalidValue;
  EpiPairFilter epi{rec, counter, cap, thr_lo, r0, n};
  return launch_gemm_tc<__nv_bfloat16, 256>(tm_strip, tm_rows, rows, cols, dim, r0, epi, err, device_sm_count(),
                                            st);
}

cudaError_t dup_rescore(const __nv_bfloat16* db, int dim, const int4* rec, long long m, double* s64,
                        cudaStream_t st) {
  if (m <= 0) return cudaSuccess;
  const long long blocks = (m + 255) / 256;
  const int grid = static_cast<int>(blocks < 4096 ? blocks : 4096);
  pair_rescore_kernel<<<grid, 256, 0, st>>>(db, dim, rec, m, s64);
  return cudaGetLastError();
}

}  // namespace rv
