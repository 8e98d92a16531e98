// Fused candidate filter of the exact top-k scan.
//
// After a first block of rows has given every query a candidate list of kp rows, the rest of
// the database is scored by the tcgen05 GEMM (128 x 256 tiles) with A = database rows (each row
// tile read from HBM once) and B = the bf16 queries (L2-resident), and the epilogue keeps only what can still
// matter: a score strictly above the query's current kp-th best f32 score is appended to that
// query's candidate buffer.  Nothing else leaves the SM, so no score matrix is written.  After
// each block, the candidates are merged into the list, which raises the thresholds for the next
// (geometrically larger) block.
//
// Every row that is never a candidate scored at most the list's kp-th f32 score at that time,
// and the lists' kp-th scores only grow, so the exact rescoring guard (scan.cu) still covers it:
// the result is the same as scoring every row into the list.  This replaces the dense
// rank_all of the reference (crates/ripvec-core/src/similarity.rs:24-26, index.rs:172-186).
#include "gemm_tc.cuh"
#include "scan.h"
#include "scan_sort.cuh"
#include "tmap.h"

namespace rv {

namespace {

constexpr int kFilterMaxKp = 512;  // larger candidate lists use the chunked path only

// Epilogue of the filtering GEMM: row = database row of the block, col = query.  The thresholds
// of all queries are staged in shared memory.  The count keeps growing past cap, so an overflow
// is visible to the merge.
struct EpiTopKFilter {
  const float* thr;  // [nq]
  int* cand_n;       // [nq]
  float* cand_s;     // [nq, cap]
  int64_t* cand_i;   // [nq, cap]
  int cap;
  int n_thr;     // staged thresholds: nq_pad (queries past nq have +inf)
  int64_t row0;  // global index of block row 0
  const float* nthr_s = nullptr;  // staged -thr
  using Pre = NoPre;
  using Tile = NoTile;
  __device__ __forceinline__ void stage(float* s, int t, int nt) {
    for (int i = t; i < n_thr; i += nt) s[i] = -thr[i];
    nthr_s = s;
  }
  __device__ __forceinline__ void tile_load(Tile&, int, int) const {}
  __device__ __forceinline__ void load(Pre&, int, int) const {}
  __device__ __forceinline__ void keep(int q, float v, int row) const {
    const int p = atomicAdd(&cand_n[q], 1);
    if (p < cap) {
      cand_s[static_cast<size_t>(q) * cap + p] = v;
      cand_i[static_cast<size_t>(q) * cap + p] = row0 + row;
    }
  }
  // max over 32 columns of v - thr (packed adds of -thr, three-input maxima): > 0 iff a score of
  // the 32 passes (v - thr of finite floats is exact in sign; -inf / +inf thresholds give +inf /
  // -inf).
  __device__ __forceinline__ float margin32(const float (&v)[32], const float4* nt) const {
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 a = nt[i];
      float d0, d1, d2, d3;
      f2_unpack(f2_add(f2_pack(v[4 * i], v[4 * i + 1]), f2_pack(a.x, a.y)), d0, d1);
      f2_unpack(f2_add(f2_pack(v[4 * i + 2], v[4 * i + 3]), f2_pack(a.z, a.w)), d2, d3);
      mx = fmax3(mx, fmaxf(d0, d1), fmaxf(d2, d3));
    }
    return mx;
  }
  __device__ __forceinline__ void apply(const Pre&, Tile&, int row, int col, const float (&v0)[32],
                                        const float (&v1)[32]) const {
    // Queries past nq have threshold +inf in the staged copy (see scan_filter_block).
    const float4* nt = reinterpret_cast<const float4*>(nthr_s + col);
    if (fmaxf(margin32(v0, nt), margin32(v1, nt + 8)) > 0.f) {  // rare: some score passes
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (v0[i] > -nthr_s[col + i]) keep(col + i, v0[i], row);
        if (v1[i] > -nthr_s[col + 32 + i]) keep(col + 32 + i, v1[i], row);
      }
    }
  }
};

// thr[q] = the list's kp-th score (-inf while the list is short); +inf for padded queries
// [nq, nq_pad) so that they never keep anything; cand_n = 0.
__global__ void filter_prepare_kernel(const float* __restrict__ list_s, const int* __restrict__ list_n,
                                      int kp, int nq, int nq_pad, float* __restrict__ thr,
                                      int* __restrict__ cand_n) {
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nq_pad) return;
  if (q < nq) {
    thr[q] = list_n[q] == kp ? list_s[static_cast<size_t>(q) * kp + kp - 1] : -INFINITY;
    cand_n[q] = 0;
  } else {
    thr[q] = INFINITY;
  }
}

// One CTA per query: list (kp best, sorted) + the block's candidates -> the kp best, sorted.
// A query whose candidates overflowed the buffer sets *overflow (its list is then incomplete
// and the caller redoes the batch without the filter).
__global__ void __launch_bounds__(256) filter_merge_kernel(const float* __restrict__ cand_s,
                                                           const int64_t* __restrict__ cand_i,
                                                           const int* __restrict__ cand_n, int cap,
                                                           int kp, float* __restrict__ list_s,
                                                           int64_t* __restrict__ list_i,
                                                           int* __restrict__ list_n,
                                                           int* __restrict__ overflow) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int q = blockIdx.x;
  const int m_all = cand_n[q];
  if (m_all == 0) return;
  if (m_all > cap) {
    if (threadIdx.x == 0) atomicExch(overflow, 1);
    return;
  }
  const int m = m_all;
  const int n_list = list_n[q];
  int n = 1;
  while (n < m + n_list) n <<= 1;
  int64_t* cid = reinterpret_cast<int64_t*>(smem);
  float* cs = reinterpret_cast<float*>(cid + n);
  float* ls = list_s + static_cast<size_t>(q) * kp;
  int64_t* li = list_i + static_cast<size_t>(q) * kp;
  for (int i = threadIdx.x; i < m; i += blockDim.x) {
    cs[i] = cand_s[static_cast<size_t>(q) * cap + i];
    cid[i] = cand_i[static_cast<size_t>(q) * cap + i];
  }
  for (int i = threadIdx.x; i < n_list; i += blockDim.x) {
    cs[m + i] = ls[i];
    cid[m + i] = li[i];
  }
  for (int i = m + n_list + threadIdx.x; i < n; i += blockDim.x) {
    cs[i] = -INFINITY;
    cid[i] = INT64_MAX;
  }
  bitonic_sort(cs, cid, n);
  const int keep = min(kp, m + n_list);
  for (int i = threadIdx.x; i < keep; i += blockDim.x) {
    ls[i] = cs[i];
    li[i] = cid[i];
  }
  if (threadIdx.x == 0) list_n[q] = keep;
}

}  // namespace

int scan_filter_cap() { return 2048; }
int scan_filter_max_kp() { return kFilterMaxKp; }

cudaError_t scan_filter_block(const CUtensorMap& tm_rows, const CUtensorMap& tm_queries, int rows,
                              int dim, int64_t row0, int nq, int nq_pad, int kp, float* thr,
                              int* cand_n, float* cand_s, int64_t* cand_i, float* list_s,
                              int64_t* list_i, int* list_n, int* overflow, unsigned int* err,
                              cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  if (nq_pad % 256 != 0 || nq_pad > 2560 || nq > nq_pad || dim % 64 != 0 || kp > kFilterMaxKp)
    return cudaErrorInvalidValue;
  const int cap = scan_filter_cap();
  filter_prepare_kernel<<<(nq_pad + 255) / 256, 256, 0, st>>>(list_s, list_n, kp, nq, nq_pad, thr, cand_n);
  EpiTopKFilter epi{thr, cand_n, cand_s, cand_i, cap, nq_pad, row0};
  cudaError_t e = launch_gemm_tc<__nv_bfloat16, 256>(tm_rows, tm_queries, rows, nq_pad, dim, 0, epi,
                                                      err, device_sm_count(), st);
  if (e != cudaSuccess) return e;
  int n = 1;
  while (n < cap + kp) n <<= 1;
  const size_t smem = size_t(n) * (sizeof(int64_t) + sizeof(float));
  static bool attr_set[64] = {false};  // set once for the largest list (kFilterMaxKp)
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    int nmax = 1;
    while (nmax < cap + kFilterMaxKp) nmax <<= 1;
    e = cudaFuncSetAttribute(filter_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(size_t(nmax) * (sizeof(int64_t) + sizeof(float))));
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  filter_merge_kernel<<<nq, 256, smem, st>>>(cand_s, cand_i, cand_n, cap, kp, list_s, list_i, list_n,
                                             overflow);
  return cudaGetLastError();
}

}  // namespace rv
