// Fused candidate filter of the exact top-k scan.
//
// After a first block of rows has given every query a candidate list of kp rows, the rest of
// the database is scored by the tcgen05 GEMM (128 x 256 tiles; 128 x 128 for batches of at most
// 128 queries) with A = database rows (each row
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

constexpr int kFilterMaxThr = 2048;  // staged thresholds (queries); the CTA's counter follows

// Writes the records of the set bits of (m0, m1) (columns col + bit, bit 32+ for m1) from vals
// into rec[p0...] (slots past cap are dropped).  Out of line: one copy serves every call site of
// the filter epilogue, which keeps the GEMM's instruction footprint small.
__device__ __noinline__ void write_records(int4* rec, int cap, int p0, const float* vals, uint32_t m0,
                                           uint32_t m1, int col, int row) {
  int p = p0;
  while (m0) {
    const int i = __ffs(m0) - 1;
    m0 &= m0 - 1;
    if (p < cap) rec[p] = make_int4(col + i, row, __float_as_int(vals[i]), 0);
    ++p;
  }
  while (m1) {
    const int i = __ffs(m1) - 1;
    m1 &= m1 - 1;
    if (p < cap) rec[p] = make_int4(col + 32 + i, row, __float_as_int(vals[32 + i]), 0);
    ++p;
  }
}

// Epilogue of the filtering GEMM: row = database row of the block, col = query.  The negated
// thresholds of all queries and the CTA's record counter live in the staging shared memory.  A
// kept score becomes a {query, block row, score bits} record in the CTA's own region of `rec`;
// the slot comes from the shared counter, so keeping costs a shared atomic and a plain store
// instead of a global atomic round trip per candidate.  finish() publishes the count (which may
// exceed rec_cap: the bucket kernel then reports an overflow).
struct EpiTopKFilter {
  const float* thr;  // [n_thr]
  int4* rec;         // [grid][rec_cap]
  int* rec_n;        // [grid]
  int rec_cap;
  int n_thr;         // staged thresholds: nq_pad (queries past nq have +inf)
  const float* nthr_s = nullptr;  // staged -thr
  int* cnt_s = nullptr;
  using Pre = NoPre;
  using Tile = NoTile;
  __device__ __forceinline__ void stage(float* s, int t, int nt) {
    for (int i = t; i < n_thr; i += nt) s[i] = -thr[i];
    nthr_s = s;
    cnt_s = reinterpret_cast<int*>(s + kFilterMaxThr);
    if (t == 0) *cnt_s = 0;
  }
  __device__ __forceinline__ void tile_load(Tile&, int, int) const {}
  __device__ __forceinline__ void load(Pre&, int, int) const {}
  __device__ __forceinline__ void finish(int t) const {
    if (t == 0) rec_n[blockIdx.x] = *cnt_s;
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
  // Called by the lanes whose row is inside the matrix (a prefix of the warp's lanes).
  __device__ __forceinline__ void apply(const Pre&, Tile&, int row, int col, const float (&v0)[32],
                                        const float (&v1)[32]) const {
    const float4* nt = reinterpret_cast<const float4*>(nthr_s + col);
    const unsigned am = __activemask();
    const bool hit = fmaxf(margin32(v0, nt), margin32(v1, nt + 8)) > 0.f;
    if (!__any_sync(am, hit)) return;  // common case: nothing in these 64 columns passes
    // Masks of the passing columns, then slots for the warp's records: per-lane counts, a warp
    // prefix sum, one shared atomic.
    uint32_t m0 = 0u, m1 = 0u;
    if (hit) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        m0 |= (v0[i] > -nthr_s[col + i] ? 1u : 0u) << i;
        m1 |= (v1[i] > -nthr_s[col + 32 + i] ? 1u : 0u) << i;
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
    int base = 0;
    if (lane == last) base = atomicAdd(cnt_s, incl);
    base = __shfl_sync(am, base, last);
    if (cnt == 0) return;
    float vals[64];  // local copy: the writer below indexes it by bit position
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      vals[i] = v0[i];
      vals[32 + i] = v1[i];
    }
    write_records(rec + static_cast<size_t>(blockIdx.x) * rec_cap, rec_cap, base + incl - cnt, vals,
                  m0, m1, col, row);
  }
};

// Block c moves the records of GEMM CTA c into the per-query candidate buffers (global row =
// row0 + block row).  A CTA that kept more records than its region holds sets *overflow.
__global__ void __launch_bounds__(256) filter_bucket_kernel(const int4* __restrict__ rec,
                                                            const int* __restrict__ rec_n, int rec_cap,
                                                            int64_t row0, int cap, int* __restrict__ cand_n,
                                                            float* __restrict__ cand_s,
                                                            int64_t* __restrict__ cand_i,
                                                            int* __restrict__ overflow) {
  const int c = blockIdx.x;
  const int n = rec_n[c];
  if (n > rec_cap && threadIdx.x == 0) atomicExch(overflow, 1);
  const int m = min(n, rec_cap);
  for (int i = threadIdx.x; i < m; i += blockDim.x) {
    const int4 r = rec[static_cast<size_t>(c) * rec_cap + i];
    const int p = atomicAdd(&cand_n[r.x], 1);
    if (p < cap) {
      cand_s[static_cast<size_t>(r.x) * cap + p] = __int_as_float(r.z);
      cand_i[static_cast<size_t>(r.x) * cap + p] = row0 + r.y;
    }
  }
}

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
int scan_filter_max_queries() { return kFilterMaxThr; }
int scan_filter_record_cap() { return 32768; }
// A batch of at most 128 queries fills one 128-column tile: half the tensor-core work of a
// 256-column tile whose other half would score padding, which keeps the small-batch scan bound
// by the database stream from HBM.
int scan_filter_bn(int nq) { return nq <= 128 ? 128 : 256; }

cudaError_t scan_filter_block(const CUtensorMap& tm_rows, const CUtensorMap& tm_queries, int rows,
                              int dim, int64_t row0, int nq, int nq_pad, int kp, float* thr,
                              int4* rec, int* rec_n, int* cand_n, float* cand_s, int64_t* cand_i,
                              float* list_s, int64_t* list_i, int* list_n, int* overflow,
                              unsigned int* err, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  const int bn = scan_filter_bn(nq);
  if (nq_pad % bn != 0 || nq_pad > kFilterMaxThr || nq > nq_pad || dim % 64 != 0 || kp > kFilterMaxKp)
    return cudaErrorInvalidValue;
  const int cap = scan_filter_cap();
  const int rec_cap = scan_filter_record_cap();
  const int sms = device_sm_count();
  filter_prepare_kernel<<<(nq_pad + 255) / 256, 256, 0, st>>>(list_s, list_n, kp, nq, nq_pad, thr, cand_n);
  EpiTopKFilter epi{thr, rec, rec_n, rec_cap, nq_pad};
  cudaError_t e = bn == 128 ? launch_gemm_tc<__nv_bfloat16, 128>(tm_rows, tm_queries, rows, nq_pad, dim, 0,
                                                                  epi, err, sms, st)
                            : launch_gemm_tc<__nv_bfloat16, 256>(tm_rows, tm_queries, rows, nq_pad, dim, 0,
                                                                  epi, err, sms, st);
  if (e != cudaSuccess) return e;
  // The GEMM ran min(tiles, sms) persistent CTAs (launch_gemm_tc), each of which wrote rec_n.
  const int64_t tiles = (int64_t(rows) + kGemmBM - 1) / kGemmBM * (nq_pad / bn);
  const int grid = static_cast<int>(tiles < sms ? tiles : sms);
  filter_bucket_kernel<<<grid, 256, 0, st>>>(rec, rec_n, rec_cap, row0, cap, cand_n, cand_s, cand_i,
                                             overflow);
  int n = 1;
  while (n < cap + kp) n <<= 1;
  const size_t smem = size_t(n) * (sizeof(int64_t) + sizeof(float));
  static PerDeviceOnce attr_set;  // per-device attribute, set once under a lock
  {
    const cudaError_t e_once = attr_set.run([&]() -> cudaError_t {
      int nmax = 1;
      while (nmax < cap + kFilterMaxKp) nmax <<= 1;
      e = cudaFuncSetAttribute(filter_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(size_t(nmax) * (sizeof(int64_t) + sizeof(float))));
      if (e != cudaSuccess) return e;
      return cudaSuccess;
    });
    if (e_once != cudaSuccess) return e_once;
  }
  filter_merge_kernel<<<nq, 256, smem, st>>>(cand_s, cand_i, cand_n, cap, kp, list_s, list_i, list_n,
                                             overflow);
  return cudaGetLastError();
}

}  // namespace rv
