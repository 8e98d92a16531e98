// Exact cosine top-k over a bf16 embedding matrix (the GPU replacement of
// crates/ripvec-core/src/similarity.rs:24-26 rank_all + index.rs:172-186 SearchIndex::rank).
//
// Pipeline per query batch:
//   1. queries f32 -> bf16 (same rounding as the stored rows);
//   2. for each chunk of database rows, the tcgen05 GEMM writes f32 scores S[nq, chunk]
//      (chunks sized so S stays in L2);
//   3. select: one CTA per query keeps a running top-kp list (f32 score desc, row asc) in global
//      memory; rows of the chunk scoring strictly above the list's current kp-th score are
//      compacted into shared memory, merged with the list by a bitonic sort and written back;
//   4. rescore: the kp candidates are re-scored exactly (sequential f64 sum of the exact
//      bf16 x bf16 products over d = 0..dim-1), sorted by (f64 score desc, row asc), and the best
//      k are written.  A margin guard proves that no row outside the candidates can enter the
//      top k given the f32 error bound; queries that fail it are redone with a wider kp.
#include <float.h>

#include "common.cuh"
#include "scan.h"
#include "scan_sort.cuh"
#include "tmap.h"

namespace rv {

namespace {

__global__ void round_bf16_kernel(const float* __restrict__ in, __nv_bfloat16* __restrict__ out,
                                  int64_t n) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) out[i] = __float2bfloat16_rn(in[i]);
}

__device__ __forceinline__ int block_sum(int v, int* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  int t = 0;
  for (int i = 0; i < (blockDim.x >> 5); ++i) t += red[i];
  return t;
}

// One CTA per query.  scores: [nq, ld] f32, valid columns [0, cols) = rows row0 + j.
// list_s / list_i: [nq, kp] sorted best first, list_n[q] entries valid.  cap: shared capacity
// (power of two >= 2 * kp).
__global__ void __launch_bounds__(256) select_kernel(const float* __restrict__ scores, int ld,
                                                     int cols, int64_t row0, int kp, int cap,
                                                     float* __restrict__ list_s,
                                                     int64_t* __restrict__ list_i,
                                                     int* __restrict__ list_n) {
  extern __shared__ __align__(16) unsigned char smem[];
  int64_t* cid = reinterpret_cast<int64_t*>(smem);
  float* cs = reinterpret_cast<float*>(cid + cap);
  __shared__ int red[8];
  __shared__ int counter;
  __shared__ float tau_s;
  const int q = blockIdx.x;
  const float* row = scores + static_cast<size_t>(q) * ld;
  float* ls = list_s + static_cast<size_t>(q) * kp;
  int64_t* li = list_i + static_cast<size_t>(q) * kp;
  int n_list = list_n[q];
  float tau = (n_list == kp) ? ls[kp - 1] : -INFINITY;

  int cnt = 0;
  for (int j = threadIdx.x; j < cols; j += blockDim.x) cnt += (row[j] > tau) ? 1 : 0;
  const int total = block_sum(cnt, red);
  if (total == 0) return;

  // Process the chunk in pieces whose survivors always fit next to the list.
  const int piece = (total + n_list <= cap) ? cols : (cap - kp);
  for (int base = 0; base < cols; base += piece) {
    const int end = min(cols, base + piece);
    if (threadIdx.x == 0) counter = 0;
    __syncthreads();
    for (int j = base + threadIdx.x; j < end; j += blockDim.x) {
      const float v = row[j];
      if (v > tau) {
        const int p = atomicAdd(&counter, 1);
        cs[p] = v;
        cid[p] = row0 + j;
      }
    }
    __syncthreads();
    const int m = counter;
    if (m == 0) continue;
    for (int i = threadIdx.x; i < n_list; i += blockDim.x) {
      cs[m + i] = ls[i];
      cid[m + i] = li[i];
    }
    int n = 1;
    while (n < m + n_list) n <<= 1;
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
    n_list = keep;
    if (threadIdx.x == 0) tau_s = (keep == kp) ? cs[kp - 1] : -INFINITY;
    __syncthreads();
    tau = tau_s;
  }
  if (threadIdx.x == 0) list_n[q] = n_list;
}

// One CTA per query: exact f64 rescoring of the candidate list, sort, guard, output of the
// best k.  qb: bf16 queries [nq, dim]; db: bf16 rows [n, dim] (global row r at db + (r - base)).
__global__ void __launch_bounds__(256) rescore_kernel(
    const __nv_bfloat16* __restrict__ db, int64_t base, int dim, const __nv_bfloat16* __restrict__ qb,
    const float* __restrict__ list_s, const int64_t* __restrict__ list_i,
    const int* __restrict__ list_n, int kp, int k, int64_t n_rows, double eps_scale, float threshold,
    int64_t* __restrict__ out_i, float* __restrict__ out_s, double* __restrict__ out_s64,
    int* __restrict__ out_cnt, int* __restrict__ guard_fail, int cap) {
  extern __shared__ __align__(16) unsigned char smem[];
  int64_t* cid = reinterpret_cast<int64_t*>(smem);
  double* cs = reinterpret_cast<double*>(cid + cap);
  float* qf = reinterpret_cast<float*>(cs + cap);
  __shared__ double qnorm2;
  const int q = blockIdx.x;
  const int n_list = list_n[q];
  const float* ls = list_s + static_cast<size_t>(q) * kp;
  const int64_t* li = list_i + static_cast<size_t>(q) * kp;
  for (int d = threadIdx.x; d < dim; d += blockDim.x)
    qf[d] = __bfloat162float(qb[static_cast<size_t>(q) * dim + d]);
  if (threadIdx.x == 0) qnorm2 = 0.0;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int d = 0; d < dim; ++d) s += double(qf[d]) * double(qf[d]);
    qnorm2 = s;
  }
  for (int c = threadIdx.x; c < n_list; c += blockDim.x) {
    const int64_t r = li[c];
    const __nv_bfloat16* rowp = db + static_cast<size_t>(r - base) * dim;
    double acc = 0.0;
    // Unrolled so that several 16-byte row loads are in flight ahead of the ordered f64 sum.
#pragma unroll 8
    for (int d = 0; d < dim; d += 8) {
      const uint4 u = *reinterpret_cast<const uint4*>(rowp + d);
      float f[8];
      unpack8<__nv_bfloat16>(u, f);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc = fma(double(f[j]), double(qf[d + j]), acc);
    }
    cs[c] = acc;
    cid[c] = r;
  }
  int n = 1;
  while (n < n_list) n <<= 1;
  for (int i = n_list + threadIdx.x; i < n; i += blockDim.x) {
    cs[i] = -DBL_MAX;
    cid[i] = INT64_MAX;
  }
  bitonic_sort(cs, cid, n);
  const int keep = min(k, n_list);
  int kept = 0;
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    int64_t oi = -1;
    float os = -INFINITY;
    double os64 = -INFINITY;
    if (i < keep && cs[i] >= double(threshold)) {
      oi = cid[i];
      os = float(cs[i]);
      os64 = cs[i];
    }
    out_i[static_cast<size_t>(q) * k + i] = oi;
    out_s[static_cast<size_t>(q) * k + i] = os;
    if (out_s64) out_s64[static_cast<size_t>(q) * k + i] = os64;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < keep; ++i)
      if (cs[i] >= double(threshold)) ++kept;
    out_cnt[q] = kept;
    // Guard: when the list is full (more rows exist than candidates), every row outside it has
    // an f32 score <= ls[kp-1], hence an exact score <= ls[kp-1] + eps.  The k-th exact score
    // must lie strictly above that bound.
    int fail = 0;
    if (n_list == kp && n_rows > kp && keep == k) {
      const double eps = eps_scale * sqrt(qnorm2);
      if (!(cs[k - 1] > double(ls[kp - 1]) + eps)) fail = 1;
    }
    guard_fail[q] = fail;
  }
}

// max over rows of the squared L2 norm (f32), as float bits through atomicMax (values >= 0).
__global__ void row_norm_max_kernel(const __nv_bfloat16* __restrict__ db, int64_t n, int dim,
                                    unsigned int* __restrict__ max_bits) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= n) return;
  const __nv_bfloat16* p = db + static_cast<size_t>(r) * dim;
  float s = 0.f;
  for (int d = lane * 8; d < dim; d += 256) {
    float f[8];
    unpack8<__nv_bfloat16>(*reinterpret_cast<const uint4*>(p + d), f);
#pragma unroll
    for (int j = 0; j < 8; ++j) s += f[j] * f[j];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) atomicMax(max_bits, __float_as_uint(s));
}

__global__ void init_lists_kernel(int* list_n, int nq) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < nq) list_n[i] = 0;
}

// Merge of per-shard results [n_lists, nq, k] (f64 scores) by (score desc, idx asc).
__global__ void __launch_bounds__(256) merge_kernel(const int64_t* __restrict__ idx_in,
                                                    const double* __restrict__ s_in, int n_lists,
                                                    int nq, int k, float threshold,
                                                    int64_t* __restrict__ idx_out,
                                                    float* __restrict__ s_out,
                                                    double* __restrict__ s64_out, int cap) {
  extern __shared__ __align__(16) unsigned char smem[];
  int64_t* cid = reinterpret_cast<int64_t*>(smem);
  double* cs = reinterpret_cast<double*>(cid + cap);
  const int q = blockIdx.x;
  const int m = n_lists * k;
  for (int i = threadIdx.x; i < cap; i += blockDim.x) {
    if (i < m) {
      const int l = i / k, j = i % k;
      const size_t off = (static_cast<size_t>(l) * nq + q) * k + j;
      const int64_t id = idx_in[off];
      cid[i] = id < 0 ? INT64_MAX : id;
      cs[i] = id < 0 ? -DBL_MAX : s_in[off];
    } else {
      cid[i] = INT64_MAX;
      cs[i] = -DBL_MAX;
    }
  }
  bitonic_sort(cs, cid, cap);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const bool ok = cid[i] != INT64_MAX && cs[i] >= double(threshold);
    idx_out[static_cast<size_t>(q) * k + i] = ok ? cid[i] : -1;
    s_out[static_cast<size_t>(q) * k + i] = ok ? float(cs[i]) : -INFINITY;
    if (s64_out) s64_out[static_cast<size_t>(q) * k + i] = ok ? cs[i] : -INFINITY;
  }
}

}  // namespace

int scan_cap_for(int kp) {
  int cap = 4096;
  while (cap < 2 * kp) cap <<= 1;
  return cap;
}

cudaError_t scan_round_queries(const float* q, __nv_bfloat16* out, int64_t n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  round_bf16_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(q, out, n);
  return cudaGetLastError();
}

cudaError_t scan_row_norm_max(const __nv_bfloat16* db, int64_t n, int dim, unsigned int* max_bits,
                              cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  row_norm_max_kernel<<<static_cast<unsigned>((n + 7) / 8), 256, 0, st>>>(db, n, dim, max_bits);
  return cudaGetLastError();
}

cudaError_t scan_init_lists(int* list_n, int nq, cudaStream_t st) {
  init_lists_kernel<<<(nq + 255) / 256, 256, 0, st>>>(list_n, nq);
  return cudaGetLastError();
}

cudaError_t scan_select(const float* scores, int ld, int cols, int64_t row0, int nq, int kp,
                        float* list_s, int64_t* list_i, int* list_n, cudaStream_t st) {
  const int cap = scan_cap_for(kp);
  const size_t smem = static_cast<size_t>(cap) * (8 + 4);
  static PerDeviceOnce attr;  // per-device attribute, set once under a lock
  {
    const cudaError_t e_once = attr.run([&]() -> cudaError_t {
      return cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    });
    if (e_once != cudaSuccess) return e_once;
  }
  select_kernel<<<nq, 256, smem, st>>>(scores, ld, cols, row0, kp, cap, list_s, list_i, list_n);
  return cudaGetLastError();
}

cudaError_t scan_rescore(const __nv_bfloat16* db, int64_t base, int dim, const __nv_bfloat16* qb,
                         int nq, const float* list_s, const int64_t* list_i, const int* list_n,
                         int kp, int k, int64_t n_rows, double eps_scale, float threshold,
                         int64_t* out_i, float* out_s, double* out_s64, int* out_cnt,
                         int* guard_fail, cudaStream_t st) {
  int cap = 1;
  while (cap < kp) cap <<= 1;
  const size_t smem = static_cast<size_t>(cap) * 16 + static_cast<size_t>(dim) * 4;
  static PerDeviceOnce attr;  // per-device attribute, set once under a lock
  {
    const cudaError_t e_once = attr.run([&]() -> cudaError_t {
      return cudaFuncSetAttribute(rescore_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    });
    if (e_once != cudaSuccess) return e_once;
  }
  rescore_kernel<<<nq, 256, smem, st>>>(db, base, dim, qb, list_s, list_i, list_n, kp, k, n_rows,
                                        eps_scale, threshold, out_i, out_s, out_s64, out_cnt,
                                        guard_fail, cap);
  return cudaGetLastError();
}

cudaError_t scan_merge(const int64_t* idx_in, const double* s_in, int n_lists, int nq, int k,
                       float threshold, int64_t* idx_out, float* s_out, double* s64_out,
                       cudaStream_t st) {
  int cap = 1;
  while (cap < n_lists * k) cap <<= 1;
  const size_t smem = static_cast<size_t>(cap) * 16;
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  static PerDeviceOnce attr;  // per-device attribute, set once under a lock
  {
    const cudaError_t e_once = attr.run([&]() -> cudaError_t {
      return cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    });
    if (e_once != cudaSuccess) return e_once;
  }
  merge_kernel<<<nq, 256, smem, st>>>(idx_in, s_in, n_lists, nq, k, threshold, idx_out, s_out,
                                      s64_out, cap);
  return cudaGetLastError();
}

}  // namespace rv
