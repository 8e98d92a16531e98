// Truncated, re-normalised embeddings for the two-phase MRL cascade search
// (crates/ripvec-core/src/index.rs:99-132 for the rows, :262-283 for the query).
//
// Per vector x of dim values: mean = (sum of x) / dim, var = (sum of (x - mean)^2) / dim,
// inv_std = 1 / sqrt(var + 1e-5), ln_j = (x_j - mean) * inv_std for the first t dimensions,
// norm = max(sqrt(sum of ln_j^2), 1e-12), out_j = ln_j / norm.  Every sum runs over the
// dimensions in order in f32 (the reference's iter().sum()), every operation rounded as written
// (no fused multiply-add), so the result is a pure function of the input on host and device.
//
// Rows: 32 rows per CTA, one thread per row over rows staged in shared memory with an odd word
// stride (conflict-free column reads), outputs staged the same way and written coalesced.
#include "cascade.h"
#include "common.cuh"
#include "tmap.h"

namespace rv {

namespace {

struct Stats {
  float mean, inv;
};

// Loader: value d of the vector.
template <class Get>
__device__ __forceinline__ Stats ln_stats(const Get& get, int dim) {
  float s = 0.f;
  for (int d = 0; d < dim; ++d) s = __fadd_rn(s, get(d));
  const float fd = static_cast<float>(dim);
  const float mean = __fdiv_rn(s, fd);
  float v = 0.f;
  for (int d = 0; d < dim; ++d) {
    const float c = __fsub_rn(get(d), mean);
    v = __fadd_rn(v, __fmul_rn(c, c));
  }
  const float var = __fdiv_rn(v, fd);
  return {mean, __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)))};
}

template <class Get>
__device__ __forceinline__ float ln_norm(const Get& get, const Stats& st, int t) {
  float nn = 0.f;
  for (int j = 0; j < t; ++j) {
    const float ln = __fmul_rn(__fsub_rn(get(j), st.mean), st.inv);
    nn = __fadd_rn(nn, __fmul_rn(ln, ln));
  }
  return fmaxf(__fsqrt_rn(nn), 1e-12f);
}

__global__ void __launch_bounds__(32) cascade_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t n,
                                                          int dim, int t, __nv_bfloat16* __restrict__ out) {
  extern __shared__ uint32_t sm[];
  const int w_in = dim / 2 + 1;   // odd word stride per staged input row
  const int w_out = t / 2 + 1;    // odd word stride per staged output row
  uint32_t* sin = sm;
  uint32_t* sout = sm + 32 * w_in;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * 32;
  const int lane = threadIdx.x;
  const uint32_t* src = reinterpret_cast<const uint32_t*>(x);
  for (int r = 0; r < 32; ++r) {
    const int64_t row = row0 + r;
    for (int k = lane; k < dim / 2; k += 32)
      sin[r * w_in + k] = row < n ? src[row * (dim / 2) + k] : 0u;
  }
  __syncwarp();
  const uint32_t* mine = sin + lane * w_in;
  auto get = [&](int d) -> float {
    const uint32_t w = mine[d >> 1];
    return __uint_as_float((d & 1) ? (w & 0xffff0000u) : (w << 16));
  };
  const Stats st = ln_stats(get, dim);
  const float norm = ln_norm(get, st, t);
  for (int j = 0; j < t; j += 2) {
    const float a = __fdiv_rn(__fmul_rn(__fsub_rn(get(j), st.mean), st.inv), norm);
    const float b = __fdiv_rn(__fmul_rn(__fsub_rn(get(j + 1), st.mean), st.inv), norm);
    const __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
    sout[lane * w_out + j / 2] = *reinterpret_cast<const uint32_t*>(&p);
  }
  __syncwarp();
  uint32_t* dst = reinterpret_cast<uint32_t*>(out);
  for (int r = 0; r < 32; ++r) {
    const int64_t row = row0 + r;
    if (row >= n) break;
    for (int k = lane; k < t / 2; k += 32) dst[row * (t / 2) + k] = sout[r * w_out + k];
  }
}

// One thread per query (f32 in, f32 out).
__global__ void cascade_queries_kernel(const float* __restrict__ q, int nq, int dim, int t, float* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nq) return;
  const float* v = q + static_cast<size_t>(i) * dim;
  auto get = [&](int d) -> float { return v[d]; };
  const Stats st = ln_stats(get, dim);
  const float norm = ln_norm(get, st, t);
  for (int j = 0; j < t; ++j)
    out[static_cast<size_t>(i) * t + j] = __fdiv_rn(__fmul_rn(__fsub_rn(v[j], st.mean), st.inv), norm);
}

}  // namespace

size_t cascade_rows_smem(int dim, int t) { return size_t(32) * (dim / 2 + 1 + t / 2 + 1) * sizeof(uint32_t); }

cudaError_t cascade_rows(const __nv_bfloat16* x, int64_t n, int dim, int t, __nv_bfloat16* out, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  if (dim % 2 != 0 || t % 2 != 0 || t > dim || t <= 0) return cudaErrorInvalidValue;
  const size_t smem = cascade_rows_smem(dim, t);
  if (smem > kCascadeMaxSmem) return cudaErrorInvalidValue;
  static PerDeviceOnce attr;  // per-device attribute, set once under a lock
  {
    const cudaError_t e_once = attr.run([&]() -> cudaError_t {
      cudaError_t e = cudaFuncSetAttribute(cascade_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(kCascadeMaxSmem));
      if (e != cudaSuccess) return e;
      return cudaSuccess;
    });
    if (e_once != cudaSuccess) return e_once;
  }
  const int64_t blocks = (n + 31) / 32;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
  cascade_rows_kernel<<<static_cast<unsigned>(blocks), 32, smem, st>>>(x, n, dim, t, out);
  return cudaGetLastError();
}

cudaError_t cascade_queries(const float* q, int nq, int dim, int t, float* out, cudaStream_t st) {
  if (nq <= 0) return cudaSuccess;
  cascade_queries_kernel<<<(nq + 63) / 64, 64, 0, st>>>(q, nq, dim, t, out);
  return cudaGetLastError();
}

}  // namespace rv
