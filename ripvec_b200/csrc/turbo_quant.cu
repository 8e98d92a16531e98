// PolarQuant ("TurboQuant") compressed scan on the GPU: the approximate first phase of
// SearchIndex::rank_turboquant (crates/ripvec-core/src/index.rs:196-234) over the codes of
// crates/ripvec-core/src/turbo_quant.rs.
//
// Codes.  Every row x (the bf16 values the index stores) is rotated, rotated = R x, and each
// pair (a, b) = (rotated[2i], rotated[2i+1]) becomes a radius r = sqrt(a*a + b*b) (f32) and an
// angle bin min(trunc((atan2(b, a) + PI) / (2 PI) * levels), levels - 1) (turbo_quant.rs:311-318).
// The rotation sums x_d * R[j][d] over d = 0..dim-1 in order, each product and sum rounded
// (no fused multiply-add); the angle is the f64 atan2 rounded to f32.  Both choices make the
// codes a pure function of the inputs, identical on the host and the device.
//
// Device layout, interleaved by groups of 32 rows (one warp reads one group): radii as float4
// [groups][pairs / 4][32] and bins as 16-byte words [groups][pairs / 16][32], so each load of a
// warp is one contiguous 512-byte segment.  4 + 1 bytes per pair, 1920 bytes per 768-d row,
// like the reference's SoA corpus (turbo_quant.rs:39-49).
//
// Scan.  One thread per row: score = sum_i r_i * table[i][bin_i], accumulated pair by pair in
// f32 with rounded products (turbo_quant.rs:248-289 adds in the same order), the query tables
// (turbo_quant.rs:212-241) in shared memory.  All scores of a query batch are written to a
// [nq, rows] f32 matrix (4 bytes per row next to the 1920 bytes of codes read).
//
// Selection.  The best `pre` rows per query by (approximate score desc, row asc) are found
// exactly: a radix select over order-preserving 32-bit keys (four passes of 8-bit histograms)
// gives the pre-th largest key T and how many rows of key T are needed; rows above T are
// collected, and the rows equal to T are sorted by row number and the lowest taken.
#include <float.h>

#include "common.cuh"
#include "scan_sort.cuh"
#include "tmap.h"
#include "turbo_quant.h"

namespace rv {

namespace {

constexpr float kPiF = 3.14159265358979323846f;  // the f32 nearest to pi
constexpr int kEncTile = 64;                      // rows and rotated columns per encode CTA
constexpr int kEncK = 16;                         // dimensions per shared-memory step

// ---------------------------------------------------------------- encode
// grid (ceil(n / 64), dim / 64), 256 threads: thread (ty, tx) owns rows ty*4..+3 and rotated
// columns tx*4..+3 (two pairs) of the CTA's 64 x 64 tile.  rt[d * dim + j] = R[j][d].
__global__ void __launch_bounds__(256) polar_encode_kernel(const __nv_bfloat16* __restrict__ x,
                                                           int64_t n, int dim,
                                                           const float* __restrict__ rt, int levels,
                                                           float* __restrict__ radii,
                                                           uint8_t* __restrict__ bins) {
  __shared__ __align__(16) float xs[kEncK][kEncTile + 4];
  __shared__ __align__(16) float rs[kEncK][kEncTile];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kEncTile;
  const int col0 = blockIdx.y * kEncTile;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  for (int k0 = 0; k0 < dim; k0 += kEncK) {
    {  // rows: 64 x 16 bf16, four per thread (one 8-byte load)
      const int r = threadIdx.x >> 2, dd = (threadIdx.x & 3) * 4;
      const int64_t row = row0 + r;
      float f[4] = {0.f, 0.f, 0.f, 0.f};
      if (row < n) {
        const uint2 u = *reinterpret_cast<const uint2*>(x + row * dim + k0 + dd);
        const __nv_bfloat162 p0 = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
        const __nv_bfloat162 p1 = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
        f[0] = __low2float(p0);
        f[1] = __high2float(p0);
        f[2] = __low2float(p1);
        f[3] = __high2float(p1);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) xs[dd + j][r] = f[j];
    }
    {  // rotation: 16 x 64 f32, one float4 per thread
      const int d = threadIdx.x >> 4, c = (threadIdx.x & 15) * 4;
      *reinterpret_cast<float4*>(&rs[d][c]) =
          *reinterpret_cast<const float4*>(rt + static_cast<size_t>(k0 + d) * dim + col0 + c);
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kEncK; ++kk) {
      const float4 av = *reinterpret_cast<const float4*>(&xs[kk][ty * 4]);
      const float4 bv = *reinterpret_cast<const float4*>(&rs[kk][tx * 4]);
      const float a[4] = {av.x, av.y, av.z, av.w};
      const float b[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a[i], b[j]));
    }
    __syncthreads();
  }
  const int pairs = dim / 2;
  const float two_pi = __fmul_rn(2.0f, kPiF);
  const float lv = static_cast<float>(levels);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t row = row0 + ty * 4 + i;
    if (row >= n) continue;
    const int64_t g = row >> 5;
    const int lane = static_cast<int>(row & 31);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float a = acc[i][2 * h], b = acc[i][2 * h + 1];
      const int p = (col0 + tx * 4) / 2 + h;
      const float r = __fsqrt_rn(__fadd_rn(__fmul_rn(a, a), __fmul_rn(b, b)));
      const float theta = __double2float_rn(atan2(static_cast<double>(b), static_cast<double>(a)));
      const float scaled = __fmul_rn(__fdiv_rn(__fadd_rn(theta, kPiF), two_pi), lv);
      int bin = __float2int_rz(scaled);
      bin = bin < 0 ? 0 : (bin > levels - 1 ? levels - 1 : bin);
      radii[((g * (pairs / 4) + p / 4) * 32 + lane) * 4 + (p & 3)] = r;
      bins[((g * (pairs / 16) + p / 16) * 32 + lane) * 16 + (p & 15)] = static_cast<uint8_t>(bin);
    }
  }
}

// ---------------------------------------------------------------- query tables
// grid (ceil(pairs / 128), nq), 128 threads: thread p of query blockIdx.y rotates its pair of
// the query (same order as the rows) and writes that pair's centroid table
// lut[q][p][j] = a_p * cos_j + b_p * sin_j (turbo_quant.rs:212-241).  The d loop is unrolled so
// that many rotation loads (L2-resident) are in flight ahead of the ordered sums.
__global__ void __launch_bounds__(128) polar_lut_kernel(const float* __restrict__ q, int dim,
                                                        const float* __restrict__ rt,
                                                        const float* __restrict__ cos_sin, int levels,
                                                        float* __restrict__ lut) {
  extern __shared__ float qs[];
  const int qi = blockIdx.y;
  const int pairs = dim / 2;
  for (int d = threadIdx.x; d < dim; d += blockDim.x) qs[d] = q[static_cast<size_t>(qi) * dim + d];
  __syncthreads();
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= pairs) return;
  float a = 0.f, b = 0.f;
  const float* col = rt + 2 * p;
  for (int d0 = 0; d0 < dim; d0 += 16) {  // dim is a multiple of 64
    float2 r[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) r[k] = *reinterpret_cast<const float2*>(col + static_cast<size_t>(d0 + k) * dim);
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      a = __fadd_rn(a, __fmul_rn(qs[d0 + k], r[k].x));
      b = __fadd_rn(b, __fmul_rn(qs[d0 + k], r[k].y));
    }
  }
  float* out = lut + (static_cast<size_t>(qi) * pairs + p) * levels;
  for (int j = 0; j < levels; ++j)
    out[j] = __fadd_rn(__fmul_rn(a, cos_sin[j]), __fmul_rn(b, cos_sin[levels + j]));
}

// ---------------------------------------------------------------- scan
// Threads per scan CTA: the 4-query tables (4 x 24 KB at 768 dims) allow two CTAs per SM and the
// 8-query tables (192 KB) one, so those variants run 16 and 32 warps per CTA to keep 32 warps of
// loads in flight per SM.
template <int QB>
constexpr int scan_threads() {
  return QB == 8 ? 1024 : QB == 4 ? 512 : 256;
}

// The QB table entries (queries 0..QB-1 of one pair and bin) in one or two shared loads.  slot()
// is where query qq of bin `bin` sits among the QB words of its entry: the 8-query tables swap
// their two 16-byte halves for the bins whose bit 2 is set, so that for each half the 16 bins of a
// pair fall on all eight 16-byte bank groups instead of four (a warp's lanes read random bins of
// the same pair, and two lanes on one bank group with different addresses serialise).
template <int QB>
struct QVec;
template <>
struct QVec<1> {
  __device__ __forceinline__ static int slot(int qq, int) { return qq; }
  __device__ __forceinline__ static void get(const float* p, int, float (&v)[1]) { v[0] = *p; }
};
template <>
struct QVec<2> {
  __device__ __forceinline__ static int slot(int qq, int) { return qq; }
  __device__ __forceinline__ static void get(const float* p, int, float (&v)[2]) {
    const float2 t = *reinterpret_cast<const float2*>(p);
    v[0] = t.x;
    v[1] = t.y;
  }
};
template <>
struct QVec<4> {
  __device__ __forceinline__ static int slot(int qq, int) { return qq; }
  __device__ __forceinline__ static void get(const float* p, int, float (&v)[4]) {
    const float4 t = *reinterpret_cast<const float4*>(p);
    v[0] = t.x;
    v[1] = t.y;
    v[2] = t.z;
    v[3] = t.w;
  }
};
template <>
struct QVec<8> {
  __device__ __forceinline__ static int slot(int qq, int bin) { return qq ^ (bin & 4); }
  __device__ __forceinline__ static void get(const float* p, int bin, float (&v)[8]) {
    const int sw = bin & 4;  // 0, or 4 when the halves are swapped
    const float4 a = *reinterpret_cast<const float4*>(p + sw);
    const float4 b = *reinterpret_cast<const float4*>(p + (4 - sw));
    v[0] = a.x;
    v[1] = a.y;
    v[2] = a.z;
    v[3] = a.w;
    v[4] = b.x;
    v[5] = b.y;
    v[6] = b.z;
    v[7] = b.w;
  }
};

// Warp w of the grid scores row groups g = w, w + warps, ... of [g_begin, g_begin + g_count):
// lane l owns row 32 g + l.  The QB queries of a pass share each loaded code word; their tables
// sit interleaved in shared memory, lut_s[(pair * levels + bin) * QB + QVec<QB>::slot(query, bin)],
// so one load (two for 8 queries) brings the entries of all QB queries.  Scores go to s[qq * ld + 32 (g - g_begin) + l] for the
// rows inside the first `valid` of the launch.
template <int QB>
__global__ void __launch_bounds__(scan_threads<QB>()) polar_scan_kernel(
    const float4* __restrict__ radii, const uint4* __restrict__ bins, int pairs, int64_t g_begin,
    int64_t g_count, int64_t valid, const float* __restrict__ lut, int levels, float* __restrict__ s,
    int64_t ld) {
  extern __shared__ __align__(16) float lut_s[];
  const int tab = pairs * levels;
#pragma unroll
  for (int qq = 0; qq < QB; ++qq)
    for (int r = threadIdx.x; r < tab; r += blockDim.x) lut_s[r * QB + QVec<QB>::slot(qq, r % levels)] = lut[qq * tab + r];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int p4n = pairs / 4, p16n = pairs / 16;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); g < g_count;
       g += warps) {
    const float4* rp = radii + (g_begin + g) * p4n * 32 + lane;
    const uint4* bp = bins + (g_begin + g) * p16n * 32 + lane;
    float acc[QB];
#pragma unroll
    for (int qq = 0; qq < QB; ++qq) acc[qq] = 0.f;
#pragma unroll 2
    for (int c = 0; c < p16n; ++c) {
      const uint4 bw = __ldcs(bp + c * 32);
      float4 rv4[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) rv4[k] = __ldcs(rp + (c * 4 + k) * 32);
      const uint32_t words[4] = {bw.x, bw.y, bw.z, bw.w};
      const float* row_tab = lut_s + c * 16 * levels * QB;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int code = (words[j >> 2] >> (8 * (j & 3))) & 0xff;
        const float4 r4 = rv4[j >> 2];
        const float rad = (j & 3) == 0 ? r4.x : (j & 3) == 1 ? r4.y : (j & 3) == 2 ? r4.z : r4.w;
        float t[QB];
        QVec<QB>::get(row_tab + (j * levels + code) * QB, code, t);
#pragma unroll
        for (int qq = 0; qq < QB; ++qq) acc[qq] = __fadd_rn(acc[qq], __fmul_rn(rad, t[qq]));
      }
    }
    const int64_t col = g * 32 + lane;
    if (col < valid) {
#pragma unroll
      for (int qq = 0; qq < QB; ++qq) s[qq * ld + col] = acc[qq];
    }
  }
}

// ---------------------------------------------------------------- exact selection of the best pre
// Order-preserving key: a larger float gives a larger unsigned key.
__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Per query: st[4q + 0] = key prefix found so far, + 1 = its mask, + 2 = rows still wanted
// among the keys that match the prefix (starts at pre).
__global__ void sel_init_kernel(uint32_t* st, int nq, int pre, uint32_t* hist) {
  const int q = blockIdx.x;
  if (threadIdx.x == 0) {
    st[4 * q + 0] = 0u;
    st[4 * q + 1] = 0u;
    st[4 * q + 2] = static_cast<uint32_t>(pre);
    st[4 * q + 3] = 0u;
  }
  hist[q * 256 + threadIdx.x] = 0u;
}

// Histogram of the digit at `shift` over the keys that match the prefix.  grid (x, nq).
__global__ void __launch_bounds__(256) sel_hist_kernel(const float* __restrict__ s, int64_t ld, int64_t n,
                                                       const uint32_t* __restrict__ st, int shift,
                                                       uint32_t* __restrict__ hist) {
  __shared__ uint32_t h[256];
  const int q = blockIdx.y;
  h[threadIdx.x] = 0u;
  __syncthreads();
  const uint32_t prefix = st[4 * q], mask = st[4 * q + 1];
  const float* row = s + q * ld;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t k = fkey(row[i]);
    if ((k & mask) == prefix) atomicAdd(&h[(k >> shift) & 0xffu], 1u);
  }
  __syncthreads();
  if (h[threadIdx.x]) atomicAdd(&hist[q * 256 + threadIdx.x], h[threadIdx.x]);
}

// Picks the digit holding the wanted-th largest key and narrows the prefix; clears the histogram.
__global__ void sel_pick_kernel(uint32_t* __restrict__ st, int shift, uint32_t* __restrict__ hist) {
  __shared__ uint32_t h[256];
  const int q = blockIdx.x;
  h[threadIdx.x] = hist[q * 256 + threadIdx.x];
  hist[q * 256 + threadIdx.x] = 0u;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t want = st[4 * q + 2];
    int b = 255;
    for (; b > 0; --b) {
      if (h[b] >= want) break;
      want -= h[b];
    }
    st[4 * q + 0] |= static_cast<uint32_t>(b) << shift;
    st[4 * q + 1] |= 0xffu << shift;
    st[4 * q + 2] = want;
  }
}

// Rows with key > T go to the list (their count is pre - wanted); rows with key == T go to the
// tie buffer (at most tie_cap kept, the count is recorded in full).  grid (x, nq).
__global__ void __launch_bounds__(256) sel_collect_kernel(const float* __restrict__ s, int64_t ld, int64_t n,
                                                          int64_t row_base, const uint32_t* __restrict__ st,
                                                          int pre, int64_t* __restrict__ list_i,
                                                          uint32_t* __restrict__ counters,
                                                          int64_t* __restrict__ ties, int tie_cap) {
  const int q = blockIdx.y;
  const uint32_t t = st[4 * q];
  const float* row = s + q * ld;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t k = fkey(row[i]);
    if (k > t) {
      const uint32_t p = atomicAdd(&counters[2 * q], 1u);
      if (p < static_cast<uint32_t>(pre)) list_i[static_cast<size_t>(q) * pre + p] = row_base + i;
    } else if (k == t) {
      const uint32_t p = atomicAdd(&counters[2 * q + 1], 1u);
      if (p < static_cast<uint32_t>(tie_cap)) ties[static_cast<size_t>(q) * tie_cap + p] = row_base + i;
    }
  }
}

// One CTA per query: the lowest `wanted` tie rows complete the list; list_n = pre.  Sets
// *overflow when more ties exist than the buffer holds (the selection would be incomplete).
__global__ void __launch_bounds__(256) sel_ties_kernel(const uint32_t* __restrict__ st,
                                                       const uint32_t* __restrict__ counters,
                                                       const int64_t* __restrict__ ties, int tie_cap,
                                                       int pre, int64_t* __restrict__ list_i,
                                                       int* __restrict__ list_n, int* __restrict__ overflow) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int q = blockIdx.x;
  const uint32_t wanted = st[4 * q + 2];
  const uint32_t m = counters[2 * q + 1];
  const int above = pre - static_cast<int>(wanted);
  if (m > static_cast<uint32_t>(tie_cap)) {
    if (threadIdx.x == 0) {
      atomicExch(overflow, 1);
      list_n[q] = above;
    }
    return;
  }
  int n2 = 1;
  while (n2 < static_cast<int>(m)) n2 <<= 1;
  int64_t* id = reinterpret_cast<int64_t*>(smem);
  double* key = reinterpret_cast<double*>(id + n2);
  for (int i = threadIdx.x; i < n2; i += blockDim.x) {
    const bool v = i < static_cast<int>(m);
    id[i] = v ? ties[static_cast<size_t>(q) * tie_cap + i] : INT64_MAX;
    key[i] = 0.0;  // equal keys: bitonic_sort orders by id ascending
  }
  bitonic_sort(key, id, n2);
  for (int i = threadIdx.x; i < static_cast<int>(wanted); i += blockDim.x)
    list_i[static_cast<size_t>(q) * pre + above + i] = id[i];
  if (threadIdx.x == 0) list_n[q] = pre;
}

// Every row is a candidate (n <= pre).
__global__ void sel_all_kernel(int64_t n, int64_t row_base, int pre, int nq, int64_t* __restrict__ list_i,
                               int* __restrict__ list_n) {
  const int q = blockIdx.y;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    list_i[static_cast<size_t>(q) * pre + i] = row_base + i;
  if (blockIdx.x == 0 && threadIdx.x == 0) list_n[q] = static_cast<int>(n);
}

int scan_qb(int pairs, int levels, int qn) {
  const size_t tab = size_t(pairs) * levels * sizeof(float);
  int qb = 8;
  while (qb > 1 && (qb > qn || tab * qb > kPolarMaxLutBytes)) qb >>= 1;
  return qb;
}

template <int QB>
cudaError_t launch_scan(const float* radii, const uint8_t* bins, int pairs, int64_t g_begin, int64_t g_count,
                        int64_t valid, const float* lut, int levels, float* s, int64_t ld, int sms,
                        cudaStream_t st) {
  const size_t smem = size_t(QB) * pairs * levels * sizeof(float);
  static PerDeviceOnce attr;  // per-device attribute, set once under a lock
  {
    const cudaError_t e_once = attr.run([&]() -> cudaError_t {
      cudaError_t e = cudaFuncSetAttribute(polar_scan_kernel<QB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(kPolarMaxLutBytes));
      if (e != cudaSuccess) return e;
      return cudaSuccess;
    });
    if (e_once != cudaSuccess) return e_once;
  }
  constexpr int threads = scan_threads<QB>();
  constexpr int warps_per_cta = threads / 32;
  const int64_t blocks_needed = (g_count + warps_per_cta - 1) / warps_per_cta;
  // One wave of persistent CTAs: as many per SM as the shared tables and threads allow.
  int per_sm = 0;
  cudaError_t oe = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, polar_scan_kernel<QB>, threads, smem);
  if (oe != cudaSuccess) return oe;
  const int64_t cap = int64_t(sms) * (per_sm > 0 ? per_sm : 1);
  const int grid = static_cast<int>(blocks_needed < cap ? blocks_needed : cap);
  polar_scan_kernel<QB><<<grid, threads, smem, st>>>(reinterpret_cast<const float4*>(radii),
                                                      reinterpret_cast<const uint4*>(bins), pairs, g_begin, g_count,
                                                      valid, lut, levels, s, ld);
  return cudaGetLastError();
}

}  // namespace

cudaError_t polar_encode(const __nv_bfloat16* x, int64_t n, int dim, const float* rt, int levels, float* radii,
                         uint8_t* bins, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  if (dim % 64 != 0) return cudaErrorInvalidValue;
  const int64_t tiles = (n + kEncTile - 1) / kEncTile;
  if (tiles > 0x7fffffffLL) return cudaErrorInvalidValue;
  dim3 grid(static_cast<unsigned>(tiles), static_cast<unsigned>(dim / kEncTile));
  polar_encode_kernel<<<grid, 256, 0, st>>>(x, n, dim, rt, levels, radii, bins);
  return cudaGetLastError();
}

cudaError_t polar_query_tables(const float* q, int nq, int dim, const float* rt, const float* cos_sin, int levels,
                               float* lut, cudaStream_t st) {
  if (nq <= 0) return cudaSuccess;
  if (nq > 65535) return cudaErrorInvalidValue;
  const size_t smem = size_t(dim) * sizeof(float);
  static PerDeviceOnce attr;  // per-device attribute, set once under a lock
  {
    const cudaError_t e_once = attr.run([&]() -> cudaError_t {
      cudaError_t e = cudaFuncSetAttribute(polar_lut_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           64 * 1024);
      if (e != cudaSuccess) return e;
      return cudaSuccess;
    });
    if (e_once != cudaSuccess) return e_once;
  }
  const dim3 grid(static_cast<unsigned>((dim / 2 + 127) / 128), static_cast<unsigned>(nq));
  polar_lut_kernel<<<grid, 128, smem, st>>>(q, dim, rt, cos_sin, levels, lut);
  return cudaGetLastError();
}

cudaError_t polar_scan(const float* radii, const uint8_t* bins, int pairs, int64_t row_begin, int64_t rows,
                       const float* lut, int nq, int levels, float* s, int64_t ld, cudaStream_t st) {
  if (rows <= 0 || nq <= 0) return cudaSuccess;
  if (row_begin % 32 != 0 || pairs % 16 != 0) return cudaErrorInvalidValue;
  const int sms = device_sm_count();
  const int64_t g_begin = row_begin / 32;
  const int64_t g_count = (rows + 31) / 32;
  const size_t tab = size_t(pairs) * levels;
  for (int q0 = 0; q0 < nq; ) {
    // scan_qb never exceeds the queries left, so every pass scores exactly qb queries.
    const int qb = scan_qb(pairs, levels, nq - q0);
    cudaError_t e;
    if (qb == 8)
      e = launch_scan<8>(radii, bins, pairs, g_begin, g_count, rows, lut + q0 * tab, levels, s + q0 * ld, ld, sms,
                         st);
    else if (qb == 4)
      e = launch_scan<4>(radii, bins, pairs, g_begin, g_count, rows, lut + q0 * tab, levels, s + q0 * ld, ld, sms,
                         st);
    else if (qb == 2)
      e = launch_scan<2>(radii, bins, pairs, g_begin, g_count, rows, lut + q0 * tab, levels, s + q0 * ld, ld, sms,
                         st);
    else
      e = launch_scan<1>(radii, bins, pairs, g_begin, g_count, rows, lut + q0 * tab, levels, s + q0 * ld, ld, sms,
                         st);
    if (e != cudaSuccess) return e;
    q0 += qb;
  }
  return cudaSuccess;
}

int polar_tie_cap() { return 8192; }

cudaError_t polar_select(const float* s, int64_t ld, int64_t n, int64_t row_base, int nq, int pre,
                         uint32_t* state, uint32_t* hist, uint32_t* counters, int64_t* ties, int64_t* list_i,
                         int* list_n, int* overflow, cudaStream_t st) {
  if (nq <= 0) return cudaSuccess;
  if (n <= pre) {
    dim3 grid(static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 1024))),
              static_cast<unsigned>(nq));
    sel_all_kernel<<<grid, 256, 0, st>>>(n, row_base, pre, nq, list_i, list_n);
    return cudaGetLastError();
  }
  const int sms = device_sm_count();
  sel_init_kernel<<<nq, 256, 0, st>>>(state, nq, pre, hist);
  const int64_t want_blocks = (n + 255) / 256;
  const unsigned gx = static_cast<unsigned>(std::min<int64_t>(want_blocks, std::max(1, (4 * sms) / nq + 1)));
  for (int shift = 24; shift >= 0; shift -= 8) {
    sel_hist_kernel<<<dim3(gx, nq), 256, 0, st>>>(s, ld, n, state, shift, hist);
    sel_pick_kernel<<<nq, 256, 0, st>>>(state, shift, hist);
  }
  cudaError_t e = cudaMemsetAsync(counters, 0, sizeof(uint32_t) * 2 * size_t(nq), st);
  if (e != cudaSuccess) return e;
  const int tie_cap = polar_tie_cap();
  sel_collect_kernel<<<dim3(gx, nq), 256, 0, st>>>(s, ld, n, row_base, state, pre, list_i, counters, ties,
                                                    tie_cap);
  const size_t smem = size_t(tie_cap) * (sizeof(int64_t) + sizeof(double));
  static PerDeviceOnce attr;  // per-device attribute, set once under a lock
  {
    const cudaError_t e_once = attr.run([&]() -> cudaError_t {
      e = cudaFuncSetAttribute(sel_ties_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (e != cudaSuccess) return e;
      return cudaSuccess;
    });
    if (e_once != cudaSuccess) return e_once;
  }
  sel_ties_kernel<<<nq, 256, smem, st>>>(state, counters, ties, tie_cap, pre, list_i, list_n, overflow);
  return cudaGetLastError();
}

}  // namespace rv
