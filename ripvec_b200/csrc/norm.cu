// Memory-bound kernels of the encoder: positions, embedding + LayerNorm, LayerNorm, and the
// fused final-LayerNorm + segmented mean-pool + L2 normalisation.  One warp per token row for
// the LayerNorms (16-byte vector loads, shuffle reductions, f32 statistics); one CTA per
// sequence for pooling.
//
// Reference semantics (crates/ripvec-core/src/backend/driver/cpu.rs): LayerNorm :892-916 (mean,
// biased variance, 1/sqrt(var + eps), * gamma + beta), embedding gather :855-871, mean pool
// :1366-1390, L2 normalise :1392-1403 (x / norm, zero vector when norm == 0); ClassicBert
// embeddings backend/cpu.rs:232-272 and CLS pool + max(norm, 1e-12) backend/cpu.rs:736-745.
#include "common.cuh"
#include "kernels.h"

namespace rv {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void positions_kernel(const int* __restrict__ cu, int n, int total, int* __restrict__ pos) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= total) return;
  int lo = 0, hi = n;  // find the last b with cu[b] <= t
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (cu[mid] <= t) lo = mid; else hi = mid;
  }
  pos[t] = t - cu[lo];
}

// Embedding gather (+ optional learned position row and token-type row) then LayerNorm, all in
// f32; output 16-bit.  Hidden <= 768, multiple of 4.  One warp per token.
template <typename T>
__global__ void embed_ln_kernel(const int* __restrict__ ids, int total, const float* __restrict__ table,
                                int vocab, const float* __restrict__ gamma,
                                const float* __restrict__ beta, const float* __restrict__ pos_table,
                                const int* __restrict__ pos, const float* __restrict__ type_row,
                                int hidden, float eps, T* __restrict__ out, unsigned int* err) {
  constexpr int kMax = 6;  // float4 chunks per lane: 6 * 32 * 4 = 768
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= total) return;
  int id = ids[t];
  if (id < 0 || id >= vocab) {
    if (lane == 0) atomicOr(err, kErrBadShape);
    id = 0;
  }
  const int n4 = hidden >> 2;
  const float4* src = reinterpret_cast<const float4*>(table + static_cast<size_t>(id) * hidden);
  const float4* psrc =
      pos_table ? reinterpret_cast<const float4*>(pos_table + static_cast<size_t>(pos[t]) * hidden)
                : nullptr;
  const float4* tsrc = reinterpret_cast<const float4*>(type_row);
  float x[kMax][4];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kMax; ++i) {
    const int c = lane + 32 * i;
    if (c < n4) {
      float4 v = src[c];
      if (psrc) {
        const float4 p = psrc[c];
        v.x += p.x; v.y += p.y; v.z += p.z; v.w += p.w;
      }
      if (tsrc) {
        const float4 p = tsrc[c];
        v.x += p.x; v.y += p.y; v.z += p.z; v.w += p.w;
      }
      x[i][0] = v.x; x[i][1] = v.y; x[i][2] = v.z; x[i][3] = v.w;
      s += (v.x + v.y) + (v.z + v.w);
    }
  }
  const float mean = warp_sum(s) / static_cast<float>(hidden);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < kMax; ++i)
    if (lane + 32 * i < n4)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float d = x[i][j] - mean;
        q += d * d;
      }
  const float var = warp_sum(q) / static_cast<float>(hidden);
  const float inv_std = 1.0f / sqrtf(var + eps);
  using E = Elem<T>;
  using T2 = typename E::T2;
  T2* dst = reinterpret_cast<T2*>(out + static_cast<size_t>(t) * hidden);
#pragma unroll
  for (int i = 0; i < kMax; ++i) {
    const int c = lane + 32 * i;
    if (c < n4) {
      float o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        o[j] = (x[i][j] - mean) * inv_std * gamma[4 * c + j] + (beta ? beta[4 * c + j] : 0.f);
      dst[2 * c] = E::pack(o[0], o[1]);
      dst[2 * c + 1] = E::pack(o[2], o[3]);
    }
  }
}

// LayerNorm of 16-bit rows, hidden <= 768 and a multiple of 8.  One warp per row.
template <typename T>
__global__ void layernorm_kernel(const T* __restrict__ in, T* __restrict__ out, int rows, int hidden,
                                 const float* __restrict__ gamma, const float* __restrict__ beta,
                                 float eps) {
  constexpr int kMax = 3;  // 16-byte chunks per lane: 3 * 32 * 8 = 768
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const int n8 = hidden >> 3;
  const uint4* src = reinterpret_cast<const uint4*>(in + static_cast<size_t>(r) * hidden);
  float x[kMax][8];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kMax; ++i) {
    const int c = lane + 32 * i;
    if (c < n8) {
      unpack8<T>(src[c], x[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) s += x[i][j];
    }
  }
  const float mean = warp_sum(s) / static_cast<float>(hidden);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < kMax; ++i)
    if (lane + 32 * i < n8)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = x[i][j] - mean;
        q += d * d;
      }
  const float var = warp_sum(q) / static_cast<float>(hidden);
  const float inv_std = 1.0f / sqrtf(var + eps);
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(r) * hidden);
#pragma unroll
  for (int i = 0; i < kMax; ++i) {
    const int c = lane + 32 * i;
    if (c < n8) {
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        o[j] = (x[i][j] - mean) * inv_std * gamma[8 * c + j] + (beta ? beta[8 * c + j] : 0.f);
      dst[c] = pack8<T>(o);
    }
  }
}

// One CTA (8 warps) per sequence.  mode 0: LN(gamma) each token then mean; 1: mean; 2: first
// token.  Then L2 normalisation into out[b, :] (f32).
template <typename T>
__global__ void __launch_bounds__(256) pool_l2_kernel(const T* __restrict__ hs, const int* __restrict__ cu,
                                                      int hidden, int mode,
                                                      const float* __restrict__ gamma, float eps,
                                                      float l2_floor, float* __restrict__ out) {
  constexpr int kMax = 3;
  __shared__ float part[8][768];
  __shared__ float red[8];
  const int b = blockIdx.x;
  const int s0 = cu[b], s1 = cu[b + 1];
  const int L = s1 - s0;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n8 = hidden >> 3;
  float acc[kMax][8];
#pragma unroll
  for (int i = 0; i < kMax; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  const int t_end = (mode == 2) ? (L > 0 ? s0 + 1 : s0) : s1;
  for (int t = s0 + w; t < t_end; t += 8) {
    const uint4* src = reinterpret_cast<const uint4*>(hs + static_cast<size_t>(t) * hidden);
    float x[kMax][8];
#pragma unroll
    for (int i = 0; i < kMax; ++i)
      if (lane + 32 * i < n8) unpack8<T>(src[lane + 32 * i], x[i]);
    if (mode == 0) {
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < kMax; ++i)
        if (lane + 32 * i < n8)
#pragma unroll
          for (int j = 0; j < 8; ++j) s += x[i][j];
      const float mean = warp_sum(s) / static_cast<float>(hidden);
      float q = 0.f;
#pragma unroll
      for (int i = 0; i < kMax; ++i)
        if (lane + 32 * i < n8)
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float d = x[i][j] - mean;
            q += d * d;
          }
      const float inv_std = 1.0f / sqrtf(warp_sum(q) / static_cast<float>(hidden) + eps);
#pragma unroll
      for (int i = 0; i < kMax; ++i) {
        const int c = lane + 32 * i;
        if (c < n8)
#pragma unroll
          for (int j = 0; j < 8; ++j) x[i][j] = (x[i][j] - mean) * inv_std * gamma[8 * c + j];
      }
    }
#pragma unroll
    for (int i = 0; i < kMax; ++i)
      if (lane + 32 * i < n8)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] += x[i][j];
  }
#pragma unroll
  for (int i = 0; i < kMax; ++i) {
    const int c = lane + 32 * i;
    if (c < n8)
#pragma unroll
      for (int j = 0; j < 8; ++j) part[w][8 * c + j] = acc[i][j];
  }
  __syncthreads();
  const float inv_len = (mode == 2 || L == 0) ? (L > 0 ? 1.f : 0.f) : 1.0f / static_cast<float>(L);
  float ss = 0.f;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    float v = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) v += part[k][i];
    v *= inv_len;
    part[0][i] = v;
    ss += v * v;
  }
  ss = warp_sum(ss);
  if (lane == 0) red[w] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) tot += red[k];
  const float norm = sqrtf(tot);
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    const float v = part[0][i];
    float o;
    if (l2_floor > 0.f) o = v / fmaxf(norm, l2_floor);
    else o = v * (norm > 0.f ? 1.0f / norm : 0.f);
    out[static_cast<size_t>(b) * hidden + i] = o;
  }
}

template <typename T>
__global__ void convert_kernel(const float* __restrict__ in, T* __restrict__ out, int64_t n) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) out[i] = Elem<T>::from_f(in[i]);
}

}  // namespace

cudaError_t build_positions(const int* cu_seqlens, int n_seqs, int total, int* pos,
                            cudaStream_t st) {
  if (total <= 0) return cudaSuccess;
  positions_kernel<<<(total + 255) / 256, 256, 0, st>>>(cu_seqlens, n_seqs, total, pos);
  return cudaGetLastError();
}

cudaError_t embed_ln(Act act, const int* ids, int total, const float* table, int vocab,
                     const float* gamma, const float* beta, const float* pos_table,
                     const int* pos, const float* type_row, int hidden, float eps, void* out,
                     unsigned int* err, cudaStream_t st) {
  if (total <= 0) return cudaSuccess;
  if (hidden > 768 || hidden % 8 != 0) return cudaErrorInvalidValue;
  const int grid = (total + 7) / 8;
  if (act == Act::kBf16)
    embed_ln_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(ids, total, table, vocab, gamma, beta,
                                                         pos_table, pos, type_row, hidden, eps,
                                                         static_cast<__nv_bfloat16*>(out), err);
  else
    embed_ln_kernel<__half><<<grid, 256, 0, st>>>(ids, total, table, vocab, gamma, beta,
                                                  pos_table, pos, type_row, hidden, eps,
                                                  static_cast<__half*>(out), err);
  return cudaGetLastError();
}

cudaError_t layernorm(Act act, const void* in, void* out, int rows, int hidden,
                      const float* gamma, const float* beta, float eps, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  if (hidden > 768 || hidden % 8 != 0) return cudaErrorInvalidValue;
  const int grid = (rows + 7) / 8;
  if (act == Act::kBf16)
    layernorm_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(in), static_cast<__nv_bfloat16*>(out), rows, hidden,
        gamma, beta, eps);
  else
    layernorm_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(in),
                                                   static_cast<__half*>(out), rows, hidden, gamma,
                                                   beta, eps);
  return cudaGetLastError();
}

cudaError_t pool_l2(Act act, const void* hidden_states, const int* cu_seqlens, int n_seqs,
                    int hidden, int mode, const float* gamma, float eps, float l2_floor,
                    float* out, cudaStream_t st) {
  if (n_seqs <= 0) return cudaSuccess;
  if (hidden > 768 || hidden % 8 != 0) return cudaErrorInvalidValue;
  if (act == Act::kBf16)
    pool_l2_kernel<__nv_bfloat16><<<n_seqs, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(hidden_states), cu_seqlens, hidden, mode, gamma, eps,
        l2_floor, out);
  else
    pool_l2_kernel<__half><<<n_seqs, 256, 0, st>>>(static_cast<const __half*>(hidden_states),
                                                   cu_seqlens, hidden, mode, gamma, eps, l2_floor,
                                                   out);
  return cudaGetLastError();
}

cudaError_t convert_f32(Act act, const float* in, void* out, int64_t n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  const unsigned grid = static_cast<unsigned>((n + 255) / 256);
  if (act == Act::kBf16)
    convert_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(in, static_cast<__nv_bfloat16*>(out), n);
  else
    convert_kernel<__half><<<grid, 256, 0, st>>>(in, static_cast<__half*>(out), n);
  return cudaGetLastError();
}

}  // namespace rv
