// Varlen bidirectional attention with global or sliding-window masking and online softmax,
// reading the packed QKV projection [T, 3H] directly (no padding, no per-head copies) and
// writing the context [T, H] in the layout the output projection consumes.
//
// One CTA = one (64-query tile of one sequence, head).  Four warps each own 16 query rows; K/V
// tiles of 64 keys are double-buffered in shared memory with cp.async; Q K^T and P V use
// m16n8k16 tensor-core MMAs with f32 accumulation; masked keys are skipped exactly (weight 0),
// and sliding-window tiles that lie outside [q0 - w, q0 + 63 + w] are never loaded.
//
// Reference semantics (crates/ripvec-core/src/backend/driver/cpu.rs): scores q.k * 1/sqrt(d)
// (backend/arch/modern_bert.rs:250-263), additive -1e9 mask for padding and, on local layers,
// for |i - j| > window/2 (driver/cpu.rs:1016-1074), max-subtracted softmax (:704-715), P V and
// head merge (modern_bert.rs:286-322).  Padding does not exist here, and exp(-1e9 - max) is
// exactly 0 in f32, so skipping masked keys reproduces the reference.
#include "common.cuh"
#include "kernels.h"

namespace rv {

namespace {

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)),
               "l"(gmem), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4],
                                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                 uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  auto v = Elem<T>::pack(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <typename T, int D>
__global__ void __launch_bounds__(128) attn_varlen_kernel(const T* __restrict__ qkv, T* __restrict__ ctx,
                                                          const int* __restrict__ cu,
                                                          const int* __restrict__ qts, int n_seqs,
                                                          int H, int window_half,
                                                          float scale_log2) {
  constexpr int BQ = 64, BKV = 64, LD = D + 8, CPR = D / 8;
  constexpr int NT = BKV / 8;  // score n-tiles per warp
  constexpr int KS = D / 16;   // k-steps over the head dim
  constexpr int NO = D / 8;    // output n-tiles
  __shared__ __align__(128) T sQ[BQ * LD];
  __shared__ __align__(128) T sK[2][BKV * LD];
  __shared__ __align__(128) T sV[2][BKV * LD];

  const int tile = blockIdx.x, h = blockIdx.y;
  int lo = 0, hi = n_seqs;  // last b with qts[b] <= tile
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (qts[mid] <= tile) lo = mid; else hi = mid;
  }
  const int b = lo;
  const int s0 = cu[b];
  const int L = cu[b + 1] - s0;
  const int q0 = (tile - qts[b]) * BQ;
  if (q0 >= L) return;
  const int ldq = 3 * H;
  const T* Qg = qkv + static_cast<size_t>(s0) * ldq + h * D;
  const T* Kg = Qg + H;
  const T* Vg = Qg + 2 * H;

  int kv_lo = 0, kv_hi = L;
  if (window_half >= 0) {
    kv_lo = max(0, q0 - window_half);
    kv_hi = min(L, q0 + BQ + window_half);
  }
  const int t_lo = kv_lo / BKV, t_hi = (kv_hi + BKV - 1) / BKV;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  for (int i = tid; i < BQ * CPR; i += 128) {
    const int r = i / CPR, c = i % CPR;
    const bool ok = q0 + r < L;
    cp_async16(&sQ[r * LD + c * 8], Qg + static_cast<size_t>(ok ? q0 + r : 0) * ldq + c * 8,
               ok ? 16 : 0);
  }
  auto load_kv = [&](int t, int buf) {
    const int k0 = t * BKV;
    for (int i = tid; i < BKV * CPR; i += 128) {
      const int r = i / CPR, c = i % CPR;
      const bool ok = k0 + r < L;
      const size_t off = static_cast<size_t>(ok ? k0 + r : 0) * ldq + c * 8;
      cp_async16(&sK[buf][r * LD + c * 8], Kg + off, ok ? 16 : 0);
      cp_async16(&sV[buf][r * LD + c * 8], Vg + off, ok ? 16 : 0);
    }
  };
  load_kv(t_lo, 0);
  cp_async_commit();

  float o[NO][4];
#pragma unroll
  for (int j = 0; j < NO; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_i[2] = {-INFINITY, -INFINITY};
  float l_i[2] = {0.f, 0.f};
  uint32_t qf[KS][4];

  const int row_a = q0 + warp * 16 + (lane >> 2);  // query index (within the sequence)
  const int row_b = row_a + 8;

  for (int t = t_lo; t < t_hi; ++t) {
    const int buf = (t - t_lo) & 1;
    if (t + 1 < t_hi) {
      load_kv(t + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (t == t_lo) {
#pragma unroll
      for (int ks = 0; ks < KS; ++ks)
        ldsm_x4(qf[ks], &sQ[(warp * 16 + (lane & 15)) * LD + ks * 16 + (lane >> 4) * 8]);
    }

    // S = Q K^T for this warp's 16 rows x 64 keys.
    float s[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
#pragma unroll
      for (int kp = 0; kp < KS / 2; ++kp) {
        uint32_t kb[4];
        ldsm_x4(kb, &sK[buf][(j * 8 + (lane & 7)) * LD + kp * 32 + (lane >> 3) * 8]);
        mma16816<T>(s[j], qf[2 * kp], kb[0], kb[1]);
        mma16816<T>(s[j], qf[2 * kp + 1], kb[2], kb[3]);
      }
    }

    // Mask, scale (log2 domain) and online softmax.
    const int k0 = t * BKV;
    float mx[2] = {m_i[0], m_i[1]};
#pragma unroll
    for (int j = 0; j < NT; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = k0 + j * 8 + 2 * (lane & 3) + (e & 1);
        const int qi = (e < 2) ? row_a : row_b;
        bool ok = key < L;
        if (window_half >= 0) ok = ok && abs(qi - key) <= window_half;
        const float v = ok ? s[j][e] * scale_log2 : -INFINITY;
        s[j][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float alpha[2], mu[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mu[r] = (mx[r] == -INFINITY) ? 0.f : mx[r];
      alpha[r] = exp2f(m_i[r] - mu[r]);
      m_i[r] = mx[r];
      l_i[r] *= alpha[r];
    }
#pragma unroll
    for (int j = 0; j < NO; ++j) {
      o[j][0] *= alpha[0];
      o[j][1] *= alpha[0];
      o[j][2] *= alpha[1];
      o[j][3] *= alpha[1];
    }
#pragma unroll
    for (int j = 0; j < NT; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float p = exp2f(s[j][e] - mu[e >> 1]);
        s[j][e] = p;
        l_i[e >> 1] += p;
      }
    }

    // O += P V.
#pragma unroll
    for (int kk = 0; kk < BKV / 16; ++kk) {
      uint32_t pa[4];
      pa[0] = pack2<T>(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack2<T>(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack2<T>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack2<T>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int jp = 0; jp < NO / 2; ++jp) {
        uint32_t vb[4];
        const int mtx = lane >> 3;
        ldsm_x4_t(vb, &sV[buf][(kk * 16 + (lane & 7) + 8 * (mtx & 1)) * LD + jp * 16 + 8 * (mtx >> 1)]);
        mma16816<T>(o[2 * jp], pa, vb[0], vb[1]);
        mma16816<T>(o[2 * jp + 1], pa, vb[2], vb[3]);
      }
    }
    __syncthreads();
  }

#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_i[r] += __shfl_xor_sync(0xffffffffu, l_i[r], 1);
    l_i[r] += __shfl_xor_sync(0xffffffffu, l_i[r], 2);
  }
  const float inv_a = l_i[0] > 0.f ? 1.0f / l_i[0] : 0.f;
  const float inv_b = l_i[1] > 0.f ? 1.0f / l_i[1] : 0.f;
  T* out = ctx + static_cast<size_t>(s0) * H + h * D + 2 * (lane & 3);
#pragma unroll
  for (int j = 0; j < NO; ++j) {
    if (row_a < L)
      *reinterpret_cast<uint32_t*>(out + static_cast<size_t>(row_a) * H + j * 8) =
          pack2<T>(o[j][0] * inv_a, o[j][1] * inv_a);
    if (row_b < L)
      *reinterpret_cast<uint32_t*>(out + static_cast<size_t>(row_b) * H + j * 8) =
          pack2<T>(o[j][2] * inv_b, o[j][3] * inv_b);
  }
}

template <typename T>
cudaError_t launch_attn(const void* qkv, void* ctx, const int* cu, const int* qts, int n_seqs,
                        int total_q_tiles, int num_heads, int head_dim, int window_half,
                        float scale, cudaStream_t st) {
  const float scale_log2 = scale * 1.4426950408889634f;
  dim3 grid(total_q_tiles, num_heads);
  if (head_dim == 64)
    attn_varlen_kernel<T, 64><<<grid, 128, 0, st>>>(static_cast<const T*>(qkv), static_cast<T*>(ctx),
                                                   cu, qts, n_seqs, num_heads * 64, window_half,
                                                   scale_log2);
  else if (head_dim == 32)
    attn_varlen_kernel<T, 32><<<grid, 128, 0, st>>>(static_cast<const T*>(qkv), static_cast<T*>(ctx),
                                                   cu, qts, n_seqs, num_heads * 32, window_half,
                                                   scale_log2);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace

cudaError_t attention_varlen(Act act, const void* qkv, void* ctx, const int* cu_seqlens,
                             const int* q_tile_starts, int n_seqs, int total_q_tiles,
                             int num_heads, int head_dim, int window_half, float scale,
                             cudaStream_t st) {
  if (total_q_tiles <= 0 || n_seqs <= 0) return cudaSuccess;
  if (act == Act::kBf16)
    return launch_attn<__nv_bfloat16>(qkv, ctx, cu_seqlens, q_tile_starts, n_seqs, total_q_tiles,
                                      num_heads, head_dim, window_half, scale, st);
  return launch_attn<__half>(qkv, ctx, cu_seqlens, q_tile_starts, n_seqs, total_q_tiles, num_heads,
                             head_dim, window_half, scale, st);
}

}  // namespace rv
