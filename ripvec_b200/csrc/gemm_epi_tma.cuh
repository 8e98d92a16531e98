// Epilogue functors for the TMA-staged epilogue of the two-CTA GEMM (gemm_tc2_tma_kernel).
//
// The kernel moves data; the functor only computes.  For one output row and one group of 64
// accumulator columns it receives v0 (columns col..col+31) and v1 (col+32..col+63) in f32 and,
// when kReadsC, the 64 current values of the output row (the residual) already read from shared
// memory; it leaves its kOutCols results in v0 (then v1).  The kernel packs them into the staging
// tile and a single thread writes the tile with a TMA store, so the epilogue threads never wait
// on global memory.
#pragma once

#include "gemm_ln_epi.cuh"

namespace rv {

// tanh-GELU through the identity 0.5 (1 + tanh(y)) = 1 / (1 + e^(-2y)):
// gelu(x) = x / (1 + 2^(-2 log2(e) y)), y = sqrt(2/pi) (x + 0.044715 x^3).  The hardware base-2
// exponential and reciprocal (ex2.approx, rcp.approx) give it to about 1e-6 relative over the
// whole range, far below the 16-bit rounding of the stored result, in a handful of instructions
// (tanhf costs several times more, and 1 + tanh(y) would cancel for negative x).
__device__ __forceinline__ float gelu_tanh_fast(float x) {
  const float k = -2.0f * 1.4426950408889634f * 0.7978845608028654f;  // -2 log2(e) sqrt(2/pi)
  const float t = k * (x + 0.044715f * x * x * x);
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(t));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + e));
  return x * r;
}

// x <- x + acc, then LayerNorm partials of the stored (rounded) row per 256-column tile.
template <typename T>
struct TEpiResidualStats {
  float2* stats;
  int stats_ld;
  static constexpr int kOutCols = 64;
  static constexpr bool kReadsC = true;
  struct Tile {
    float n, mean, m2;
  };
  __device__ __forceinline__ void stage(float*, int, int) {}
  __device__ __forceinline__ void tile_load(Tile& t, int, int) const {
    t.n = 0.f;
    t.mean = 0.f;
    t.m2 = 0.f;
  }
  __device__ __forceinline__ void compute(Tile& t, int row, int col, const float* r, float (&v0)[32],
                                          float (&v1)[32], bool live) const {
    // The 64 stored (rounded) values of this group, their mean and M2 (two passes, four partial
    // sums each), then one pairwise (Chan) merge into the tile's running (n, mean, M2).
    float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float* v = (i < 4) ? &v0[8 * i] : &v1[8 * (i - 4)];
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[j] + r[8 * i + j];
      unpack8<T>(pack8<T>(o), o);  // the values as they will be stored
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[j] = o[j];
        s4[j & 3] += o[j];
      }
    }
    const float m = ((s4[0] + s4[1]) + (s4[2] + s4[3])) * (1.0f / 64.0f);
    float q4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      const float d = (i < 32 ? v0[i] : v1[i - 32]) - m;
      q4[i & 3] = fmaf(d, d, q4[i & 3]);
    }
    const float q = (q4[0] + q4[1]) + (q4[2] + q4[3]);
    const float tot = t.n + 64.f;
    const float w = 64.f / tot;
    const float d = m - t.mean;
    t.mean += d * w;
    t.m2 += q + d * d * (t.n * w);
    t.n = tot;
    if (live && (col & 255) == 192)
      stats[static_cast<size_t>(row) * stats_ld + (col >> 8)] = make_float2(t.mean, t.m2);
  }
};

// Rotary embedding of the Q / K heads (columns < rope_cols), optionally after a folded LayerNorm.
template <typename T, bool kNorm>
struct TEpiQkv {
  int rope_cols;
  const int* pos;
  const float* cos_t;
  const float* sin_t;
  LnFold ln;
  float* cs_smem = nullptr;
  static constexpr int kOutCols = 64;
  static constexpr bool kReadsC = false;
  struct Tile {
    float4 cv[8], sv[8];
    float mu, rstd;
  };
  __device__ __forceinline__ void stage(float* s, int t, int nt) {
    if (kNorm) {
      ln.stage_into(s, t, nt);
      cs_smem = s;
    }
  }
  __device__ __forceinline__ void tile_load(Tile& t, int row, int n0) const {
    if (n0 < rope_cols) {
      const int p = pos[row];
      const float4* cs = reinterpret_cast<const float4*>(cos_t + static_cast<size_t>(p) * 32);
      const float4* sn = reinterpret_cast<const float4*>(sin_t + static_cast<size_t>(p) * 32);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        t.cv[i] = cs[i];
        t.sv[i] = sn[i];
      }
    }
    if (kNorm) row_stats(ln.stats + static_cast<size_t>(row) * ln.stats_ld, ln.stats_n, ln.eps, t.mu, t.rstd);
  }
  __device__ __forceinline__ void compute(Tile& t, int, int col, const float*, float (&v0)[32],
                                          float (&v1)[32], bool) const {
    if (kNorm) {
      const float4* cs = reinterpret_cast<const float4*>(cs_smem + col);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 c0 = cs[i], c1 = cs[8 + i];
        const float ca[4] = {c0.x, c0.y, c0.z, c0.w}, cb[4] = {c1.x, c1.y, c1.z, c1.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          v0[4 * i + j] = t.rstd * (v0[4 * i + j] - t.mu * ca[j]);
          v1[4 * i + j] = t.rstd * (v1[4 * i + j] - t.mu * cb[j]);
        }
      }
    }
    if (col < rope_cols) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float cc[4] = {t.cv[i].x, t.cv[i].y, t.cv[i].z, t.cv[i].w};
        const float ss[4] = {t.sv[i].x, t.sv[i].y, t.sv[i].z, t.sv[i].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float f = v0[4 * i + j], s = v1[4 * i + j];
          v0[4 * i + j] = f * cc[j] - s * ss[j];
          v1[4 * i + j] = f * ss[j] + s * cc[j];
        }
      }
    }
  }
};

// Folded LayerNorm, then GeGLU over the interleaved value (v0) / gate (v1) halves; the 32 results
// are left in v0.
template <typename T>
struct TEpiNormGeglu {
  LnFold ln;
  float* cs_smem = nullptr;
  static constexpr int kOutCols = 32;
  static constexpr bool kReadsC = false;
  struct Tile {
    float mu, rstd;
  };
  __device__ __forceinline__ void stage(float* s, int t, int nt) {
    ln.stage_into(s, t, nt);
    cs_smem = s;
  }
  __device__ __forceinline__ void tile_load(Tile& t, int row, int) const {
    row_stats(ln.stats + static_cast<size_t>(row) * ln.stats_ld, ln.stats_n, ln.eps, t.mu, t.rstd);
  }
  __device__ __forceinline__ void compute(Tile& t, int, int col, const float*, float (&v0)[32],
                                          float (&v1)[32], bool) const {
    const float4* cs = reinterpret_cast<const float4*>(cs_smem + col);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 c0 = cs[i], c1 = cs[8 + i];
      const float ca[4] = {c0.x, c0.y, c0.z, c0.w}, cb[4] = {c1.x, c1.y, c1.z, c1.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = t.rstd * (v0[4 * i + j] - t.mu * ca[j]);
        const float g = t.rstd * (v1[4 * i + j] - t.mu * cb[j]);
        v0[4 * i + j] = gelu_tanh_fast(a) * g;
      }
    }
  }
};

}  // namespace rv
