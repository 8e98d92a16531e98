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

__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// Folded LayerNorm of four values, two per instruction: rstd * (v - mu * c) evaluated as
// v * rstd + (-rstd * mu) * c (r2 = {rstd, rstd}, nm2 = {-rstd * mu, -rstd * mu}).
__device__ __forceinline__ void ln_fold4(float* v, const float4 c, uint64_t r2, uint64_t nm2) {
  uint64_t a = f2_fma(f2_pack(v[0], v[1]), r2, f2_mul(nm2, f2_pack(c.x, c.y)));
  uint64_t b = f2_fma(f2_pack(v[2], v[3]), r2, f2_mul(nm2, f2_pack(c.z, c.w)));
  f2_unpack(a, v[0], v[1]);
  f2_unpack(b, v[2], v[3]);
}

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
      const float nm = -t.rstd * t.mu;
      const uint64_t r2 = f2_pack(t.rstd, t.rstd), nm2 = f2_pack(nm, nm);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        ln_fold4(&v0[4 * i], cs[i], r2, nm2);
        ln_fold4(&v1[4 * i], cs[8 + i], r2, nm2);
      }
    }
    if (col < rope_cols) {
      // (f, s) -> (f cc - s ss, f ss + s cc), two columns per instruction.
      const uint64_t m1 = f2_pack(-1.f, -1.f);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 c = t.cv[i], n = t.sv[i];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint64_t cc = h ? f2_pack(c.z, c.w) : f2_pack(c.x, c.y);
          const uint64_t ss = h ? f2_pack(n.z, n.w) : f2_pack(n.x, n.y);
          const uint64_t f = f2_pack(v0[4 * i + 2 * h], v0[4 * i + 2 * h + 1]);
          const uint64_t s = f2_pack(v1[4 * i + 2 * h], v1[4 * i + 2 * h + 1]);
          const uint64_t o0 = f2_fma(f2_mul(s, ss), m1, f2_mul(f, cc));
          const uint64_t o1 = f2_fma(f, ss, f2_mul(s, cc));
          f2_unpack(o0, v0[4 * i + 2 * h], v0[4 * i + 2 * h + 1]);
          f2_unpack(o1, v1[4 * i + 2 * h], v1[4 * i + 2 * h + 1]);
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
    const float nm = -t.rstd * t.mu;
    const uint64_t r2 = f2_pack(t.rstd, t.rstd), nm2 = f2_pack(nm, nm);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      ln_fold4(&v0[4 * i], cs[i], r2, nm2);
      ln_fold4(&v1[4 * i], cs[8 + i], r2, nm2);
#pragma unroll
      for (int j = 0; j < 4; ++j) v0[4 * i + j] = gelu_tanh_fast(v0[4 * i + j]) * v1[4 * i + j];
    }
  }
};

}  // namespace rv
