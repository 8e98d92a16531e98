// Epilogues that fold the pre-attention and pre-MLP LayerNorms of ModernBERT into the projection
// GEMMs, so no separate LayerNorm pass over the residual stream is needed.
//
// LN(x) W^T with LN(x)_k = (x_k - mu) * rstd * gamma_k equals rstd * (x W'^T - mu * c) where
// W' = W diag(gamma) (folded on the host) and c_n = sum_k W'_nk.  So the GEMM multiplies the raw
// residual row x (bf16, as stored) and the epilogue applies rstd and mu per row.  The row
// statistics come from the GEMM that wrote x: its residual epilogue reduces each 256-column tile
// of the stored (rounded) row to (mean, M2) with Chan's pairwise update, and the consuming
// epilogue merges the tiles' partials the same way, so the variance is the two-pass biased
// variance of the reference LayerNorm (backend/driver/cpu.rs:892-916), not E[x^2] - mu^2.
#pragma once

#include "gemm_tc.cuh"

namespace rv {

// Merges the per-256-column (mean, M2) partials of one row into (mu, rstd).
__device__ __forceinline__ void row_stats(const float2* __restrict__ st, int n_parts, float eps,
                                          float& mu, float& rstd) {
  float mean = 0.f, m2 = 0.f, n = 0.f;
  for (int i = 0; i < n_parts; ++i) {
    const float2 p = st[i];
    const float nb = 256.f, tot = n + nb;
    const float d = p.x - mean;
    mean += d * (nb / tot);
    m2 += p.y + d * d * (n * nb / tot);
    n = tot;
  }
  mu = mean;
  rstd = 1.0f / sqrtf(m2 / n + eps);
}

// Residual add that also emits the LayerNorm partials of the updated row: x <- x + acc, and for
// every 256-column tile (mean, M2) of the rounded values into stats[row * stats_ld + col / 256].
template <typename T>
struct EpiResidualStats {
  T* c;
  int ldc;
  float2* stats;
  int stats_ld;
  struct Pre {
    uint4 r[8];
  };
  struct Tile {
    float n, mean, m2;
  };
  __device__ __forceinline__ void stage(float*, int, int) const {}
  __device__ __forceinline__ void tile_load(Tile& t, int, int) const {
    t.n = 0.f;
    t.mean = 0.f;
    t.m2 = 0.f;
  }
  __device__ __forceinline__ void load(Pre& p, int row, int col) const {
    const uint4* src = reinterpret_cast<const uint4*>(c + static_cast<size_t>(row) * ldc + col);
#pragma unroll
    for (int i = 0; i < 8; ++i) p.r[i] = src[i];
  }
  __device__ __forceinline__ void apply(const Pre& p, Tile& t, int row, int col, const float (&v0)[32],
                                        const float (&v1)[32]) const {
    uint4* dst = reinterpret_cast<uint4*>(c + static_cast<size_t>(row) * ldc + col);
    float r[8], o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      unpack8<T>(p.r[i], r);
      const float* v = (i < 4) ? &v0[8 * i] : &v1[8 * (i - 4)];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[j] + r[j];
      const uint4 packed = pack8<T>(o);
      dst[i] = packed;
      unpack8<T>(packed, o);  // statistics of the values as stored
      float m = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) m += o[j];
      m *= 0.125f;
      float q = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) q += (o[j] - m) * (o[j] - m);
      const float tot = t.n + 8.f;
      const float d = m - t.mean;
      t.mean += d * (8.f / tot);
      t.m2 += q + d * d * (t.n * 8.f / tot);
      t.n = tot;
    }
    if ((col & 255) == 192) stats[static_cast<size_t>(row) * stats_ld + (col >> 8)] = make_float2(t.mean, t.m2);
  }
};

// Fields shared by the two LayerNorm-folding epilogues.
struct LnFold {
  const float2* stats;  // partials of the input rows, stats_ld per row, stats_n valid
  int stats_ld;
  int stats_n;
  const float* csum;    // c_n = sum_k W'_nk over the bf16 folded weights, [N]
  float eps;
  int n;                // length of csum (<= 2560: it is staged in shared memory)
  // Copies csum into the CTA's shared memory (called once per CTA by the 128 epilogue threads).
  __device__ __forceinline__ void stage_into(float* s, int t, int nt) const {
    for (int i = t; i < n; i += nt) s[i] = csum[i];
  }
};

// QKV projection of a LayerNorm'd row, then rotary embedding on Q and K (see EpiQkvRope).
template <typename T>
struct EpiNormQkvRope {
  EpiQkvRope<T> rope;
  LnFold ln;
  using Pre = NoPre;
  struct Tile {
    typename EpiQkvRope<T>::Tile r;
    float mu, rstd;
  };
  float* cs_smem = nullptr;  // set by stage()
  __device__ __forceinline__ void stage(float* s, int t, int nt) {
    ln.stage_into(s, t, nt);
    cs_smem = s;
  }
  __device__ __forceinline__ void tile_load(Tile& t, int row, int n0) const {
    rope.tile_load(t.r, row, n0);
    row_stats(ln.stats + static_cast<size_t>(row) * ln.stats_ld, ln.stats_n, ln.eps, t.mu, t.rstd);
  }
  __device__ __forceinline__ void load(Pre&, int, int) const {}
  __device__ __forceinline__ void apply(const Pre& p, Tile& t, int row, int col, const float (&v0)[32],
                                        const float (&v1)[32]) const {
    float a[32], b[32];
    const float4* cs = reinterpret_cast<const float4*>(cs_smem + col);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 c0 = cs[i], c1 = cs[8 + i];
      const float ca[4] = {c0.x, c0.y, c0.z, c0.w}, cb[4] = {c1.x, c1.y, c1.z, c1.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        a[4 * i + j] = t.rstd * (v0[4 * i + j] - t.mu * ca[j]);
        b[4 * i + j] = t.rstd * (v1[4 * i + j] - t.mu * cb[j]);
      }
    }
    rope.apply(p, t.r, row, col, a, b);
  }
};

// Wi projection of a LayerNorm'd row, then GeGLU on the interleaved value / gate columns.
template <typename T>
struct EpiNormGeglu {
  EpiGeglu<T> geglu;
  LnFold ln;
  using Pre = NoPre;
  struct Tile {
    float mu, rstd;
  };
  float* cs_smem = nullptr;  // set by stage()
  __device__ __forceinline__ void stage(float* s, int t, int nt) {
    ln.stage_into(s, t, nt);
    cs_smem = s;
  }
  __device__ __forceinline__ void tile_load(Tile& t, int row, int) const {
    row_stats(ln.stats + static_cast<size_t>(row) * ln.stats_ld, ln.stats_n, ln.eps, t.mu, t.rstd);
  }
  __device__ __forceinline__ void load(Pre&, int, int) const {}
  __device__ __forceinline__ void apply(const Pre& p, Tile& t, int row, int col, const float (&v0)[32],
                                        const float (&v1)[32]) const {
    float a[32], b[32];
    const float4* cs = reinterpret_cast<const float4*>(cs_smem + col);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 c0 = cs[i], c1 = cs[8 + i];
      const float ca[4] = {c0.x, c0.y, c0.z, c0.w}, cb[4] = {c1.x, c1.y, c1.z, c1.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        a[4 * i + j] = t.rstd * (v0[4 * i + j] - t.mu * ca[j]);
        b[4 * i + j] = t.rstd * (v1[4 * i + j] - t.mu * cb[j]);
      }
    }
    NoTile nt;
    geglu.apply(NoPre{}, nt, row, col, a, b);
  }
};

}  // namespace rv
