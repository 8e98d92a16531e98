// Host-callable launchers of the sm_100a kernels (definitions in the .cu files).  All device
// pointers; every launcher returns the launch status and never synchronizes.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rv {

// Error bits written to a device error word by kernels that give up.
enum DeviceError : unsigned int {
  kErrWaitTimeout = 1u << 0,   // an mbarrier wait ran past its cycle limit
  kErrBadShape = 1u << 1,      // a kernel saw an input it does not support (token id range)
  kErrScanOverflow = 1u << 2,  // a candidate buffer of the top-k scan filled up
};

enum class Act { kBf16 = 0, kF16 = 1 };

// Which epilogue a projection GEMM runs.
enum class GemmEpi {
  kStore = 0,      // C = A B^T
  kResidual = 1,   // C += A B^T (+ bias)
  kGeglu = 2,      // out = gelu(value) * gate over an interleaved Wi
  kQkvRope = 3,    // C = A B^T, rotary embedding on the first rope_cols columns
  kBias = 4,       // C = A B^T + bias
  kBiasGelu = 5,   // C = gelu(A B^T + bias)
  kStoreF32 = 6,   // C(f32) = A B^T
  kResidualStats = 7,  // C += A B^T and per-256-column (mean, M2) LayerNorm partials of C
  kNormQkvRope = 8,    // LayerNorm folded (A = raw rows + partials), then QKV + rotary
  kNormGeglu = 9,      // LayerNorm folded, then GeGLU
};

struct GemmArgs {
  const CUtensorMap* tmA;  // A [M,K] K-major, box 64 x 128
  const CUtensorMap* tmB;  // B [N,K] K-major, box 64 x BN
  const CUtensorMap* tmC;  // optional: output C for the TMA-staged epilogue (box 64 x 32, 128-B
                           // swizzle; 32 x 32 with 64-B swizzle for GeGLU: one box per warp)
  int M, N, K;
  int bn;                  // 128 or 256 (N % bn == 0)
  int b_row_offset;        // added to the B-operand row coordinate (chunked scans)
  bool pair;               // two-CTA 256 x 256 tiles (tmB must then have a 64 x 128 box)
  GemmEpi epi;
  void* c;                 // output (or in/out for kResidual)
  int ldc;                 // elements
  const float* bias;       // kResidual / kBias / kBiasGelu (may be null)
  int rope_cols;           // kQkvRope
  const int* pos;          // kQkvRope: [M] position inside the sequence
  const float* cos_t;      // kQkvRope: [max_pos, 32]
  const float* sin_t;
  void* stats;             // float2 partials: written by kResidualStats, read by kNorm*
  int stats_ld;            // partials per row in the buffer
  int stats_n;             // kNorm*: partials that make up one row (hidden / 256)
  const float* csum;       // kNorm*: column sums of the folded weights, [N]
  float eps;               // kNorm*: LayerNorm epsilon
};

cudaError_t gemm_tc(Act act, const GemmArgs& a, unsigned int* err, cudaStream_t st);

// pos[t] = t - cu_seqlens[seq(t)] for t < total (binary search over cu_seqlens[0..n]).
cudaError_t build_positions(const int* cu_seqlens, int n_seqs, int total, int* pos,
                            cudaStream_t st);

// ModernBERT embedding + LayerNorm: out[t] = LN(table_f32[ids[t]]) * gamma.
cudaError_t embed_ln(Act act, const int* ids, int total, const float* table, int vocab,
                     const float* gamma, const float* beta, const float* pos_table,
                     const int* pos, const float* type_row, int hidden, float eps, void* out,
                     unsigned int* err, cudaStream_t st);

// out[t] = LN(in[t]) * gamma (+ beta), f32 statistics, 16-bit in/out.
cudaError_t layernorm(Act act, const void* in, void* out, int rows, int hidden,
                      const float* gamma, const float* beta, float eps, cudaStream_t st);

// Pooling: mode 0 = final LN then mean over the sequence, 1 = mean (no LN), 2 = first token.
// Then L2 normalisation: x / max(norm, l2_floor) when l2_floor > 0, else x / norm if norm > 0.
cudaError_t pool_l2(Act act, const void* hidden_states, const int* cu_seqlens, int n_seqs,
                    int hidden, int mode, const float* gamma, float eps, float l2_floor,
                    float* out, cudaStream_t st);

// Varlen bidirectional attention over packed qkv [T, 3*H] (Q | K | V, head h at h*D).
// window_half < 0: global; else key j is visible from query i iff |i - j| <= window_half.
// q_tile_starts[b] = first 64-query tile of sequence b (prefix sum of ceil(L_b/64)), n+1 entries.
cudaError_t attention_varlen(Act act, const void* qkv, void* ctx, const int* cu_seqlens,
                             const int* q_tile_starts, int n_seqs, int total_q_tiles,
                             int num_heads, int head_dim, int window_half, float scale,
                             cudaStream_t st);

// The same on the 5th-generation tensor cores, head_dim 64 only.  tiles[t] = {sequence start,
// length | first query << 16} of 128-query tile t (fill_attention_tiles); total_tokens bounds the
// TMA view of qkv (total_tokens * heads * 64 < 2^31).  A pipeline wait that expires sets
// kErrWaitTimeout in *err.
cudaError_t attention_varlen_tc(Act act, const void* qkv, void* ctx, int total_tokens,
                                const int2* tiles, int n_tiles, int num_heads, int window_half,
                                float scale, unsigned int* err, cudaStream_t st);
// Longest sequence the tile records encode.
constexpr int kMaxAttnSeq = 32767;
// Host: writes the 128-query tile records of a packed batch (sum of ceil(L_b / 128) entries,
// at most total_tokens / 128 + n_seqs) and returns their count, or -1 when a length is negative
// or above kMaxAttnSeq.
int fill_attention_tiles(const int* cu_seqlens, int n_seqs, int2* out);
// Test hook of the device error path: while enabled, every tcgen05 attention launch withholds
// the score signal of each CTA's first tile and bounds its waits by wait_limit_cycles, so the
// launch ends through its bounded-wait exit and reports kErrWaitTimeout.
void attention_set_stall(int enable, long long wait_limit_cycles);
// Test hook: y = exp2_poly(x) on n floats (device pointers), the FMA-pipe exponential that the
// tcgen05 attention's softmax uses beside the MUFU ex2 when RV_ATTN_EXP2_POLY=1.
cudaError_t exp2_poly_eval(const float* x, float* y, int64_t n, cudaStream_t st);

// f32 -> 16-bit conversion (weights upload), n elements.
cudaError_t convert_f32(Act act, const float* in, void* out, int64_t n, cudaStream_t st);

}  // namespace rv
