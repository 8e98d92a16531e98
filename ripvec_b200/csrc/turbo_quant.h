// Launchers of the PolarQuant ("TurboQuant") compressed scan (turbo_quant.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <algorithm>

namespace rv {

// Largest query-table bytes a scan CTA stages (tables of up to 4 queries per pass).
constexpr size_t kPolarMaxLutBytes = 200 * 1024;

// Codes of rows x [n, dim] bf16 (dim a multiple of 64) under rt (rt[d * dim + j] = R[j][d]):
// radii [ceil(n / 32) * 32 * dim / 2] f32 and bins (same count, u8) in the interleaved layout.
cudaError_t polar_encode(const __nv_bfloat16* x, int64_t n, int dim, const float* rt, int levels, float* radii,
                         uint8_t* bins, cudaStream_t st);
// Query tables lut [nq, dim / 2, levels] of f32 queries q [nq, dim]; cos_sin = [cos[levels], sin[levels]].
cudaError_t polar_query_tables(const float* q, int nq, int dim, const float* rt, const float* cos_sin, int levels,
                               float* lut, cudaStream_t st);
// Approximate scores of rows [row_begin, row_begin + rows) (row_begin a multiple of 32) into
// s[q * ld + (row - row_begin)] for every query.
cudaError_t polar_scan(const float* radii, const uint8_t* bins, int pairs, int64_t row_begin, int64_t rows,
                       const float* lut, int nq, int levels, float* s, int64_t ld, cudaStream_t st);
// Rows past this many equal keys at the selection boundary make polar_select set *overflow.
int polar_tie_cap();
// The best `pre` rows of each query's scores s[q * ld + i], i < n, by (score desc, row asc),
// as rows row_base + i into list_i [nq, pre]; list_n[q] = min(pre, n).  Scratch: state [4 nq],
// hist [256 nq] (zero on entry after the first call: every call leaves it cleared), counters
// [2 nq], ties [nq, polar_tie_cap()].
cudaError_t polar_select(const float* s, int64_t ld, int64_t n, int64_t row_base, int nq, int pre,
                         uint32_t* state, uint32_t* hist, uint32_t* counters, int64_t* ties, int64_t* list_i,
                         int* list_n, int* overflow, cudaStream_t st);

}  // namespace rv
