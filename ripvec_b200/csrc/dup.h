// Launchers of the all-pairs near-duplicate search (dup.cu).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "tmap.h"

namespace rv {

// Scores strip rows [r0, r0 + rows) (tm_strip: their [rows, dim] bf16 view, box 64 x 128)
// against rows [r0, r0 + cols) of the index (tm_rows: the whole [n, dim] matrix, box 64 x 256;
// cols a multiple of 256, rows past n read as zeros) and appends every pair (i, j) with j > i,
// j < n and f32 score >= thr_lo as an {i, j, score bits, 0} record at rec[*counter++] (records
// past cap are counted, not written).
cudaError_t dup_candidates(const CUtensorMap& tm_strip, const CUtensorMap& tm_rows, int rows, int cols, int dim,
                           int r0, int n, float thr_lo, int4* rec, unsigned long long* counter, long long cap,
                           unsigned int* err, cudaStream_t st);
// s64[t] = exact score of record t's pair (sequential f64 sum of the bf16 products).
cudaError_t dup_rescore(const __nv_bfloat16* db, int dim, const int4* rec, long long m, double* s64,
                        cudaStream_t st);

}  // namespace rv
