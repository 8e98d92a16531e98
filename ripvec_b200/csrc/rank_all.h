// Launchers of the full ranking (rank_all.cu): every row whose exact score reaches a threshold.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace rv {

// Rows [0, n) of db [n, dim] whose f32 score against the bf16 query qb [dim] is >= lo are
// appended (as local row numbers, in no fixed order) to cand; *count (zeroed by the caller)
// receives how many.  cand must hold n entries.
cudaError_t rank_filter(const __nv_bfloat16* db, int64_t n, int dim, const __nv_bfloat16* qb, float lo,
                        int* cand, unsigned long long* count, cudaStream_t st);
// Exact scores (sequential f64 sums of the bf16 products) of the m candidates (cand == nullptr:
// rows 0..m-1); those >= threshold are appended as (score, base + row) to out_s / out_i, *count
// (zeroed by the caller) receiving how many.
cudaError_t rank_exact(const __nv_bfloat16* db, int dim, const __nv_bfloat16* qb, const int* cand, int64_t m,
                       int64_t base, double threshold, double* out_s, int64_t* out_i,
                       unsigned long long* count, cudaStream_t st);
// Radix sort of m (score, row) pairs by score, descending.  With temp == nullptr only sets
// *temp_bytes to the scratch size the sort needs.
cudaError_t rank_sort_desc(void* temp, size_t* temp_bytes, const double* keys_in, double* keys_out,
                           const int64_t* vals_in, int64_t* vals_out, int64_t m, cudaStream_t st);

}  // namespace rv
