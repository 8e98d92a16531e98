// Launchers of the MRL cascade transform (cascade.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace rv {

// Largest shared memory of the row transform (32 staged input rows + 32 output rows).
constexpr size_t kCascadeMaxSmem = 200 * 1024;
size_t cascade_rows_smem(int dim, int t);
// out [n, t] bf16 = the truncated, re-normalised LayerNorm of rows x [n, dim] bf16.
cudaError_t cascade_rows(const __nv_bfloat16* x, int64_t n, int dim, int t, __nv_bfloat16* out, cudaStream_t st);
// out [nq, t] f32, the same transform of f32 queries q [nq, dim].
cudaError_t cascade_queries(const float* q, int nq, int dim, int t, float* out, cudaStream_t st);

}  // namespace rv
