// Launchers of the exact top-k scan kernels (scan.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rv {

int scan_cap_for(int kp);
cudaError_t scan_round_queries(const float* q, __nv_bfloat16* out, int64_t n, cudaStream_t st);
cudaError_t scan_row_norm_max(const __nv_bfloat16* db, int64_t n, int dim, unsigned int* max_bits,
                              cudaStream_t st);
cudaError_t scan_init_lists(int* list_n, int nq, cudaStream_t st);
cudaError_t scan_select(const float* scores, int ld, int cols, int64_t row0, int nq, int kp,
                        float* list_s, int64_t* list_i, int* list_n, cudaStream_t st);
cudaError_t scan_rescore(const __nv_bfloat16* db, int64_t base, int dim, const __nv_bfloat16* qb,
                         int nq, const float* list_s, const int64_t* list_i, const int* list_n,
                         int kp, int k, int64_t n_rows, double eps_scale, float threshold,
                         int64_t* out_i, float* out_s, double* out_s64, int* out_cnt,
                         int* guard_fail, cudaStream_t st);
cudaError_t scan_merge(const int64_t* idx_in, const double* s_in, int n_lists, int nq, int k,
                       float threshold, int64_t* idx_out, float* s_out, double* s64_out,
                       cudaStream_t st);

}  // namespace rv
