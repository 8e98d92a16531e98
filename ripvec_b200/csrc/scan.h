// Launchers of the exact top-k scan kernels (scan.cu).
#pragma once

#include <cuda.h>
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

// Fused filter (scan_fused.cu).  Candidate buffer size per query, largest list width, most
// queries per batch, records per GEMM CTA.
int scan_filter_cap();
int scan_filter_max_kp();
int scan_filter_max_queries();
int scan_filter_record_cap();
// Query columns per filter GEMM tile for a batch of nq queries (128 or 256).
int scan_filter_bn(int nq);
// Scores database rows [row0, row0 + rows) (tm_rows: their [rows, dim] bf16 view, box 64 x 128)
// against the queries (tm_queries: [nq, dim] bf16, box 64 x scan_filter_bn(nq), read as nq_pad
// rows, nq_pad a multiple of scan_filter_bn(nq) and <= scan_filter_max_queries()), keeps scores above each query's current
// kp-th list score, and merges them into the lists.  thr: [nq_pad]; rec: [sms, record cap];
// rec_n: [sms]; cand_*: [nq, scan_filter_cap()].  *overflow is set when a CTA or a query kept
// more candidates than its buffer holds (the lists are then incomplete).
cudaError_t scan_filter_block(const CUtensorMap& tm_rows, const CUtensorMap& tm_queries, int rows,
                              int dim, int64_t row0, int nq, int nq_pad, int kp, float* thr,
                              int4* rec, int* rec_n, int* cand_n, float* cand_s, int64_t* cand_i,
                              float* list_s, int64_t* list_i, int* list_n, int* overflow,
                              unsigned int* err, cudaStream_t st);

}  // namespace rv
