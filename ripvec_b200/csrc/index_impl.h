// The search index object shared by the C ABI translation units of the scan.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <mutex>
#include <string>

template <typename T>
struct DevBuf {
  T* p = nullptr;
  size_t cap = 0;
  // Ensures room for `need` elements (contents are not preserved).  False on allocation failure.
  bool reserve(size_t need) {
    if (p && cap >= need) return true;
    if (p) cudaFree(p);
    p = nullptr;
    cap = 0;
    if (cudaMalloc(reinterpret_cast<void**>(&p), (need ? need : 1) * sizeof(T)) != cudaSuccess) return false;
    cap = need;
    return true;
  }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    cap = 0;
  }
};

struct rv_index {
  int device = 0;
  std::mutex mu;
  std::string err;
  cudaStream_t stream = nullptr;
  __nv_bfloat16* db = nullptr;
  int64_t n = 0;
  int dim = 0;
  int64_t base = 0;
  double max_norm = 0.0;
  CUtensorMap tmap_db;
  unsigned int* d_err = nullptr;
  // scratch, grown on demand
  DevBuf<float> scores, qf, list_s, os;
  DevBuf<__nv_bfloat16> qb;
  DevBuf<int64_t> list_i, oi;
  DevBuf<int> list_n, cnt, guard;
  DevBuf<double> os64;
  // fused filter (scan_fused.cu): thresholds, candidate buffers, overflow flag
  DevBuf<float> thr, cand_s;
  DevBuf<int64_t> cand_i;
  DevBuf<int> cand_n, overflow, rec_n;
  DevBuf<int4> rec;
  // PolarQuant ("TurboQuant") corpus (turbo_quant.cu), built by rv_index_build_polar:
  // interleaved radii / angle bins, the transposed rotation, the cos / sin tables, and the
  // per-call query tables, approximate scores and selection scratch.
  int pq_levels = 0;  // 0: no compressed corpus
  DevBuf<float> pq_radii, pq_rt, pq_cs, pq_lut, pq_s;
  DevBuf<uint8_t> pq_bins;
  DevBuf<uint32_t> pq_state, pq_hist, pq_counters;
  DevBuf<int64_t> pq_ties;
  // MRL cascade (cascade.cu): an index over the truncated, re-normalised rows, built by
  // rv_index_build_cascade, and the per-call truncated queries and first-phase candidates.
  rv_index* cascade = nullptr;
  DevBuf<float> c_q, c_os;
  DevBuf<int64_t> c_oi;
  // find_duplicates (dup.cu): candidate pair records, their counter and exact scores.
  DevBuf<int4> dup_rec;
  DevBuf<unsigned long long> dup_cnt;
  DevBuf<double> dup_s64;
  // Full ranking (rank_all.cu): candidate rows, the two counters, (score, row) pairs and their
  // sorted copies, and the radix sort's scratch.
  DevBuf<int> rank_cand;
  DevBuf<unsigned long long> rank_cnt;
  DevBuf<double> rank_s, rank_s2;
  DevBuf<int64_t> rank_i, rank_i2;
  DevBuf<uint8_t> rank_tmp;
  int64_t launches = 0;
  bool filter_off = false;  // RV_SCAN_FILTER=0 at creation
  // Orders work queued on another index's stream (the cascade's truncated index) after this
  // index's stream without a host synchronisation; created on first use.
  cudaEvent_t order_ev = nullptr;
};

