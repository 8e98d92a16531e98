// C ABI of the search side: a bf16 device copy of the embedding matrix (SearchIndex::new,
// crates/ripvec-core/src/index.rs:76-165) and the exact cosine top-k (SearchIndex::rank,
// index.rs:172-186, restricted to the best k with the (score desc, row asc) order).
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/ripvec_b200.h"
#include "engine.h"
#include "cascade.h"
#include "comm_impl.h"
#include "dup.h"
#include "index_impl.h"
#include "kernels.h"
#include "rank_all.h"
#include "scan.h"
#include "tmap.h"
#include "turbo_quant.h"

namespace {

int ifail(rv_index* x, int code, const std::string& m) {
  if (x) x->err = m;
  return code;
}

#define IX_TRY(x, expr)                                                                  \
  do {                                                                                   \
    cudaError_t _e = (expr);                                                             \
    if (_e != cudaSuccess)                                                               \
      return ifail(x, RV_E_CUDA, std::string(#expr) + ": " + cudaGetErrorString(_e));    \
  } while (0)

struct Dev {
  int prev = -1;
  explicit Dev(int d) {
    cudaGetDevice(&prev);
    if (prev != d) cudaSetDevice(d);
  }
  ~Dev() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// Runs one query batch end to end on x->stream for candidate width kp.
// Rows scored by the chunked path before the fused filter takes over (its lists give the
// first thresholds): one small chunk, so that the fixed cost per query batch stays low.
constexpr int64_t kFilterPrefixRows = 1024;

// Runs one query batch end to end on x->stream for candidate width kp.  With `fused`, rows past
// the first kFilterPrefixRows go through the filtering GEMM (scan_fused.cu) in blocks that grow
// with the rows already seen; *x->overflow is set if a block kept more candidates than the
// buffers hold, and the caller then redoes the batch without it.
// qb holds nq_rows >= nq rows (a whole number of query tiles, zero past nq), so no TMA box of
// the query operand reaches past the buffer: boxes that were mostly out of bounds (zero-filled
// by the copy engine) made 1-64-query scans about 1.5x slower than 128-query ones.
int topk_pass(rv_index* x, const __nv_bfloat16* qb, int nq, int nq_rows, int k, int kp, float threshold,
              int64_t* out_i, float* out_s, double* out_s64, bool fused) {
  cudaStream_t st = x->stream;
  if (!x->list_s.reserve(size_t(nq) * kp) || !x->list_i.reserve(size_t(nq) * kp) ||
      !x->list_n.reserve(size_t(nq)))
    return ifail(x, RV_E_NOMEM, "scan list allocation failed");
  IX_TRY(x, rv::scan_init_lists(x->list_n.p, nq, st));
  x->launches++;
  const int cap = rv::scan_cap_for(kp);
  if (x->n > 0) {
    CUtensorMap tq;
    std::string why;
    if (!rv::make_tmap_2d_16bit(&tq, qb, true, x->dim, nq_rows, uint64_t(x->dim) * 2, 64, 128, &why))
      return ifail(x, RV_E_CUDA, why);
    // Chunk schedule: the first chunk fits the select buffer with an empty list; later chunks
    // grow with the rows already seen so the expected number of survivors stays well below
    // the buffer; S = [nq, chunk] f32 is kept near 32 MB so it stays in L2.
    int64_t cmax = (int64_t(32) << 20) / (int64_t(nq) * 4);
    cmax = std::max<int64_t>(256, std::min<int64_t>(cmax, int64_t(1) << 22)) / 256 * 256;
    if (!x->scores.reserve(size_t(nq) * size_t(cmax)))
      return ifail(x, RV_E_NOMEM, "scan score buffer allocation failed");
    int64_t r0 = 0;
    int64_t chunk = std::max<int64_t>(256, (cap - kp) / 256 * 256);
    const int64_t chunked_end = fused ? std::min<int64_t>(x->n, kFilterPrefixRows) : x->n;
    while (r0 < chunked_end) {
      const int64_t valid = std::min<int64_t>(chunk, chunked_end - r0);
      const int64_t ncols = (valid + 255) / 256 * 256;
      rv::GemmArgs g{};
      g.tmA = &tq;
      g.tmB = &x->tmap_db;
      g.M = nq;
      g.N = static_cast<int>(ncols);
      g.K = x->dim;
      g.bn = 256;
      g.b_row_offset = static_cast<int>(r0);
      g.epi = rv::GemmEpi::kStoreF32;
      g.c = x->scores.p;
      g.ldc = static_cast<int>(ncols);
      IX_TRY(x, rv::gemm_tc(rv::Act::kBf16, g, x->d_err, st));
      IX_TRY(x, rv::scan_select(x->scores.p, static_cast<int>(ncols), static_cast<int>(valid),
                                x->base + r0, nq, kp, x->list_s.p, x->list_i.p, x->list_n.p, st));
      x->launches += 2;
      r0 += valid;
      const int64_t grow_to = (int64_t(cap - kp) * r0) / (4 * int64_t(kp));
      chunk = std::max<int64_t>(256, std::min<int64_t>(cmax, grow_to) / 256 * 256);
    }
    if (r0 < x->n) {
      // Fused filter over the rest.  A block of b rows after s rows seen keeps about kp * b / s
      // candidates per query on rows in random order; blocks of s rows keep about kp each, and
      // the total over the log2(n / s0) blocks, 1.45 kp ln(n / s0), is about half of what fewer,
      // larger blocks keep.  Starting from a 1024-row prefix costs a few small blocks instead of
      // a long chunked prefix, which matters when a rank's shard is small (strong scaling).
      const int fcap = rv::scan_filter_cap();
      const int bn = rv::scan_filter_bn(nq);
      const int nq_pad = (nq + bn - 1) / bn * bn;
      const int sms = rv::device_sm_count();
      if (!x->thr.reserve(size_t(nq_pad)) || !x->cand_n.reserve(size_t(nq)) ||
          !x->cand_s.reserve(size_t(nq) * fcap) || !x->cand_i.reserve(size_t(nq) * fcap) ||
          !x->rec_n.reserve(size_t(sms)) ||
          !x->rec.reserve(size_t(sms) * size_t(rv::scan_filter_record_cap())))
        return ifail(x, RV_E_NOMEM, "scan filter buffer allocation failed");
      CUtensorMap tqb;  // B operand: bn query rows per tile
      if (!rv::make_tmap_2d_16bit(&tqb, qb, true, x->dim, nq_rows, uint64_t(x->dim) * 2, 64, bn, &why))
        return ifail(x, RV_E_CUDA, why);
      // Small batches with lists of at most 256 grow the blocks 5x instead of 2x: their merges are
      // cheap, and fewer blocks mean fewer launches and partial last waves per pass over the
      // database (a block of 4s rows after s seen keeps about 4 kp <= 1024 candidates per query,
      // inside the 2048-entry buffer).
      const int64_t grow = (nq <= 128 && kp <= 256) ? 4 : 1;
      while (r0 < x->n) {
        const int64_t rows = std::min<int64_t>({x->n - r0, grow * r0, int64_t(1) << 24});
        CUtensorMap trows;
        if (!rv::make_tmap_2d_16bit(&trows, x->db + size_t(r0) * x->dim, true, x->dim, uint64_t(rows),
                                    uint64_t(x->dim) * 2, 64, 128, &why))
          return ifail(x, RV_E_CUDA, why);
        IX_TRY(x, rv::scan_filter_block(trows, tqb, static_cast<int>(rows), x->dim, x->base + r0, nq,
                                        nq_pad, kp, x->thr.p, x->rec.p, x->rec_n.p, x->cand_n.p,
                                        x->cand_s.p, x->cand_i.p,
                                        x->list_s.p, x->list_i.p, x->list_n.p, x->overflow.p, x->d_err,
                                        st));
        x->launches += 3;
        r0 += rows;
      }
    }
  }
  if (!x->cnt.reserve(size_t(nq)) || !x->guard.reserve(size_t(nq)))
    return ifail(x, RV_E_NOMEM, "scan output allocation failed");
  const double eps_scale = double(x->dim) * std::ldexp(1.0, -22) * x->max_norm;
  IX_TRY(x, rv::scan_rescore(x->db, x->base, x->dim, qb, nq, x->list_s.p, x->list_i.p, x->list_n.p,
                             kp, k, x->n, eps_scale, threshold, out_i, out_s, out_s64, x->cnt.p,
                             x->guard.p, st));
  x->launches++;
  return RV_OK;
}

int topk_device(rv_index* x, const float* q_dev, int nq, int k, float threshold, int64_t* out_i,
                float* out_s, double* out_s64, std::vector<int>* counts) {
  if (nq <= 0) return RV_OK;
  if (k <= 0 || k > 2048) return ifail(x, RV_E_INVALID, "k must be in [1, 2048]");
  cudaStream_t st = x->stream;
  // Query rows padded with zeros to whole tiles of the filter GEMM (128 rows up to 128 queries,
  // else 256).
  const int nq_rows = nq <= 128 ? 128 : (nq + 255) / 256 * 256;
  if (!x->qb.reserve(size_t(nq_rows) * x->dim)) return ifail(x, RV_E_NOMEM, "query buffer");
  IX_TRY(x, rv::scan_round_queries(q_dev, x->qb.p, int64_t(nq) * x->dim, st));
  if (nq_rows > nq)
    IX_TRY(x, cudaMemsetAsync(x->qb.p + size_t(nq) * x->dim, 0, size_t(nq_rows - nq) * x->dim * 2, st));
  x->launches++;
  int kp = std::max(128, 2 * k);
  // The fused filter needs the thresholds of all queries in shared memory.
  bool fused = nq <= rv::scan_filter_max_queries() && !x->filter_off;
  if (!x->overflow.reserve(1)) return ifail(x, RV_E_NOMEM, "scan flag allocation failed");
  for (;;) {
    const bool use_fused = fused && kp <= rv::scan_filter_max_kp();
    IX_TRY(x, cudaMemsetAsync(x->overflow.p, 0, sizeof(int), st));
    int rc = topk_pass(x, x->qb.p, nq, nq_rows, k, kp, threshold, out_i, out_s, out_s64, use_fused);
    if (rc) return rc;
    std::vector<int> g(nq);
    unsigned int e = 0;
    int ovf = 0;
    IX_TRY(x, cudaMemcpyAsync(g.data(), x->guard.p, sizeof(int) * nq, cudaMemcpyDeviceToHost, st));
    IX_TRY(x, cudaMemcpyAsync(&e, x->d_err, 4, cudaMemcpyDeviceToHost, st));
    IX_TRY(x, cudaMemcpyAsync(&ovf, x->overflow.p, sizeof(int), cudaMemcpyDeviceToHost, st));
    if (counts) {
      counts->resize(nq);
      IX_TRY(x, cudaMemcpyAsync(counts->data(), x->cnt.p, sizeof(int) * nq, cudaMemcpyDeviceToHost, st));
    }
    IX_TRY(x, cudaStreamSynchronize(st));
    if (e) {
      cudaMemset(x->d_err, 0, 4);
      return ifail(x, RV_E_DEVICE, "scan kernel reported device error flags " + std::to_string(e));
    }
    if (ovf) {
      // A query kept more filter candidates than its buffer: same kp, chunked path only.
      fused = false;
      continue;
    }
    bool any = false;
    for (int v : g) any |= (v != 0);
    if (!any) return RV_OK;
    if (kp >= 4096)
      return ifail(x, RV_E_DEVICE,
                   "exact top-k needs more than 4096 candidates (too many near-equal scores)");
    kp = std::min(4096, kp * 4);
  }
}

// SearchIndex::rank_turboquant (index.rs:196-234) over device queries: approximate PolarQuant
// scores of every row, the best pre = min(10 top_k, n) by (approximate score desc, row asc),
// exact rescoring of those (the exact path's definition: f64 sums of the bf16 products), rows
// below the threshold dropped, the best top_k by (score desc, row asc).  Without a compressed
// corpus it is the exact top-k (the reference falls back to rank, index.rs:202-204).
constexpr int kTqMaxTopK = 800;  // pre <= 8000 candidates per query

int tq_device(rv_index* x, const float* q_dev, int nq, int top_k, float threshold, int64_t* out_i, float* out_s,
              double* out_s64, std::vector<int>* counts) {
  if (nq <= 0) return RV_OK;
  if (top_k <= 0 || top_k > kTqMaxTopK)
    return ifail(x, RV_E_INVALID, "top_k must be in [1, " + std::to_string(kTqMaxTopK) + "]");
  if (x->pq_levels == 0 || x->n == 0)
    return topk_device(x, q_dev, nq, top_k, threshold, out_i, out_s, out_s64, counts);
  cudaStream_t st = x->stream;
  const int dim = x->dim, pairs = dim / 2, levels = x->pq_levels;
  const int pre = static_cast<int>(std::min<int64_t>(int64_t(10) * top_k, x->n));
  // Queries per batch: the approximate scores [batch, n] f32 stay under 1 GiB.
  const int64_t per_q = x->n * 4;
  const int qg = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(64, (int64_t(1) << 30) / per_q)));
  const int bq_max = std::min(qg, nq);
  if (!x->qb.reserve(size_t(bq_max) * dim) || !x->pq_lut.reserve(size_t(bq_max) * pairs * levels) ||
      !x->pq_s.reserve(size_t(bq_max) * x->n) || !x->pq_state.reserve(size_t(4) * bq_max) ||
      !x->pq_hist.reserve(size_t(256) * bq_max) || !x->pq_counters.reserve(size_t(2) * bq_max) ||
      !x->pq_ties.reserve(size_t(bq_max) * rv::polar_tie_cap()) || !x->list_s.reserve(size_t(bq_max) * pre) ||
      !x->list_i.reserve(size_t(bq_max) * pre) || !x->list_n.reserve(size_t(bq_max)) ||
      !x->cnt.reserve(size_t(nq)) || !x->guard.reserve(size_t(bq_max)) || !x->overflow.reserve(1))
    return ifail(x, RV_E_NOMEM, "turboquant scratch allocation failed");
  IX_TRY(x, cudaMemsetAsync(x->overflow.p, 0, sizeof(int), st));
  for (int b0 = 0; b0 < nq; b0 += bq_max) {
    const int bq = std::min(bq_max, nq - b0);
    const float* qd = q_dev + size_t(b0) * dim;
    IX_TRY(x, rv::scan_round_queries(qd, x->qb.p, int64_t(bq) * dim, st));
    IX_TRY(x, rv::polar_query_tables(qd, bq, dim, x->pq_rt.p, x->pq_cs.p, levels, x->pq_lut.p, st));
    IX_TRY(x, rv::polar_scan(x->pq_radii.p, x->pq_bins.p, pairs, 0, x->n, x->pq_lut.p, bq, levels, x->pq_s.p,
                             x->n, st));
    IX_TRY(x, rv::polar_select(x->pq_s.p, x->n, x->n, x->base, bq, pre, x->pq_state.p, x->pq_hist.p,
                               x->pq_counters.p, x->pq_ties.p, x->list_i.p, x->list_n.p, x->overflow.p, st));
    const size_t o = size_t(b0) * top_k;
    IX_TRY(x, rv::scan_rescore(x->db, x->base, dim, x->qb.p, bq, x->list_s.p, x->list_i.p, x->list_n.p, pre,
                               top_k, x->n, 0.0, threshold, out_i + o, out_s + o,
                               out_s64 ? out_s64 + o : nullptr, x->cnt.p + b0, x->guard.p, st));
    x->launches += 13;
  }
  int ovf = 0;
  unsigned int e = 0;
  IX_TRY(x, cudaMemcpyAsync(&ovf, x->overflow.p, sizeof(int), cudaMemcpyDeviceToHost, st));
  IX_TRY(x, cudaMemcpyAsync(&e, x->d_err, 4, cudaMemcpyDeviceToHost, st));
  if (counts) {
    counts->resize(nq);
    IX_TRY(x, cudaMemcpyAsync(counts->data(), x->cnt.p, sizeof(int) * nq, cudaMemcpyDeviceToHost, st));
  }
  IX_TRY(x, cudaStreamSynchronize(st));
  if (e) {
    cudaMemset(x->d_err, 0, 4);
    return ifail(x, RV_E_DEVICE, "turboquant kernel reported device error flags " + std::to_string(e));
  }
  if (ovf)
    return ifail(x, RV_E_DEVICE,
                 "turboquant: more than " + std::to_string(rv::polar_tie_cap()) +
                     " rows share the approximate score at the pre-filter boundary");
  return RV_OK;
}

}  // namespace

extern "C" {

int rv_index_create(int device, const void* src, int64_t n, int32_t dim, int32_t src_dtype,
                    int32_t src_on_device, rv_index** out) {
  if (!out) return RV_E_INVALID;
  *out = nullptr;
  if (n < 0 || dim <= 0 || dim % 64 != 0 || dim > 8192 || (n > 0 && !src)) return RV_E_INVALID;
  if (src_dtype != RV_DTYPE_F32 && src_dtype != RV_DTYPE_BF16) return RV_E_INVALID;
  if (n > (int64_t(1) << 31) - 1) return RV_E_INVALID;
  Dev g(device);
  rv_index* x = new rv_index();
  x->device = device;
  x->n = n;
  x->dim = dim;
  // RV_SCAN_FILTER=0: score every row through the chunked GEMM + select path.
  if (const char* e = std::getenv("RV_SCAN_FILTER")) x->filter_off = std::strcmp(e, "0") == 0;
  auto bail = [&](int code) {
    rv_index_destroy(x);
    return code;
  };
  if (cudaStreamCreateWithFlags(&x->stream, cudaStreamNonBlocking) != cudaSuccess) return bail(RV_E_CUDA);
  if (cudaMalloc(&x->d_err, 4) != cudaSuccess || cudaMemset(x->d_err, 0, 4) != cudaSuccess)
    return bail(RV_E_NOMEM);
  const size_t elems = size_t(n) * dim;
  if (n > 0 && cudaMalloc(&x->db, elems * 2) != cudaSuccess) return bail(RV_E_NOMEM);
  if (n > 0) {
    if (src_on_device) {
      if (src_dtype == RV_DTYPE_BF16) {
        if (cudaMemcpyAsync(x->db, src, elems * 2, cudaMemcpyDeviceToDevice, x->stream) != cudaSuccess)
          return bail(RV_E_CUDA);
      } else if (rv::scan_round_queries(static_cast<const float*>(src), x->db, int64_t(elems),
                                        x->stream) != cudaSuccess) {
        return bail(RV_E_CUDA);
      }
    } else {
      const size_t chunk = size_t(1) << 24;
      std::vector<uint16_t> tmp;
      for (size_t s = 0; s < elems; s += chunk) {
        const size_t e = std::min(elems, s + chunk);
        const void* from;
        if (src_dtype == RV_DTYPE_F32) {
          tmp.resize(e - s);
          const float* f = static_cast<const float*>(src);
          for (size_t i = s; i < e; ++i) tmp[i - s] = rv::f32_to_bf16_bits(f[i]);
          from = tmp.data();
        } else {
          from = static_cast<const uint16_t*>(src) + s;
        }
        if (cudaMemcpy(x->db + s, from, (e - s) * 2, cudaMemcpyHostToDevice) != cudaSuccess)
          return bail(RV_E_CUDA);
      }
    }
    unsigned int* mx = nullptr;
    unsigned int hmx = 0;
    if (cudaMalloc(&mx, 4) != cudaSuccess) return bail(RV_E_NOMEM);
    cudaMemsetAsync(mx, 0, 4, x->stream);
    rv::scan_row_norm_max(x->db, n, dim, mx, x->stream);
    cudaMemcpyAsync(&hmx, mx, 4, cudaMemcpyDeviceToHost, x->stream);
    if (cudaStreamSynchronize(x->stream) != cudaSuccess) {
      cudaFree(mx);
      return bail(RV_E_CUDA);
    }
    cudaFree(mx);
    float m2;
    std::memcpy(&m2, &hmx, 4);
    // Norm from the f32 sum of squares, widened by a relative 1e-3 for its rounding.
    x->max_norm = std::sqrt(double(m2)) * 1.001 + 1e-30;
    std::string why;
    if (!rv::make_tmap_2d_16bit(&x->tmap_db, x->db, true, dim, n, uint64_t(dim) * 2, 64, 256, &why)) {
      x->err = why;
      return bail(RV_E_CUDA);
    }
  }
  *out = x;
  return RV_OK;
}

void rv_index_destroy(rv_index* x) {
  if (!x) return;
  rv_index_destroy(x->cascade);
  x->cascade = nullptr;
  {
    Dev g(x->device);
    if (x->stream) cudaStreamSynchronize(x->stream);
    if (x->db) cudaFree(x->db);
    if (x->d_err) cudaFree(x->d_err);
    x->scores.release();
    x->qf.release();
    x->list_s.release();
    x->os.release();
    x->qb.release();
    x->list_i.release();
    x->oi.release();
    x->list_n.release();
    x->cnt.release();
    x->guard.release();
    x->os64.release();
    x->thr.release();
    x->cand_s.release();
    x->cand_i.release();
    x->cand_n.release();
    x->overflow.release();
    x->rec_n.release();
    x->rec.release();
    x->pq_radii.release();
    x->pq_rt.release();
    x->pq_cs.release();
    x->pq_lut.release();
    x->pq_s.release();
    x->pq_bins.release();
    x->pq_state.release();
    x->pq_hist.release();
    x->pq_counters.release();
    x->pq_ties.release();
    x->c_q.release();
    x->c_os.release();
    x->c_oi.release();
    x->dup_rec.release();
    x->dup_cnt.release();
    x->dup_s64.release();
    x->rank_cand.release();
    x->rank_cnt.release();
    x->rank_s.release();
    x->rank_s2.release();
    x->rank_i.release();
    x->rank_i2.release();
    x->rank_tmp.release();
    if (x->order_ev) cudaEventDestroy(x->order_ev);
    if (x->stream) cudaStreamDestroy(x->stream);
  }
  delete x;
}

const char* rv_index_last_error(const rv_index* x) { return x ? x->err.c_str() : "null index"; }
int64_t rv_index_size(const rv_index* x) { return x ? x->n : 0; }
int64_t rv_index_kernel_launches(rv_index* x) {
  if (!x) return 0;
  std::lock_guard<std::mutex> lk(x->mu);
  return x->launches;
}
int rv_index_set_base(rv_index* x, int64_t base) {
  if (!x || base < 0) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(x->mu);
  x->base = base;
  return RV_OK;
}

int rv_index_topk_device(rv_index* x, const float* q_dev, int32_t nq, int32_t k, float threshold,
                         int64_t* out_i, float* out_s, double* out_s64, void* stream) {
  if (!x) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(x->mu);
  if (nq < 0 || (nq > 0 && (!q_dev || !out_i || !out_s))) return ifail(x, RV_E_INVALID, "null argument");
  Dev g(x->device);
  cudaStream_t user = static_cast<cudaStream_t>(stream);
  cudaEvent_t ev = nullptr;
  if (user) {
    IX_TRY(x, cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    IX_TRY(x, cudaEventRecord(ev, user));
    IX_TRY(x, cudaStreamWaitEvent(x->stream, ev, 0));
  }
  int rc = topk_device(x, q_dev, nq, k, threshold, out_i, out_s, out_s64, nullptr);
  if (ev) {
    if (rc == RV_OK) {
      cudaEventRecord(ev, x->stream);
      cudaStreamWaitEvent(user, ev, 0);
    }
    cudaEventDestroy(ev);
  }
  return rc;
}

int rv_index_topk_sharded(rv_index* x, rv_comm* comm, const float* q_dev, int32_t nq, int32_t k,
                          float threshold, int64_t* out_i, float* out_s, double* out_s64, void* stream) {
  if (!x) return RV_E_INVALID;
  if (!comm) return ifail(x, RV_E_INVALID, "null communicator");
  std::lock_guard<std::mutex> lk(x->mu);
  std::lock_guard<std::mutex> lkc(comm->mu);
  if (nq < 0 || (nq > 0 && (!q_dev || !out_i || !out_s))) return ifail(x, RV_E_INVALID, "null argument");
  if (comm->device != x->device) return ifail(x, RV_E_INVALID, "index and communicator are on different devices");
  if (nq == 0) return RV_OK;
  if (k <= 0 || k > 2048) return ifail(x, RV_E_INVALID, "k must be in [1, 2048]");
  if (int64_t(comm->world) * k > 8192)
    return ifail(x, RV_E_INVALID, "world * k must be at most 8192 (the merge keeps every list in shared memory)");
  Dev g(x->device);
  cudaStream_t user = static_cast<cudaStream_t>(stream);
  cudaEvent_t ev = nullptr;
  if (user) {
    IX_TRY(x, cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    IX_TRY(x, cudaEventRecord(ev, user));
    IX_TRY(x, cudaStreamWaitEvent(x->stream, ev, 0));
  }
  // This shard's best k (global row numbers through the index's base), then every rank's lists
  // on every rank, then the device merge by (score desc, row asc): the exact global top k, since
  // the f64 scores are exact and every shard's list holds all of its rows that can be in it.
  const size_t nk = size_t(nq) * k;
  int rc = RV_OK;
  if (!x->oi.reserve(nk) || !x->os.reserve(nk) || !x->os64.reserve(nk)) rc = ifail(x, RV_E_NOMEM, "shard lists");
  if (!rc) rc = topk_device(x, q_dev, nq, k, threshold, x->oi.p, x->os.p, x->os64.p, nullptr);
  int64_t* gi = nullptr;
  double* gs = nullptr;
  if (!rc) {
    rc = rv_comm_allgather_lists(comm, x->oi.p, x->os64.p, nk, &gi, &gs, x->stream);
    if (rc) x->err = comm->err;
  }
  if (!rc && rv::scan_merge(gi, gs, comm->world, nq, k, threshold, out_i, out_s, out_s64, x->stream) != cudaSuccess)
    rc = ifail(x, RV_E_CUDA, "top-k merge launch failed");
  if (!rc) x->launches += 2;
  if (ev) {
    if (rc == RV_OK) {
      cudaEventRecord(ev, x->stream);
      cudaStreamWaitEvent(user, ev, 0);
    }
    cudaEventDestroy(ev);
  }
  return rc;
}

int rv_index_topk(rv_index* x, const float* queries, int32_t nq, int32_t k, float threshold,
                  int64_t* out_idx, float* out_score, double* out_score64, int32_t* out_count) {
  if (!x) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(x->mu);
  if (nq < 0 || (nq > 0 && (!queries || !out_idx || !out_score)))
    return ifail(x, RV_E_INVALID, "null argument");
  if (nq == 0) return RV_OK;
  if (k <= 0 || k > 2048) return ifail(x, RV_E_INVALID, "k must be in [1, 2048]");
  Dev g(x->device);
  cudaStream_t st = x->stream;
  const size_t nk = size_t(nq) * k;
  if (!x->qf.reserve(size_t(nq) * x->dim) || !x->oi.reserve(nk) || !x->os.reserve(nk) ||
      (out_score64 && !x->os64.reserve(nk)))
    return ifail(x, RV_E_NOMEM, "topk buffers");
  IX_TRY(x, cudaMemcpyAsync(x->qf.p, queries, sizeof(float) * size_t(nq) * x->dim,
                            cudaMemcpyHostToDevice, st));
  std::vector<int> counts;
  int rc = topk_device(x, x->qf.p, nq, k, threshold, x->oi.p, x->os.p,
                       out_score64 ? x->os64.p : nullptr, &counts);
  if (rc) return rc;
  IX_TRY(x, cudaMemcpyAsync(out_idx, x->oi.p, sizeof(int64_t) * nk, cudaMemcpyDeviceToHost, st));
  IX_TRY(x, cudaMemcpyAsync(out_score, x->os.p, sizeof(float) * nk, cudaMemcpyDeviceToHost, st));
  if (out_score64)
    IX_TRY(x, cudaMemcpyAsync(out_score64, x->os64.p, sizeof(double) * nk, cudaMemcpyDeviceToHost, st));
  IX_TRY(x, cudaStreamSynchronize(st));
  if (out_count)
    for (int q = 0; q < nq; ++q) out_count[q] = counts[q];
  return RV_OK;
}

int rv_index_rank(rv_index* x, const float* query, float threshold, int64_t capacity, int64_t* out_idx,
                  float* out_score, double* out_score64, int64_t* out_count) {
  if (!x) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(x->mu);
  if (!query || !out_count || capacity < 0 || (capacity > 0 && (!out_idx || !out_score)))
    return ifail(x, RV_E_INVALID, "null argument");
  *out_count = 0;
  if (x->n == 0) return RV_OK;
  Dev g(x->device);
  cudaStream_t st = x->stream;
  const int64_t n = x->n;
  if (!x->qf.reserve(size_t(x->dim)) || !x->qb.reserve(size_t(x->dim)) || !x->rank_cnt.reserve(2) ||
      !x->rank_s.reserve(size_t(n)) || !x->rank_i.reserve(size_t(n)) || !x->rank_s2.reserve(size_t(n)) ||
      !x->rank_i2.reserve(size_t(n)))
    return ifail(x, RV_E_NOMEM, "rank buffers");
  IX_TRY(x, cudaMemcpyAsync(x->qf.p, query, sizeof(float) * x->dim, cudaMemcpyHostToDevice, st));
  IX_TRY(x, rv::scan_round_queries(x->qf.p, x->qb.p, x->dim, st));
  IX_TRY(x, cudaMemsetAsync(x->rank_cnt.p, 0, 2 * sizeof(unsigned long long), st));
  // Candidates: every row when nothing can be filtered, else the rows whose f32 score reaches
  // threshold - eps (eps: the f32 accumulation bound the top-k guard uses).
  const bool all_rows = !(threshold > -INFINITY);
  unsigned long long m = static_cast<unsigned long long>(n);
  if (!all_rows) {
    double qn2 = 0.0;
    for (int d = 0; d < x->dim; ++d) {
      const uint32_t bits = uint32_t(rv::f32_to_bf16_bits(query[d])) << 16;
      float v;
      std::memcpy(&v, &bits, 4);
      qn2 += double(v) * v;
    }
    const double eps = double(x->dim) * std::ldexp(1.0, -22) * x->max_norm * std::sqrt(qn2);
    const float lo = static_cast<float>(double(threshold) - eps - std::fabs(double(threshold)) * 1e-6);
    if (!x->rank_cand.reserve(size_t(n))) return ifail(x, RV_E_NOMEM, "rank candidate buffer");
    IX_TRY(x, rv::rank_filter(x->db, n, x->dim, x->qb.p, lo, x->rank_cand.p, x->rank_cnt.p, st));
    IX_TRY(x, cudaMemcpyAsync(&m, x->rank_cnt.p, sizeof(m), cudaMemcpyDeviceToHost, st));
    IX_TRY(x, cudaStreamSynchronize(st));
    x->launches++;
  }
  IX_TRY(x, rv::rank_exact(x->db, x->dim, x->qb.p, all_rows ? nullptr : x->rank_cand.p, int64_t(m), x->base,
                           double(threshold), x->rank_s.p, x->rank_i.p, x->rank_cnt.p + 1, st));
  unsigned long long kept = 0;
  IX_TRY(x, cudaMemcpyAsync(&kept, x->rank_cnt.p + 1, sizeof(kept), cudaMemcpyDeviceToHost, st));
  unsigned int e = 0;
  IX_TRY(x, cudaMemcpyAsync(&e, x->d_err, 4, cudaMemcpyDeviceToHost, st));
  IX_TRY(x, cudaStreamSynchronize(st));
  x->launches++;
  if (e) {
    cudaMemset(x->d_err, 0, 4);
    return ifail(x, RV_E_DEVICE, "rank kernel reported device error flags " + std::to_string(e));
  }
  *out_count = static_cast<int64_t>(kept);
  if (kept == 0 || capacity == 0) return RV_OK;
  size_t tmp_bytes = 0;
  IX_TRY(x, rv::rank_sort_desc(nullptr, &tmp_bytes, x->rank_s.p, x->rank_s2.p, x->rank_i.p, x->rank_i2.p,
                               int64_t(kept), st));
  if (!x->rank_tmp.reserve(tmp_bytes)) return ifail(x, RV_E_NOMEM, "rank sort scratch");
  IX_TRY(x, rv::rank_sort_desc(x->rank_tmp.p, &tmp_bytes, x->rank_s.p, x->rank_s2.p, x->rank_i.p,
                               x->rank_i2.p, int64_t(kept), st));
  x->launches++;
  // Every pair comes back: equal scores arrive in no fixed order and are put in row order here,
  // including a run that crosses the capacity.
  std::vector<double> hs(kept);
  std::vector<int64_t> hi(kept);
  IX_TRY(x, cudaMemcpyAsync(hs.data(), x->rank_s2.p, sizeof(double) * kept, cudaMemcpyDeviceToHost, st));
  IX_TRY(x, cudaMemcpyAsync(hi.data(), x->rank_i2.p, sizeof(int64_t) * kept, cudaMemcpyDeviceToHost, st));
  IX_TRY(x, cudaStreamSynchronize(st));
  const size_t out_n = std::min<size_t>(kept, size_t(capacity));
  for (size_t a = 0; a < out_n;) {
    size_t b = a + 1;
    while (b < kept && hs[b] == hs[a]) ++b;
    if (b - a > 1) std::sort(hi.begin() + a, hi.begin() + b);
    a = b;
  }
  for (size_t i = 0; i < out_n; ++i) {
    out_idx[i] = hi[i];
    out_score[i] = static_cast<float>(hs[i]);
    if (out_score64) out_score64[i] = hs[i];
  }
  return RV_OK;
}

int rv_topk_merge_device(int device, const int64_t* idx_in, const double* score_in, int32_t n_lists,
                         int32_t nq, int32_t k, float threshold, int64_t* idx_out, float* score_out,
                         double* score64_out, void* stream) {
  if (n_lists <= 0 || nq < 0 || k <= 0 || !idx_in || !score_in || !idx_out || !score_out)
    return RV_E_INVALID;
  if (int64_t(n_lists) * k > 8192) return RV_E_INVALID;
  if (nq == 0) return RV_OK;
  Dev g(device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rv::scan_merge(idx_in, score_in, n_lists, nq, k, threshold, idx_out, score_out, score64_out, st) !=
      cudaSuccess)
    return RV_E_CUDA;
  return cudaStreamSynchronize(st) == cudaSuccess ? RV_OK : RV_E_CUDA;
}

int rv_index_build_polar(rv_index* x, const float* rotation, int32_t bits) {
  if (!x) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(x->mu);
  if (!rotation) return ifail(x, RV_E_INVALID, "null rotation");
  if (bits < 1 || bits > 4) return ifail(x, RV_E_INVALID, "bits must be in [1, 4]");
  if (x->n <= 0) return ifail(x, RV_E_INVALID, "empty index");
  const int dim = x->dim, pairs = dim / 2, levels = 1 << bits;
  if (size_t(pairs) * levels * sizeof(float) > rv::kPolarMaxLutBytes)
    return ifail(x, RV_E_INVALID, "dimension too large for the PolarQuant query tables");
  Dev g(x->device);
  cudaStream_t st = x->stream;
  // rt[d * dim + j] = R[j][d]: the encode and table kernels read a column of R per dimension.
  std::vector<float> rt(size_t(dim) * dim);
  for (int j = 0; j < dim; ++j)
    for (int d = 0; d < dim; ++d) rt[size_t(d) * dim + j] = rotation[size_t(j) * dim + d];
  // theta_j = (j / levels) * 2 * PI - PI in f32 (turbo_quant.rs:104-109); cos / sin from the f64
  // functions rounded to f32.
  std::vector<float> cs(size_t(2) * levels);
  const float pi_f = 3.14159265358979323846f;
  for (int j = 0; j < levels; ++j) {
    volatile float t = static_cast<float>(j) / static_cast<float>(levels);
    t = t * 2.0f;
    t = t * pi_f;
    t = t - pi_f;
    cs[j] = static_cast<float>(std::cos(static_cast<double>(t)));
    cs[levels + j] = static_cast<float>(std::sin(static_cast<double>(t)));
  }
  const size_t rows_padded = size_t((x->n + 31) / 32) * 32;
  if (!x->pq_rt.reserve(rt.size()) || !x->pq_cs.reserve(cs.size()) ||
      !x->pq_radii.reserve(rows_padded * pairs) || !x->pq_bins.reserve(rows_padded * pairs))
    return ifail(x, RV_E_NOMEM, "PolarQuant corpus allocation failed");
  IX_TRY(x, cudaMemcpyAsync(x->pq_rt.p, rt.data(), rt.size() * sizeof(float), cudaMemcpyHostToDevice, st));
  IX_TRY(x, cudaMemcpyAsync(x->pq_cs.p, cs.data(), cs.size() * sizeof(float), cudaMemcpyHostToDevice, st));
  IX_TRY(x, cudaMemsetAsync(x->pq_radii.p, 0, rows_padded * pairs * sizeof(float), st));
  IX_TRY(x, cudaMemsetAsync(x->pq_bins.p, 0, rows_padded * pairs, st));
  IX_TRY(x, rv::polar_encode(x->db, x->n, dim, x->pq_rt.p, levels, x->pq_radii.p, x->pq_bins.p, st));
  x->launches++;
  IX_TRY(x, cudaStreamSynchronize(st));
  x->pq_levels = levels;
  return RV_OK;
}

int rv_index_has_polar(const rv_index* x) { return x && x->pq_levels ? 1 : 0; }

int rv_index_polar_export(rv_index* x, float* radii, uint8_t* bins) {
  if (!x) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(x->mu);
  if (!x->pq_levels) return ifail(x, RV_E_NOT_READY, "no PolarQuant corpus");
  if (!radii || !bins) return ifail(x, RV_E_INVALID, "null argument");
  Dev g(x->device);
  const int pairs = x->dim / 2;
  const size_t rows_padded = size_t((x->n + 31) / 32) * 32;
  std::vector<float> r(rows_padded * pairs);
  std::vector<uint8_t> b(rows_padded * pairs);
  IX_TRY(x, cudaMemcpyAsync(r.data(), x->pq_radii.p, r.size() * sizeof(float), cudaMemcpyDeviceToHost, x->stream));
  IX_TRY(x, cudaMemcpyAsync(b.data(), x->pq_bins.p, b.size(), cudaMemcpyDeviceToHost, x->stream));
  IX_TRY(x, cudaStreamSynchronize(x->stream));
  for (int64_t row = 0; row < x->n; ++row) {
    const int64_t grp = row / 32;
    const int lane = static_cast<int>(row % 32);
    for (int p = 0; p < pairs; ++p) {
      radii[size_t(row) * pairs + p] = r[((size_t(grp) * (pairs / 4) + p / 4) * 32 + lane) * 4 + (p % 4)];
      bins[size_t(row) * pairs + p] = b[((size_t(grp) * (pairs / 16) + p / 16) * 32 + lane) * 16 + (p % 16)];
    }
  }
  return RV_OK;
}

int rv_index_polar_scores(rv_index* x, const float* queries, int32_t nq, float* scores) {
  if (!x) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(x->mu);
  if (!x->pq_levels) return ifail(x, RV_E_NOT_READY, "no PolarQuant corpus");
  if (nq < 0 || (nq > 0 && (!queries || !scores))) return ifail(x, RV_E_INVALID, "null argument");
  if (nq == 0) return RV_OK;
  Dev g(x->device);
  cudaStream_t st = x->stream;
  const int dim = x->dim, pairs = dim / 2, levels = x->pq_levels;
  if (!x->qf.reserve(size_t(nq) * dim) || !x->pq_lut.reserve(size_t(nq) * pairs * levels) ||
      !x->pq_s.reserve(size_t(nq) * x->n))
    return ifail(x, RV_E_NOMEM, "PolarQuant score buffers");
  IX_TRY(x, cudaMemcpyAsync(x->qf.p, queries, sizeof(float) * size_t(nq) * dim, cudaMemcpyHostToDevice, st));
  IX_TRY(x, rv::polar_query_tables(x->qf.p, nq, dim, x->pq_rt.p, x->pq_cs.p, levels, x->pq_lut.p, st));
  IX_TRY(x, rv::polar_scan(x->pq_radii.p, x->pq_bins.p, pairs, 0, x->n, x->pq_lut.p, nq, levels, x->pq_s.p, x->n,
                           st));
  IX_TRY(x, cudaMemcpyAsync(scores, x->pq_s.p, sizeof(float) * size_t(nq) * x->n, cudaMemcpyDeviceToHost, st));
  IX_TRY(x, cudaStreamSynchronize(st));
  return RV_OK;
}

int rv_index_rank_turboquant_device(rv_index* x, const float* q_dev, int32_t nq, int32_t top_k, float threshold,
                                    int64_t* out_i, float* out_s, double* out_s64, void* stream) {
  if (!x) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(x->mu);
  if (nq < 0 || (nq > 0 && (!q_dev || !out_i || !out_s))) return ifail(x, RV_E_INVALID, "null argument");
  Dev g(x->device);
  cudaStream_t user = static_cast<cudaStream_t>(stream);
  cudaEvent_t ev = nullptr;
  if (user) {
    IX_TRY(x, cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    IX_TRY(x, cudaEventRecord(ev, user));
    IX_TRY(x, cudaStreamWaitEvent(x->stream, ev, 0));
  }
  int rc = tq_device(x, q_dev, nq, top_k, threshold, out_i, out_s, out_s64, nullptr);
  if (ev) {
    if (rc == RV_OK) {
      cudaEventRecord(ev, x->stream);
      cudaStreamWaitEvent(user, ev, 0);
    }
    cudaEventDestroy(ev);
  }
  return rc;
}

int rv_index_rank_turboquant(rv_index* x, const float* queries, int32_t nq, int32_t top_k, float threshold,
                             int64_t* out_idx, float* out_score, double* out_score64, int32_t* out_count) {
  if (!x) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(x->mu);
  if (nq < 0 || (nq > 0 && (!queries || !out_idx || !out_score)))
    return ifail(x, RV_E_INVALID, "null argument");
  if (nq == 0) return RV_OK;
  if (top_k <= 0 || top_k > kTqMaxTopK)
    return ifail(x, RV_E_INVALID, "top_k must be in [1, " + std::to_string(kTqMaxTopK) + "]");
  Dev g(x->device);
  cudaStream_t st = x->stream;
  const size_t nk = size_t(nq) * top_k;
  if (!x->qf.reserve(size_t(nq) * x->dim) || !x->oi.reserve(nk) || !x->os.reserve(nk) ||
      (out_score64 && !x->os64.reserve(nk)))
    return ifail(x, RV_E_NOMEM, "turboquant buffers");
  IX_TRY(x, cudaMemcpyAsync(x->qf.p, queries, sizeof(float) * size_t(nq) * x->dim, cudaMemcpyHostToDevice, st));
  std::vector<int> counts;
  int rc = tq_device(x, x->qf.p, nq, top_k, threshold, x->oi.p, x->os.p, out_score64 ? x->os64.p : nullptr,
                     &counts);
  if (rc) return rc;
  IX_TRY(x, cudaMemcpyAsync(out_idx, x->oi.p, sizeof(int64_t) * nk, cudaMemcpyDeviceToHost, st));
  IX_TRY(x, cudaMemcpyAsync(out_score, x->os.p, sizeof(float) * nk, cudaMemcpyDeviceToHost, st));
  if (out_score64)
    IX_TRY(x, cudaMemcpyAsync(out_score64, x->os64.p, sizeof(double) * nk, cudaMemcpyDeviceToHost, st));
  IX_TRY(x, cudaStreamSynchronize(st));
  if (out_count)
    for (int q = 0; q < nq; ++q) out_count[q] = counts[q];
  return RV_OK;
}

int rv_index_build_cascade(rv_index* x, int32_t trunc_dim) {
  if (!x) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(x->mu);
  if (x->n <= 0) return ifail(x, RV_E_INVALID, "empty index");
  const int t = std::min<int>(trunc_dim, x->dim);  // index.rs:99 clamps to hidden_dim
  if (t <= 0 || t % 64 != 0) return ifail(x, RV_E_INVALID, "truncated dimension must be a positive multiple of 64");
  if (rv::cascade_rows_smem(x->dim, t) > rv::kCascadeMaxSmem)
    return ifail(x, RV_E_INVALID, "dimension too large for the cascade transform");
  Dev g(x->device);
  __nv_bfloat16* tmp = nullptr;
  IX_TRY(x, cudaMalloc(&tmp, size_t(x->n) * t * 2));
  cudaError_t e = rv::cascade_rows(x->db, x->n, x->dim, t, tmp, x->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(x->stream);
  if (e != cudaSuccess) {
    cudaFree(tmp);
    return ifail(x, RV_E_CUDA, std::string("cascade_rows: ") + cudaGetErrorString(e));
  }
  x->launches++;
  rv_index* c = nullptr;
  const int rc = rv_index_create(x->device, tmp, x->n, t, RV_DTYPE_BF16, 1, &c);
  cudaFree(tmp);
  if (rc != RV_OK) return ifail(x, rc, "truncated index creation failed");
  rv_index_destroy(x->cascade);
  x->cascade = c;
  return RV_OK;
}

int rv_index_cascade_dim(const rv_index* x) { return x && x->cascade ? x->cascade->dim : 0; }

int rv_index_rank_cascade(rv_index* x, const float* queries, int32_t nq, int32_t top_k, float threshold,
                          int64_t* out_idx, float* out_score, double* out_score64, int32_t* out_count) {
  if (!x) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(x->mu);
  if (nq < 0 || (nq > 0 && (!queries || !out_idx || !out_score)))
    return ifail(x, RV_E_INVALID, "null argument");
  if (nq == 0) return RV_OK;
  // pre_filter_k = max(100, 3 top_k) (index.rs:261) must fit one exact top-k call (<= 2048).
  if (top_k <= 0 || top_k > 682) return ifail(x, RV_E_INVALID, "top_k must be in [1, 682]");
  Dev g(x->device);
  cudaStream_t st = x->stream;
  const size_t nk = size_t(nq) * top_k;
  if (!x->qf.reserve(size_t(nq) * x->dim) || !x->oi.reserve(nk) || !x->os.reserve(nk) ||
      (out_score64 && !x->os64.reserve(nk)))
    return ifail(x, RV_E_NOMEM, "cascade buffers");
  IX_TRY(x, cudaMemcpyAsync(x->qf.p, queries, sizeof(float) * size_t(nq) * x->dim, cudaMemcpyHostToDevice, st));
  std::vector<int> counts;
  int rc;
  if (!x->cascade || x->n == 0) {
    // No truncated matrix: the exact ranking (index.rs:252-254 falls back to rank).
    rc = topk_device(x, x->qf.p, nq, top_k, threshold, x->oi.p, x->os.p, out_score64 ? x->os64.p : nullptr,
                     &counts);
  } else {
    rv_index* c = x->cascade;
    const int t = c->dim;
    const int pre = std::max(100, 3 * top_k);
    if (!x->c_q.reserve(size_t(nq) * t) || !x->c_oi.reserve(size_t(nq) * pre) || !x->c_os.reserve(size_t(nq) * pre) ||
        !x->qb.reserve(size_t(nq) * x->dim) || !x->cnt.reserve(size_t(nq)) || !x->guard.reserve(size_t(nq)))
      return ifail(x, RV_E_NOMEM, "cascade buffers");
    // Phase 1: exact top-pre of the truncated queries over the truncated rows, on the truncated
    // index's stream, ordered after the query transform by an event (no host synchronisation).
    IX_TRY(x, rv::cascade_queries(x->qf.p, nq, x->dim, t, x->c_q.p, st));
    if (!x->order_ev) IX_TRY(x, cudaEventCreateWithFlags(&x->order_ev, cudaEventDisableTiming));
    IX_TRY(x, cudaEventRecord(x->order_ev, st));
    {
      std::lock_guard<std::mutex> lc(c->mu);
      c->base = x->base;
      IX_TRY(x, cudaStreamWaitEvent(c->stream, x->order_ev, 0));
      rc = topk_device(c, x->c_q.p, nq, pre, -INFINITY, x->c_oi.p, x->c_os.p, nullptr, nullptr);
      if (rc) return ifail(x, rc, "cascade first phase: " + c->err);
      // Phase 2: exact rescoring of the candidates with the full rows (index.rs:287-296).
      // topk_device returned after synchronising c's stream; its counts are in c->cnt.
      IX_TRY(x, rv::scan_round_queries(x->qf.p, x->qb.p, int64_t(nq) * x->dim, st));
      IX_TRY(x, rv::scan_rescore(x->db, x->base, x->dim, x->qb.p, nq, x->c_os.p, x->c_oi.p, c->cnt.p, pre, top_k,
                                 x->n, 0.0, threshold, x->oi.p, x->os.p, out_score64 ? x->os64.p : nullptr,
                                 x->cnt.p, x->guard.p, st));
      x->launches += 3;
      // The counts come back with the results below (one synchronisation for both).
      counts.resize(nq);
      IX_TRY(x, cudaMemcpyAsync(counts.data(), x->cnt.p, sizeof(int) * nq, cudaMemcpyDeviceToHost, st));
    }
    rc = RV_OK;
  }
  if (rc) return rc;
  IX_TRY(x, cudaMemcpyAsync(out_idx, x->oi.p, sizeof(int64_t) * nk, cudaMemcpyDeviceToHost, st));
  IX_TRY(x, cudaMemcpyAsync(out_score, x->os.p, sizeof(float) * nk, cudaMemcpyDeviceToHost, st));
  if (out_score64)
    IX_TRY(x, cudaMemcpyAsync(out_score64, x->os64.p, sizeof(double) * nk, cudaMemcpyDeviceToHost, st));
  IX_TRY(x, cudaStreamSynchronize(st));
  if (out_count)
    for (int q = 0; q < nq; ++q) out_count[q] = counts[q];
  return RV_OK;
}

int rv_index_cascade_rows(rv_index* x, float* out) {
  if (!x) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(x->mu);
  if (!x->cascade) return ifail(x, RV_E_NOT_READY, "no truncated matrix");
  if (!out) return ifail(x, RV_E_INVALID, "null argument");
  Dev g(x->device);
  const size_t m = size_t(x->n) * x->cascade->dim;
  std::vector<uint16_t> h(m);
  IX_TRY(x, cudaMemcpy(h.data(), x->cascade->db, m * 2, cudaMemcpyDeviceToHost));
  for (size_t i = 0; i < m; ++i) {
    const uint32_t u = uint32_t(h[i]) << 16;
    std::memcpy(out + i, &u, 4);
  }
  return RV_OK;
}

int rv_index_find_duplicates(rv_index* x, float threshold, int64_t max_pairs, int64_t* out_a, int64_t* out_b,
                             float* out_score, double* out_score64, int64_t* out_count) {
  if (!x) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(x->mu);
  if (!out_count || (max_pairs > 0 && (!out_a || !out_b || !out_score)) || max_pairs < 0)
    return ifail(x, RV_E_INVALID, "null argument or negative max_pairs");
  *out_count = 0;
  if (x->n < 2 || max_pairs == 0) return RV_OK;  // index.rs:327-330
  Dev g(x->device);
  cudaStream_t st = x->stream;
  const int n = static_cast<int>(x->n), dim = x->dim;
  // Candidate bound: every pair whose exact score reaches a cut c has an f32 tensor-core score of
  // at least c - eps.
  const double eps = double(dim) * std::ldexp(1.0, -22) * x->max_norm * x->max_norm;
  long long cap = 1LL << 23;  // candidate records per pass (16 bytes each; RV_DUP_CAP_RECORDS for tests)
  if (const char* e = std::getenv("RV_DUP_CAP_RECORDS")) cap = std::max(1024LL, std::atoll(e));
  int strip = 16384;          // rows per GEMM launch (RV_DUP_STRIP_ROWS for tests)
  if (const char* e = std::getenv("RV_DUP_STRIP_ROWS")) strip = std::max(128, std::atoi(e) / 128 * 128);
  if (!x->dup_rec.reserve(size_t(cap)) || !x->dup_cnt.reserve(1))
    return ifail(x, RV_E_NOMEM, "duplicate candidate buffer allocation failed");
  // One pass over the upper triangle: the candidates of cut c into dup_rec, their count into m
  // (more than cap: the buffer overflowed and holds an arbitrary subset).
  auto pass = [&](double c, unsigned long long& m) -> int {
    const float thr_lo = std::nextafter(static_cast<float>(c - eps), -INFINITY);
    IX_TRY(x, cudaMemsetAsync(x->dup_cnt.p, 0, sizeof(unsigned long long), st));
    for (int r0 = 0; r0 < n; r0 += strip) {
      const int rows = std::min(strip, n - r0);
      const int cols = (n - r0 + 255) / 256 * 256;
      CUtensorMap ts;
      std::string why;
      if (!rv::make_tmap_2d_16bit(&ts, x->db + size_t(r0) * dim, true, dim, uint64_t(rows), uint64_t(dim) * 2, 64,
                                  128, &why))
        return ifail(x, RV_E_CUDA, why);
      IX_TRY(x, rv::dup_candidates(ts, x->tmap_db, rows, cols, dim, r0, n, thr_lo, x->dup_rec.p, x->dup_cnt.p, cap,
                                   x->d_err, st));
      x->launches++;
    }
    unsigned int e = 0;
    IX_TRY(x, cudaMemcpyAsync(&m, x->dup_cnt.p, sizeof(m), cudaMemcpyDeviceToHost, st));
    IX_TRY(x, cudaMemcpyAsync(&e, x->d_err, 4, cudaMemcpyDeviceToHost, st));
    IX_TRY(x, cudaStreamSynchronize(st));
    if (e) {
      cudaMemset(x->d_err, 0, 4);
      return ifail(x, RV_E_DEVICE, "duplicate search kernel reported device error flags " + std::to_string(e));
    }
    return RV_OK;
  };
  // The threshold first.  When more than cap candidates fall within the error bound of it, the
  // best max_pairs pairs lie above a higher cut: bisect the cut between the last value that
  // overflowed and the largest possible score until a pass fits and keeps at least max_pairs
  // exact pairs (every pair below such a cut ranks after all of them).  The reference scores
  // the whole n x n matrix and keeps the best max_pairs whatever their number.
  double cut = double(threshold), lo_c = double(threshold), hi_c = x->max_norm * x->max_norm + eps;
  unsigned long long m = 0;
  std::vector<int4> rec;
  std::vector<double> s64;
  for (int it = 0;; ++it) {
    if (const int rc = pass(cut, m)) return rc;
    const bool over = m > static_cast<unsigned long long>(cap);
    size_t kept = 0;
    if (!over) {
      rec.resize(m);
      s64.resize(m);
      if (m > 0) {
        if (!x->dup_s64.reserve(size_t(m))) return ifail(x, RV_E_NOMEM, "duplicate score buffer allocation failed");
        IX_TRY(x, rv::dup_rescore(x->db, dim, x->dup_rec.p, static_cast<long long>(m), x->dup_s64.p, st));
        x->launches++;
        IX_TRY(x, cudaMemcpyAsync(rec.data(), x->dup_rec.p, sizeof(int4) * m, cudaMemcpyDeviceToHost, st));
        IX_TRY(x, cudaMemcpyAsync(s64.data(), x->dup_s64.p, sizeof(double) * m, cudaMemcpyDeviceToHost, st));
        IX_TRY(x, cudaStreamSynchronize(st));
      }
      for (size_t t = 0; t < m; ++t) kept += s64[t] >= cut;
      if (cut == double(threshold) || kept >= size_t(max_pairs)) break;
      hi_c = cut;  // too few pairs above this cut: lower it
    } else {
      lo_c = cut;  // too many candidates: raise it
    }
    const double next = 0.5 * (lo_c + hi_c);
    if (it >= 60 || !(next > lo_c && next < hi_c))
      return ifail(x, RV_E_DEVICE,
                   "more than " + std::to_string(cap) + " pairs score within the f32 error bound of every cut " +
                       "that keeps " + std::to_string(max_pairs) + " pairs; raise the threshold");
    cut = next;
  }
  // Keep exact scores >= threshold; order (score desc, a asc, b asc); the best max_pairs.
  std::vector<size_t> keep;
  keep.reserve(m);
  for (size_t t = 0; t < m; ++t)
    if (s64[t] >= cut) keep.push_back(t);
  auto before = [&](size_t u, size_t v) {
    if (s64[u] != s64[v]) return s64[u] > s64[v];
    if (rec[u].x != rec[v].x) return rec[u].x < rec[v].x;
    return rec[u].y < rec[v].y;
  };
  const size_t out_n = std::min<size_t>(keep.size(), size_t(max_pairs));
  std::partial_sort(keep.begin(), keep.begin() + out_n, keep.end(), before);
  for (size_t t = 0; t < out_n; ++t) {
    const size_t u = keep[t];
    out_a[t] = x->base + rec[u].x;
    out_b[t] = x->base + rec[u].y;
    out_score[t] = static_cast<float>(s64[u]);
    if (out_score64) out_score64[t] = s64[u];
  }
  *out_count = static_cast<int64_t>(out_n);
  return RV_OK;
}

}  // extern "C"
