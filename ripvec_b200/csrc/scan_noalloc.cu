// rv_index_topk_noalloc: the exact top-k scan for callers that cannot allocate device memory.
//
// Some callers must not call cudaMalloc: a host application whose device memory is owned by its
// own allocator or memory pool under a hard budget, or a latency-critical serving thread where
// cudaMalloc / cudaFree would synchronise the device and stall every other stream.  This entry
// point runs the same kernels as rv_index_topk_device (tcgen05 score tiles, running top-kp
// select, exact f64 rescore) but keeps all of its scratch in the file-scope device array below,
// so a call allocates nothing: the caller passes the queries and the outputs, the index already
// holds the rows.
//
// The array is part of the library image: every GPU that loads the library holds it (about
// 5 MiB) until the process exits.  Its address is looked up once per device, with that device
// current, by the first call made on that device; make that first call before any stream
// capture.  All calls share the one array and it keeps the previous call's contents, so the
// candidate counts are cleared at the start of every call, and calls that overlap on the GPU
// (two streams, two threads, two indexes on the same device) race on it: serialise them.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/ripvec_b200.h"
#include "common.cuh"
#include "index_impl.h"
#include "kernels.h"
#include "scan.h"
#include "tmap.h"

namespace {

constexpr int kMaxQueries = 16;     // queries per call
constexpr int kMaxK = 64;           // results per query
constexpr int kCandidates = 128;    // candidate list width (2k rounded up, at least 128)
constexpr int kMaxDim = 4096;       // row dimension
constexpr int kChunkCols = 65536;   // database rows scored per GEMM launch
constexpr int kQueryRows = 128;     // query rows of the bf16 buffer: one whole GEMM tile

constexpr size_t align256(size_t b) { return (b + 255) / 256 * 256; }
constexpr size_t kScoresOff = 0;
constexpr size_t kScoresBytes = size_t(kMaxQueries) * kChunkCols * sizeof(float);
constexpr size_t kQueryOff = kScoresOff + align256(kScoresBytes);
// The queries are read through a 128-row TMA box; the buffer holds all 128 rows (zero past nq)
// so no box reaches past it: boxes mostly outside their tensor map (zero-filled by the copy
// engine) make the score GEMM of a small batch about 1.5x slower.
constexpr size_t kQueryBytes = size_t(kQueryRows) * kMaxDim * sizeof(__nv_bfloat16);
constexpr size_t kListSOff = kQueryOff + align256(kQueryBytes);
constexpr size_t kListSBytes = size_t(kMaxQueries) * kCandidates * sizeof(float);
constexpr size_t kListIOff = kListSOff + align256(kListSBytes);
constexpr size_t kListIBytes = size_t(kMaxQueries) * kCandidates * sizeof(int64_t);
constexpr size_t kListNOff = kListIOff + align256(kListIBytes);
constexpr size_t kCountOff = kListNOff + align256(kMaxQueries * sizeof(int));
constexpr size_t kGuardOff = kCountOff + align256(kMaxQueries * sizeof(int));
constexpr size_t kScratchBytes = kGuardOff + align256(kMaxQueries * sizeof(int));

// The scratch.  In host code this name is only a host-side stand-in for the device array:
// kernels get the address returned by cudaGetSymbolAddress, never this symbol.
static __device__ __align__(256) unsigned char g_topk_scratch[kScratchBytes];

// Device address of g_topk_scratch per device, looked up once with that device current.
unsigned char* scratch_for_current_device(std::string* why) {
  static std::mutex mu;
  static unsigned char* addr[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *why = "no current CUDA device";
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_topk_scratch);
    if (e != cudaSuccess || !p) {
      *why = std::string("cudaGetSymbolAddress of the top-k scratch failed: ") + cudaGetErrorString(e);
      return nullptr;
    }
    addr[dev] = static_cast<unsigned char*>(p);
  }
  return addr[dev];
}

int nfail(rv_index* x, int code, const std::string& m) {
  x->err = m;
  return code;
}

}  // namespace

extern "C" int rv_index_topk_noalloc(rv_index* x, const float* queries_dev, int32_t nq, int32_t k,
                                     float threshold, int64_t* out_idx_dev, float* out_score_dev,
                                     double* out_score64_dev, void* stream) {
  if (!x) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(x->mu);
  if (nq < 0 || nq > kMaxQueries)
    return nfail(x, RV_E_INVALID, "rv_index_topk_noalloc takes at most " + std::to_string(kMaxQueries) +
                                      " queries per call");
  if (k < 1 || k > kMaxK)
    return nfail(x, RV_E_INVALID, "rv_index_topk_noalloc takes k in [1, " + std::to_string(kMaxK) + "]");
  if (x->dim > kMaxDim)
    return nfail(x, RV_E_INVALID, "rv_index_topk_noalloc supports rows of at most " +
                                      std::to_string(kMaxDim) + " dimensions");
  if (nq == 0) return RV_OK;
  if (!queries_dev || !out_idx_dev || !out_score_dev) return nfail(x, RV_E_INVALID, "null argument");

  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) return nfail(x, RV_E_CUDA, "cudaGetDevice failed");
  if (prev != x->device) {
    const cudaError_t e = cudaSetDevice(x->device);
    if (e != cudaSuccess)
      return nfail(x, RV_E_CUDA, std::string("cudaSetDevice failed: ") + cudaGetErrorString(e));
  }
  struct Restore {
    int dev;
    ~Restore() {
      int cur = -1;
      cudaGetDevice(&cur);
      if (dev >= 0 && cur != dev) cudaSetDevice(dev);
    }
  } restore{prev};

  std::string why;
  unsigned char* base = scratch_for_current_device(&why);
  if (!base) return nfail(x, RV_E_CUDA, why);
  float* scores = reinterpret_cast<float*>(base + kScoresOff);
  __nv_bfloat16* qb = reinterpret_cast<__nv_bfloat16*>(base + kQueryOff);
  float* list_s = reinterpret_cast<float*>(base + kListSOff);
  int64_t* list_i = reinterpret_cast<int64_t*>(base + kListIOff);
  int* list_n = reinterpret_cast<int*>(base + kListNOff);
  int* cnt = reinterpret_cast<int*>(base + kCountOff);
  int* guard = reinterpret_cast<int*>(base + kGuardOff);
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : x->stream;

#define NA_TRY(expr)                                                                    \
  do {                                                                                  \
    cudaError_t _e = (expr);                                                            \
    if (_e != cudaSuccess) return nfail(x, RV_E_CUDA, std::string(#expr) + ": " + cudaGetErrorString(_e)); \
  } while (0)

  NA_TRY(rv::scan_round_queries(queries_dev, qb, int64_t(nq) * x->dim, st));
  NA_TRY(cudaMemsetAsync(qb + size_t(nq) * x->dim, 0, size_t(kQueryRows - nq) * x->dim * sizeof(__nv_bfloat16),
                         st));
  NA_TRY(rv::scan_init_lists(list_n, nq, st));  // the previous call's counts must not leak in
  const int kp = kCandidates;
  const int cap = rv::scan_cap_for(kp);
  if (x->n > 0) {
    CUtensorMap tq;
    if (!rv::make_tmap_2d_16bit(&tq, qb, true, x->dim, kQueryRows, uint64_t(x->dim) * 2, 64, 128, &why))
      return nfail(x, RV_E_CUDA, why);
    int64_t r0 = 0;
    int64_t chunk = std::max<int64_t>(256, (cap - kp) / 256 * 256);
    while (r0 < x->n) {
      const int64_t valid = std::min<int64_t>(chunk, x->n - r0);
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
      g.c = scores;
      g.ldc = static_cast<int>(ncols);
      NA_TRY(rv::gemm_tc(rv::Act::kBf16, g, x->d_err, st));
      NA_TRY(rv::scan_select(scores, static_cast<int>(ncols), static_cast<int>(valid), x->base + r0, nq,
                             kp, list_s, list_i, list_n, st));
      r0 += valid;
      const int64_t grow_to = (int64_t(cap - kp) * r0) / (4 * int64_t(kp));
      chunk = std::max<int64_t>(256, std::min<int64_t>(kChunkCols, grow_to) / 256 * 256);
    }
  }
  const double eps_scale = double(x->dim) * std::ldexp(1.0, -22) * x->max_norm;
  NA_TRY(rv::scan_rescore(x->db, x->base, x->dim, qb, nq, list_s, list_i, list_n, kp, k, x->n, eps_scale,
                          threshold, out_idx_dev, out_score_dev, out_score64_dev, cnt, guard, st));
  int guard_h[kMaxQueries] = {0};
  unsigned int err_h = 0;
  NA_TRY(cudaMemcpyAsync(guard_h, guard, sizeof(int) * nq, cudaMemcpyDeviceToHost, st));
  NA_TRY(cudaMemcpyAsync(&err_h, x->d_err, sizeof(err_h), cudaMemcpyDeviceToHost, st));
  NA_TRY(cudaStreamSynchronize(st));
#undef NA_TRY
  if (err_h) {
    cudaMemsetAsync(x->d_err, 0, sizeof(err_h), st);
    cudaStreamSynchronize(st);
    return nfail(x, RV_E_DEVICE, "scan kernel reported device error flags " + std::to_string(err_h));
  }
  for (int q = 0; q < nq; ++q)
    if (guard_h[q])
      return nfail(x, RV_E_DEVICE,
                   "near-equal scores need more than " + std::to_string(kCandidates) +
                       " candidates, more than the fixed scratch holds; use rv_index_topk_device");
  return RV_OK;
}
