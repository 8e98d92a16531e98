// Single-kernel C entry points used by the parity tests (one kernel per call, device buffers).
#include <cuda_runtime.h>

#include <climits>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/ripvec_b200.h"
#include "kernels.h"
#include "tmap.h"

namespace {

// One error word per device for the standalone entry points.
unsigned int* op_err_word() {
  static std::mutex mu;
  static unsigned int* words[64] = {nullptr};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!words[dev]) {
    if (cudaMalloc(&words[dev], 4) != cudaSuccess) return nullptr;
    cudaMemset(words[dev], 0, 4);
  }
  return words[dev];
}

int check_err_word(unsigned int* w, cudaStream_t st) {
  unsigned int h = 0;
  if (cudaMemcpyAsync(&h, w, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess) return RV_E_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return RV_E_CUDA;
  if (h) {
    cudaMemset(w, 0, 4);
    return RV_E_DEVICE;
  }
  return RV_OK;
}

}  // namespace

extern "C" {

int rv_op_gemm(int32_t act_dtype, const void* a, const void* b, void* c, int32_t c_dtype,
               int32_t M, int32_t N, int32_t K, int32_t bn, void* stream) {
  if (act_dtype != RV_DTYPE_BF16 && act_dtype != RV_DTYPE_F16) return RV_E_INVALID;
  if (c_dtype != RV_DTYPE_F32 && c_dtype != act_dtype) return RV_E_INVALID;
  const bool pair = bn == 512;  // two-CTA 256 x 256 tiles
  if (pair) bn = 256;
  if (M <= 0 || N <= 0 || K <= 0 || K % 64 != 0 || (bn != 128 && bn != 256) || N % bn != 0)
    return RV_E_INVALID;
  const bool bf = act_dtype == RV_DTYPE_BF16;
  CUtensorMap ta, tb;
  std::string why;
  if (!rv::make_tmap_2d_16bit(&ta, a, bf, K, M, uint64_t(K) * 2, 64, 128, &why)) return RV_E_INVALID;
  if (!rv::make_tmap_2d_16bit(&tb, b, bf, K, N, uint64_t(K) * 2, 64, pair ? 128 : bn, &why)) return RV_E_INVALID;
  unsigned int* err = op_err_word();
  if (!err) return RV_E_NOMEM;
  rv::GemmArgs g{};
  g.tmA = &ta;
  g.tmB = &tb;
  g.M = M;
  g.N = N;
  g.K = K;
  g.bn = bn;
  g.pair = pair;
  g.epi = c_dtype == RV_DTYPE_F32 ? rv::GemmEpi::kStoreF32 : rv::GemmEpi::kStore;
  g.c = c;
  g.ldc = N;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rv::gemm_tc(bf ? rv::Act::kBf16 : rv::Act::kF16, g, err, st) != cudaSuccess) return RV_E_CUDA;
  return check_err_word(err, st);
}

int rv_op_attention(int32_t act_dtype, const void* qkv, void* ctx_out, const int32_t* cu_host,
                    int32_t n_seqs, int32_t num_heads, int32_t head_dim, int32_t window_half,
                    float scale, void* stream) {
  if (act_dtype != RV_DTYPE_BF16 && act_dtype != RV_DTYPE_F16) return RV_E_INVALID;
  if (n_seqs <= 0 || !cu_host || (head_dim != 64 && head_dim != 32)) return RV_E_INVALID;
  for (int i = 0; i < n_seqs; ++i)
    if (cu_host[i + 1] < cu_host[i]) return RV_E_INVALID;
  const int total_tokens = cu_host[n_seqs];
  // head_dim 64 runs on the tcgen05 kernel unless RV_ATTN_TC=0.
  const char* env = std::getenv("RV_ATTN_TC");
  const bool tc = head_dim == 64 && !(env && std::strcmp(env, "0") == 0) &&
                  int64_t(total_tokens) * num_heads * head_dim <= INT32_MAX;
  std::vector<int> meta;  // tc: int2 tile records; else cu_seqlens then 64-query tile starts
  int q = 0;
  if (tc) {
    meta.resize(2 * (size_t(total_tokens) / 128 + n_seqs + 1));
    q = rv::fill_attention_tiles(cu_host, n_seqs, reinterpret_cast<int2*>(meta.data()));
    if (q < 0) return RV_E_INVALID;
  } else {
    meta.resize(2 * (n_seqs + 1));
    for (int i = 0; i <= n_seqs; ++i) {
      meta[i] = cu_host[i];
      meta[n_seqs + 1 + i] = q;
      if (i < n_seqs) q += (cu_host[i + 1] - cu_host[i] + 63) / 64;
    }
  }
  unsigned int* err = op_err_word();
  if (!err) return RV_E_CUDA;
  int* d = nullptr;
  if (cudaMalloc(&d, meta.size() * 4) != cudaSuccess) return RV_E_NOMEM;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const rv::Act act = act_dtype == RV_DTYPE_BF16 ? rv::Act::kBf16 : rv::Act::kF16;
  int rc = RV_OK;
  if (cudaMemcpyAsync(d, meta.data(), meta.size() * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
    rc = RV_E_CUDA;
  if (rc == RV_OK) {
    const cudaError_t e =
        tc ? rv::attention_varlen_tc(act, qkv, ctx_out, total_tokens, reinterpret_cast<const int2*>(d), q,
                                     num_heads, window_half, scale, err, st)
           : rv::attention_varlen(act, qkv, ctx_out, d, d + n_seqs + 1, n_seqs, q, num_heads,
                                  head_dim, window_half, scale, st);
    if (e != cudaSuccess) rc = RV_E_CUDA;
  }
  if (cudaStreamSynchronize(st) != cudaSuccess) rc = RV_E_CUDA;
  cudaFree(d);
  if (rc == RV_OK) rc = check_err_word(err, st);
  return rc;
}

int rv_debug_stall_attention(int32_t enable, int64_t wait_limit_cycles) {
  if (enable && wait_limit_cycles <= 0) return RV_E_INVALID;
  rv::attention_set_stall(enable, wait_limit_cycles);
  return RV_OK;
}

int rv_debug_exp2_poly(const float* x, float* y, int64_t n, void* stream) {
  if (n < 0 || (n > 0 && (!x || !y))) return RV_E_INVALID;
  if (n == 0) return RV_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rv::exp2_poly_eval(x, y, n, st) != cudaSuccess) return RV_E_CUDA;
  return cudaStreamSynchronize(st) == cudaSuccess ? RV_OK : RV_E_CUDA;
}

int rv_op_layernorm(int32_t act_dtype, const void* in, void* out, int32_t rows, int32_t hidden,
                    const float* gamma, const float* beta, float eps, void* stream) {
  if (act_dtype != RV_DTYPE_BF16 && act_dtype != RV_DTYPE_F16) return RV_E_INVALID;
  if (rows < 0 || hidden <= 0 || hidden > 768 || hidden % 8 != 0 || !gamma) return RV_E_INVALID;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rv::layernorm(act_dtype == RV_DTYPE_BF16 ? rv::Act::kBf16 : rv::Act::kF16, in, out, rows,
                    hidden, gamma, beta, eps, st) != cudaSuccess)
    return RV_E_CUDA;
  return cudaStreamSynchronize(st) == cudaSuccess ? RV_OK : RV_E_CUDA;
}

}  // extern "C"
