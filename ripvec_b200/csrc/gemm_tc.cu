// Instantiations of the tcgen05 GEMM for the epilogues the encoders use.
#include "gemm_ln_epi.cuh"
#include "gemm_tc2.cuh"
#include "gemm_tc2_tma.cuh"
#include "kernels.h"
#include "tmap.h"

namespace rv {

namespace {

template <typename T>
EpiResidualStats<T> make_res_stats(const GemmArgs& a) {
  return EpiResidualStats<T>{static_cast<T*>(a.c), a.ldc, static_cast<float2*>(a.stats), a.stats_ld};
}
inline LnFold make_fold(const GemmArgs& a) {
  return LnFold{static_cast<const float2*>(a.stats), a.stats_ld, a.stats_n, a.csum, a.eps, a.N};
}
template <typename T>
EpiNormQkvRope<T> make_norm_rope(const GemmArgs& a) {
  return EpiNormQkvRope<T>{EpiQkvRope<T>{static_cast<T*>(a.c), a.ldc, a.rope_cols, a.pos, a.cos_t, a.sin_t},
                           make_fold(a)};
}
template <typename T>
EpiNormGeglu<T> make_norm_geglu(const GemmArgs& a) {
  return EpiNormGeglu<T>{EpiGeglu<T>{static_cast<T*>(a.c), a.ldc}, make_fold(a)};
}

template <typename T, int BN>
cudaError_t dispatch_epi(const GemmArgs& a, unsigned int* err, cudaStream_t st) {
  const int sms = device_sm_count();
  switch (a.epi) {
    case GemmEpi::kStore:
      return launch_gemm_tc<T, BN>(*a.tmA, *a.tmB, a.M, a.N, a.K, a.b_row_offset,
                                   EpiStore<T>{static_cast<T*>(a.c), a.ldc}, err, sms, st);
    case GemmEpi::kResidual:
      return launch_gemm_tc<T, BN>(*a.tmA, *a.tmB, a.M, a.N, a.K, a.b_row_offset,
                                   EpiResidual<T>{static_cast<T*>(a.c), a.ldc, a.bias}, err, sms,
                                   st);
    case GemmEpi::kGeglu:
      return launch_gemm_tc<T, BN>(*a.tmA, *a.tmB, a.M, a.N, a.K, a.b_row_offset,
                                   EpiGeglu<T>{static_cast<T*>(a.c), a.ldc}, err, sms, st);
    case GemmEpi::kQkvRope:
      return launch_gemm_tc<T, BN>(
          *a.tmA, *a.tmB, a.M, a.N, a.K, a.b_row_offset,
          EpiQkvRope<T>{static_cast<T*>(a.c), a.ldc, a.rope_cols, a.pos, a.cos_t, a.sin_t}, err,
          sms, st);
    case GemmEpi::kBias:
      return launch_gemm_tc<T, BN>(*a.tmA, *a.tmB, a.M, a.N, a.K, a.b_row_offset,
                                   EpiBias<T>{static_cast<T*>(a.c), a.ldc, a.bias}, err, sms, st);
    case GemmEpi::kBiasGelu:
      return launch_gemm_tc<T, BN>(*a.tmA, *a.tmB, a.M, a.N, a.K, a.b_row_offset,
                                   EpiBiasGelu<T>{static_cast<T*>(a.c), a.ldc, a.bias}, err, sms,
                                   st);
    case GemmEpi::kStoreF32:
      return launch_gemm_tc<T, BN>(*a.tmA, *a.tmB, a.M, a.N, a.K, a.b_row_offset,
                                   EpiStoreF32{static_cast<float*>(a.c), a.ldc}, err, sms, st);
    case GemmEpi::kResidualStats:
      if (BN != 256) return cudaErrorInvalidValue;
      return launch_gemm_tc<T, BN>(*a.tmA, *a.tmB, a.M, a.N, a.K, a.b_row_offset, make_res_stats<T>(a), err,
                                   sms, st);
    case GemmEpi::kNormQkvRope:
      return launch_gemm_tc<T, BN>(*a.tmA, *a.tmB, a.M, a.N, a.K, a.b_row_offset, make_norm_rope<T>(a), err,
                                   sms, st);
    case GemmEpi::kNormGeglu:
      return launch_gemm_tc<T, BN>(*a.tmA, *a.tmB, a.M, a.N, a.K, a.b_row_offset, make_norm_geglu<T>(a), err,
                                   sms, st);
  }
  return cudaErrorInvalidValue;
}

template <typename T>
cudaError_t dispatch_pair(const GemmArgs& a, unsigned int* err, cudaStream_t st) {
  const int sms = device_sm_count();
  if (a.tmC) {  // TMA-staged epilogue
    switch (a.epi) {
      case GemmEpi::kQkvRope:
        return launch_gemm_tc2_tma<T>(*a.tmA, *a.tmB, *a.tmC, a.M, a.N, a.K,
                                      TEpiQkv<T, false>{a.rope_cols, a.pos, a.cos_t, a.sin_t, make_fold(a)}, err,
                                      sms, st);
      case GemmEpi::kNormQkvRope:
        return launch_gemm_tc2_tma<T>(*a.tmA, *a.tmB, *a.tmC, a.M, a.N, a.K,
                                      TEpiQkv<T, true>{a.rope_cols, a.pos, a.cos_t, a.sin_t, make_fold(a)}, err,
                                      sms, st);
      case GemmEpi::kResidualStats:
        return launch_gemm_tc2_tma<T>(*a.tmA, *a.tmB, *a.tmC, a.M, a.N, a.K,
                                      TEpiResidualStats<T>{static_cast<float2*>(a.stats), a.stats_ld}, err, sms,
                                      st);
      case GemmEpi::kNormGeglu:
        return launch_gemm_tc2_tma<T>(*a.tmA, *a.tmB, *a.tmC, a.M, a.N, a.K, TEpiNormGeglu<T>{make_fold(a)}, err,
                                      sms, st);
      default:
        return cudaErrorInvalidValue;
    }
  }
  switch (a.epi) {
    case GemmEpi::kStore:
      return launch_gemm_tc2<T>(*a.tmA, *a.tmB, a.M, a.N, a.K, EpiStore<T>{static_cast<T*>(a.c), a.ldc}, err,
                                sms, st);
    case GemmEpi::kResidual:
      return launch_gemm_tc2<T>(*a.tmA, *a.tmB, a.M, a.N, a.K,
                                EpiResidual<T>{static_cast<T*>(a.c), a.ldc, a.bias}, err, sms, st);
    case GemmEpi::kGeglu:
      return launch_gemm_tc2<T>(*a.tmA, *a.tmB, a.M, a.N, a.K, EpiGeglu<T>{static_cast<T*>(a.c), a.ldc}, err,
                                sms, st);
    case GemmEpi::kQkvRope:
      return launch_gemm_tc2<T>(
          *a.tmA, *a.tmB, a.M, a.N, a.K,
          EpiQkvRope<T>{static_cast<T*>(a.c), a.ldc, a.rope_cols, a.pos, a.cos_t, a.sin_t}, err, sms, st);
    case GemmEpi::kStoreF32:
      return launch_gemm_tc2<T>(*a.tmA, *a.tmB, a.M, a.N, a.K, EpiStoreF32{static_cast<float*>(a.c), a.ldc},
                                err, sms, st);
    case GemmEpi::kBias:
      return launch_gemm_tc2<T>(*a.tmA, *a.tmB, a.M, a.N, a.K, EpiBias<T>{static_cast<T*>(a.c), a.ldc, a.bias},
                                err, sms, st);
    case GemmEpi::kBiasGelu:
      return launch_gemm_tc2<T>(*a.tmA, *a.tmB, a.M, a.N, a.K,
                                EpiBiasGelu<T>{static_cast<T*>(a.c), a.ldc, a.bias}, err, sms, st);
    case GemmEpi::kResidualStats:
      return launch_gemm_tc2<T>(*a.tmA, *a.tmB, a.M, a.N, a.K, make_res_stats<T>(a), err, sms, st);
    case GemmEpi::kNormQkvRope:
      return launch_gemm_tc2<T>(*a.tmA, *a.tmB, a.M, a.N, a.K, make_norm_rope<T>(a), err, sms, st);
    case GemmEpi::kNormGeglu:
      return launch_gemm_tc2<T>(*a.tmA, *a.tmB, a.M, a.N, a.K, make_norm_geglu<T>(a), err, sms, st);
  }
  return cudaErrorInvalidValue;
}

template <typename T>
cudaError_t dispatch_bn(const GemmArgs& a, unsigned int* err, cudaStream_t st) {
  if (a.K % kGemmBK != 0 || a.K <= 0) return cudaErrorInvalidValue;
  if ((a.epi == GemmEpi::kNormQkvRope || a.epi == GemmEpi::kNormGeglu) && a.N > 2560)
    return cudaErrorInvalidValue;  // column sums are staged in 10 KB of shared memory
  if (a.pair) {
    if (a.N % 256 != 0 || a.b_row_offset != 0) return cudaErrorInvalidValue;
    return dispatch_pair<T>(a, err, st);
  }
  if (a.bn == 256 && a.N % 256 == 0) return dispatch_epi<T, 256>(a, err, st);
  if (a.bn == 128 && a.N % 128 == 0) return dispatch_epi<T, 128>(a, err, st);
  return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t gemm_tc(Act act, const GemmArgs& a, unsigned int* err, cudaStream_t st) {
  if (act == Act::kBf16) return dispatch_bn<__nv_bfloat16>(a, err, st);
  return dispatch_bn<__half>(a, err, st);
}

}  // namespace rv
