// Instantiations of the tcgen05 GEMM for the epilogues the encoders use.
#include "gemm_tc.cuh"
#include "kernels.h"
#include "tmap.h"

namespace rv {

namespace {

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
  }
  return cudaErrorInvalidValue;
}

template <typename T>
cudaError_t dispatch_bn(const GemmArgs& a, unsigned int* err, cudaStream_t st) {
  if (a.K % kGemmBK != 0 || a.K <= 0) return cudaErrorInvalidValue;
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
