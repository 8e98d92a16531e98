// Ordering and in-shared-memory sorting of (score, row) candidate lists shared by the scan
// kernels: best first = higher score, ties broken by the lower row index.
#pragma once

#include <stdint.h>

namespace rv {
namespace {

// (score desc, idx asc) "a comes before b".
__device__ __forceinline__ bool before(float sa, int64_t ia, float sb, int64_t ib) {
  return sa > sb || (sa == sb && ia < ib);
}
__device__ __forceinline__ bool before64(double sa, int64_t ia, double sb, int64_t ib) {
  return sa > sb || (sa == sb && ia < ib);
}

// Bitonic sort of n (power of two) (score, idx) pairs in shared memory, best first.
template <typename S>
__device__ void bitonic_sort(S* s, int64_t* id, int n) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int t = threadIdx.x; t < (n >> 1); t += blockDim.x) {
        const int lo = 2 * t - (t & (stride - 1));
        const int hi = lo + stride;
        const bool up = ((lo & size) == 0);  // block sorted best-first when up
        const S s_lo = s[lo], s_hi = s[hi];
        const int64_t i_lo = id[lo], i_hi = id[hi];
        const bool hi_first = (sizeof(S) == 8) ? before64(double(s_hi), i_hi, double(s_lo), i_lo)
                                               : before(float(s_hi), i_hi, float(s_lo), i_lo);
        if (hi_first == up) {
          s[lo] = s_hi;
          s[hi] = s_lo;
          id[lo] = i_hi;
          id[hi] = i_lo;
        }
      }
    }
  }
  __syncthreads();
}

}  // namespace
}  // namespace rv
