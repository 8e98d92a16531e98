// Host helpers: TMA tensor-map encoding (through the runtime's driver entry point, so the library
// needs no link-time libcuda), per-device attribute caching and device properties.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>
#include <string>

namespace rv {

// One-time set-up per device (a kernel's shared-memory attribute, a cached property), safe when
// several host threads drive contexts on the same or different devices: run(fn) calls fn at most
// once successfully per device, under a lock; later calls see the flag without locking.  A
// failed fn is retried on the next call.
class PerDeviceOnce {
 public:
  template <class F>
  cudaError_t run(F&& fn) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return fn();
    if (done_[dev].load(std::memory_order_acquire)) return cudaSuccess;
    std::lock_guard<std::mutex> lk(mu_);
    if (done_[dev].load(std::memory_order_relaxed)) return cudaSuccess;
    e = fn();
    if (e == cudaSuccess) done_[dev].store(true, std::memory_order_release);
    return e;
  }

 private:
  static constexpr int kMaxDevices = 64;
  std::mutex mu_;
  std::atomic<bool> done_[kMaxDevices] = {};
};

// Encodes a 2-D row-major tensor [outer, inner] of 16-bit elements for tiled TMA copies with
// 128-byte (or 64-byte) swizzling and a box of [box_outer, box_inner] elements.  Returns false and fills
// *why on failure (base not 16-byte aligned, stride not a multiple of 16 bytes, ...).
bool make_tmap_2d_16bit(CUtensorMap* out, const void* base, bool is_bf16, uint64_t inner,
                        uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                        uint32_t box_outer, std::string* why, int swizzle_bytes = 128);

// Number of SMs of the current device (cached per device).
int device_sm_count();

}  // namespace rv
