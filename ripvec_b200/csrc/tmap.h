// Host helpers: TMA tensor-map encoding (through the runtime's driver entry point, so the library
// needs no link-time libcuda), per-device attribute caching and device properties.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace rv {

// Encodes a 2-D row-major tensor [outer, inner] of 16-bit elements for tiled TMA copies with
// 128-byte (or 64-byte) swizzling and a box of [box_outer, box_inner] elements.  Returns false and fills
// *why on failure (base not 16-byte aligned, stride not a multiple of 16 bytes, ...).
bool make_tmap_2d_16bit(CUtensorMap* out, const void* base, bool is_bf16, uint64_t inner,
                        uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                        uint32_t box_outer, std::string* why, int swizzle_bytes = 128);

// Number of SMs of the current device (cached per device).
int device_sm_count();

}  // namespace rv
