// ring_common.cuh -- Z_2^64 helpers shared by the ring-matmul kernels.
#pragma once

#include <cstdint>

namespace sufb200 {

// Low word of the arithmetic right shift by `sh` of the signed 128-bit
// product acc * c (beaver_scaled_acc semantics, cuda/cuda_primitives.cu:391-417).
__device__ __forceinline__ uint64_t scaled_acc(uint64_t acc, int has_scale, int64_t c, int sh) {
  if (!has_scale) return acc;
  const int64_t a = static_cast<int64_t>(acc);
  const uint64_t lo = static_cast<uint64_t>(a) * static_cast<uint64_t>(c);
  if (sh <= 0) return lo;
  const int64_t hi = __mul64hi(a, c);
  if (sh >= 64) return static_cast<uint64_t>(hi >> (sh - 64 > 63 ? 63 : sh - 64));
  return (lo >> sh) | (static_cast<uint64_t>(hi) << (64 - sh));
}

}  // namespace sufb200
