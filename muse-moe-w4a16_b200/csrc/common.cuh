// Shared device helpers for the routed W4A16 MoE kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "muse_moe.h"

namespace muse {

constexpr int kBlock = 16;            // elements per e4m3 block scale (nvfp4.py:16)
constexpr int kMaxLocalExperts = 256; // routing histogram lives in shared memory
constexpr int kMaxTopK = 16;
constexpr float kPostNormEps = 1e-8f; // reference.py:24

__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// fp8 e4m3fn byte -> float (exact). Exponent bias 7, exponent 0 is subnormal (m/8 * 2^-6),
// S.1111.111 is NaN; there are no infinities.
__device__ __forceinline__ float e4m3_to_float(uint32_t b) {
  const uint32_t e = (b >> 3) & 0xF, m = b & 0x7;
  float v;
  if (e == 0) {
    v = (float)m * (1.0f / 512.0f);  // m/8 * 2^-6
  } else {
    v = __int_as_float(((e + 120u) << 23) | (m << 20));  // 2^(e-7) * (1 + m/8)
  }
  if (e == 15 && m == 7) v = __int_as_float(0x7FC00000);
  return (b & 0x80) ? -v : v;
}

// One E2M1 code (4 bits, sign in bit 3) -> float, as nvfp4.unpack_e2m1 decodes it.
__device__ __forceinline__ float e2m1_to_float(uint32_t c) {
  // magnitudes 0, .5, 1, 1.5, 2, 3, 4, 6 in units of 0.5: 0,1,2,3,4,6,8,12
  const uint32_t halves = (0xC8643210u >> ((c & 7) * 4)) & 0xF;
  const float v = (float)halves * 0.5f;
  return (c & 8) ? -v : v;
}

__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) {
  return __uint_as_float(((uint32_t)b) << 16);
}

// Error reporting of the C ABI: positive cudaError_t, or MUSE_ERR_*.
inline int last_launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MUSE_OK : (int)e;
}

}  // namespace muse
