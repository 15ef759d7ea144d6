// Device helpers of the top-k-weighted combine, shared by the standalone combine kernel and the
// single-launch layer kernel's combine phase (reference.py:88-90,106-107). Both read every value
// through L2 (__ldcg): in the single launch the rows were written by other CTAs of the grid.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

#include "common.cuh"

namespace muse {

// Post-norm coefficient of one pair row, warp-wide: topk_weight * rsqrt(mean(y^2) + eps) from
// the row's H/32 slice sums of squares (H a multiple of 128). Lane l adds the float4 groups
// l, l + 32, ... in order, then the lanes are summed by a butterfly; every lane returns it.
__device__ __forceinline__ float post_norm_coef(const float* __restrict__ ssq_row, int H, float topk_weight) {
  const int lane = threadIdx.x & 31;
  const int groups = H >> 7;  // float4 groups of slice sums
  float sum = 0.f;
  for (int j = lane; j < groups; j += 32) {
    const float4 v = __ldcg(reinterpret_cast<const float4*>(ssq_row) + j);
    sum += (v.x + v.y) + (v.z + v.w);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  return topk_weight * rsqrtf(sum / (float)H + kPostNormEps);
}

// sum over j < n, in order, of coef[j] * ypart[row[j]][4 * h4 .. 4 * h4 + 3], fp32 (fmaf into the
// running sum). The loads of up to 8 rows are issued before their multiply-adds.
__device__ __forceinline__ float4 weighted_rows(const float* __restrict__ ypart, int H, const int* rows,
                                                const float* coefs, int n, int h4) {
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j0 = 0; j0 < n; j0 += 8) {
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (j0 + u < n) v[u] = __ldcg(reinterpret_cast<const float4*>(ypart + (size_t)rows[j0 + u] * H) + h4);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (j0 + u < n) {
        const float c = coefs[j0 + u];
        acc.x = fmaf(c, v[u].x, acc.x);
        acc.y = fmaf(c, v[u].y, acc.y);
        acc.z = fmaf(c, v[u].z, acc.z);
        acc.w = fmaf(c, v[u].w, acc.w);
      }
    }
  }
  return acc;
}

// Four fp32 -> four bf16 (round to nearest even), packed.
__device__ __forceinline__ uint2 pack_bf16x4(float4 v) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y);
  __nv_bfloat162 hi = __floats2bfloat162_rn(v.z, v.w);
  uint2 packed;
  packed.x = *reinterpret_cast<uint32_t*>(&lo);
  packed.y = *reinterpret_cast<uint32_t*>(&hi);
  return packed;
}

// Insertion sort of the local slots (row >= 0) by expert id; writes the sorted rows and
// coefficients and returns their count. One thread; top_k <= 16; `order` is scratch of top_k.
__device__ __forceinline__ int sort_local_slots(const int* row, const int* key, const float* coef, int top_k,
                                                int* order, int* srow, float* scoef) {
  int n = 0;
  for (int s = 0; s < top_k; ++s) {
    if (row[s] < 0) continue;
    int j = n++;
    while (j > 0 && key[order[j - 1]] > key[s]) {
      order[j] = order[j - 1];
      --j;
    }
    order[j] = s;
  }
  for (int j = 0; j < n; ++j) {
    srow[j] = row[order[j]];
    scoef[j] = coef[order[j]];
  }
  return n;
}

}  // namespace muse
