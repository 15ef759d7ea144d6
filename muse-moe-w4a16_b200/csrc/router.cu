// Router top-k on the device: the caller side of the layer, producing topk_ids / topk_weights
// in-graph from a [T, E] score matrix. Restates the routing of reference.generate_input
// (reference.py:64-84): scores.topk(K) -> indices in descending score order, weights = the
// selected scores divided by their sum. Mode 1 is the softmax router of the synthetic configs
// (logits -> softmax -> top-K -> renormalise), which is the softmax over the K selected
// logits, since the full softmax's denominator cancels in the renormalisation.
//
// One warp per token: lane l holds scores l, l + 32, ... in registers; K rounds of a warp
// arg-max (larger score first; equal scores: lower expert id first; NaN above every number,
// as torch.topk orders it) pick the experts in order. Integer results are exact; the weights
// sum the K selected values in selection order in fp32.
#include "common.cuh"

namespace muse {

namespace {

constexpr int kRouterThreads = 256;            // 8 tokens per CTA
constexpr int kRouterMaxPerLane = 32;          // E <= 1024

// a ranks above b: NaN first, then larger value, then lower index
__device__ __forceinline__ bool ranks_above(float av, int ai, float bv, int bi) {
  const bool an = av != av, bn = bv != bv;
  if (an != bn) return an;
  if (!an && av != bv) return av > bv;
  return ai < bi;
}

template <int kPerLane>
__global__ void __launch_bounds__(kRouterThreads)
router_topk_kernel(const float* __restrict__ scores, int tokens, int n_experts, int top_k, int mode,
                   int32_t* __restrict__ topk_ids, float* __restrict__ topk_weights) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * (kRouterThreads / 32) + (threadIdx.x >> 5);
  if (t >= tokens) return;
  const float* row = scores + (size_t)t * n_experts;
  float v[kPerLane];
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < n_experts ? __ldg(row + e) : 0.f;
  }
  uint32_t taken = 0;  // bit i: element i of this lane already selected (or out of range)
#pragma unroll
  for (int i = 0; i < kPerLane; ++i)
    if (lane + 32 * i >= n_experts) taken |= 1u << i;
  float sel_v = 0.f;   // lane k keeps the k-th selected value
  int sel_i = 0;
  for (int k = 0; k < top_k; ++k) {
    // this lane's best remaining element
    float bv = 0.f;
    int bi = 0x7fffffff;
    bool have = false;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
      if ((taken >> i) & 1u) continue;
      const int e = lane + 32 * i;
      if (!have || ranks_above(v[i], e, bv, bi)) {
        bv = v[i];
        bi = e;
        have = true;
      }
    }
    // warp arg-max (lanes without a candidate carry index INT_MAX and lose every comparison)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oi != 0x7fffffff && (bi == 0x7fffffff || ranks_above(ov, oi, bv, bi))) {
        bv = ov;
        bi = oi;
      }
    }
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    if (lane == k) {
      sel_v = bv;
      sel_i = bi;
    }
  }
  // weights, in selection order
  float w = 0.f;
  if (mode == 0) {
    float sum = 0.f;
    for (int k = 0; k < top_k; ++k) sum += __shfl_sync(0xffffffffu, sel_v, k);
    w = sel_v / sum;
  } else {
    const float vmax = __shfl_sync(0xffffffffu, sel_v, 0);
    const float ex = lane < top_k ? __expf(sel_v - vmax) : 0.f;
    float sum = 0.f;
    for (int k = 0; k < top_k; ++k) sum += __shfl_sync(0xffffffffu, ex, k);
    w = ex / sum;
  }
  if (lane < top_k) {
    topk_ids[(size_t)t * top_k + lane] = sel_i;
    topk_weights[(size_t)t * top_k + lane] = w;
  }
}

template <int kPerLane>
cudaError_t launch_router(const float* scores, int tokens, int n_experts, int top_k, int mode,
                          int32_t* ids, float* weights, cudaStream_t stream) {
  const int per_cta = kRouterThreads / 32;
  router_topk_kernel<kPerLane><<<(tokens + per_cta - 1) / per_cta, kRouterThreads, 0, stream>>>(
      scores, tokens, n_experts, top_k, mode, ids, weights);
  return cudaGetLastError();
}

}  // namespace

}  // namespace muse

extern "C" int muse_moe_router_topk(const float* scores, int tokens, int n_experts, int top_k, int mode,
                                    int32_t* topk_ids, float* topk_weights, muse_stream_t stream) {
  using namespace muse;
  if (tokens < 0 || n_experts <= 0 || top_k <= 0 || (mode != 0 && mode != 1)) return MUSE_ERR_INVALID_ARGUMENT;
  if (top_k > kMaxTopK || top_k > n_experts || n_experts > 32 * kRouterMaxPerLane) return MUSE_ERR_UNSUPPORTED_SHAPE;
  if (tokens == 0) return MUSE_OK;
  if (!scores || !topk_ids || !topk_weights) return MUSE_ERR_INVALID_ARGUMENT;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (n_experts <= 64)
    e = launch_router<2>(scores, tokens, n_experts, top_k, mode, topk_ids, topk_weights, s);
  else if (n_experts <= 256)
    e = launch_router<8>(scores, tokens, n_experts, top_k, mode, topk_ids, topk_weights, s);
  else
    e = launch_router<kRouterMaxPerLane>(scores, tokens, n_experts, top_k, mode, topk_ids, topk_weights, s);
  return e == cudaSuccess ? MUSE_OK : (int)e;
}
