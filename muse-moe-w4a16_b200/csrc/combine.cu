// Top-k-weighted combine: out[t] = sum over t's local slots of
//   topk_weight[t, s] * rsqrt(mean(ypart[p]^2) + eps) * ypart[p],   p = pair_row[t*K + s],
// in fp32, cast to bf16 (reference.py:88-90, 106-107; the role of SGLang's Triton
// fused_post_expert_norm_weighted_sum, baseline.py:149-151). Tokens with no local pair get
// zeros. Slots are summed in ascending expert order, the order ref_kernel's index_add_ uses.
#include "common.cuh"
#include "kernels.cuh"

namespace muse {

namespace {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads)
combine_kernel(const int32_t* __restrict__ ids, const float* __restrict__ topk_weights,
               const int32_t* __restrict__ pair_row, const float* __restrict__ ypart,
               const float* __restrict__ ssq, int top_k, int H, uint16_t* __restrict__ out) {
  __shared__ int s_row[kMaxTopK];
  __shared__ float s_coef[kMaxTopK];
  __shared__ int s_n;
  const int t = blockIdx.x;
  if (threadIdx.x == 0) {
    // Collect the local slots, ordered by expert id (insertion sort over <= 16 entries).
    int n = 0;
    int key[kMaxTopK];
    for (int s = 0; s < top_k; ++s) {
      const int p = pair_row[t * top_k + s];
      if (p < 0) continue;
      const int e = ids[t * top_k + s];
      const float r = rsqrtf(ssq[p] / (float)H + kPostNormEps);
      const float c = topk_weights[t * top_k + s] * r;
      int j = n++;
      while (j > 0 && key[j - 1] > e) {
        key[j] = key[j - 1];
        s_row[j] = s_row[j - 1];
        s_coef[j] = s_coef[j - 1];
        --j;
      }
      key[j] = e;
      s_row[j] = p;
      s_coef[j] = c;
    }
    s_n = n;
  }
  __syncthreads();
  const int n = s_n;
  for (int h4 = threadIdx.x; h4 < H / 4; h4 += kThreads) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < n; ++j) {
      const float4 v = reinterpret_cast<const float4*>(ypart + (size_t)s_row[j] * H)[h4];
      const float c = s_coef[j];
      acc.x = fmaf(c, v.x, acc.x);
      acc.y = fmaf(c, v.y, acc.y);
      acc.z = fmaf(c, v.z, acc.z);
      acc.w = fmaf(c, v.w, acc.w);
    }
    __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y);
    __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z, acc.w);
    uint2 packed;
    packed.x = *reinterpret_cast<uint32_t*>(&lo);
    packed.y = *reinterpret_cast<uint32_t*>(&hi);
    reinterpret_cast<uint2*>(out + (size_t)t * H)[h4] = packed;
  }
}

}  // namespace

int launch_combine(const LayerDims& d, const int32_t* ids, const float* topk_weights,
                   const Scratch& s, uint16_t* out, cudaStream_t stream) {
  combine_kernel<<<d.tokens, kThreads, 0, stream>>>(ids, topk_weights, s.pair_row, s.ypart, s.ssq,
                                                    d.top_k, d.hidden, out);
  return last_launch_status();
}

}  // namespace muse
