// Top-k-weighted combine: out[t] = sum over t's local slots of
//   topk_weight[t, s] * rsqrt(mean(ypart[p]^2) + eps) * ypart[p],   p = pair_row[t*K + s],
// in fp32, cast to bf16 (reference.py:88-90, 106-107; the role of SGLang's Triton
// fused_post_expert_norm_weighted_sum, baseline.py:149-151). Tokens with no local pair get
// zeros. Slots are summed in ascending expert order, the order ref_kernel's index_add_ uses.
// The sum of squares of a pair is added up from its H/32 slice sums in a fixed order, so the
// result does not depend on how the GEMM's CTAs were scheduled.
#include "combine.cuh"
#include "common.cuh"
#include "kernels.cuh"

namespace muse {

namespace {

constexpr int kThreads = 256;
constexpr int kColsPerCta = kThreads * 4;

// grid (tokens, column blocks): a CTA covers columns [blockIdx.y * 1024, ...) in steps of
// gridDim.y * 1024, so with one column block it computes its token's coefficients once for the
// whole row (large batches), with several the row's columns spread over CTAs (small batches).
// Warp w computes the coefficients of slots w, w + 8, ...
// kF32Out: write the fp32 sum (an expert-parallel rank's partial) instead of bf16.
template <bool kF32Out>
__global__ void __launch_bounds__(kThreads)
combine_kernel(const int32_t* __restrict__ ids, const float* __restrict__ topk_weights,
               const int32_t* __restrict__ pair_row, const float* __restrict__ ypart,
               const float* __restrict__ ssq, int top_k, int H, void* __restrict__ out) {
  __shared__ int s_row[kMaxTopK], s_key[kMaxTopK], s_order[kMaxTopK], s_srow[kMaxTopK];
  __shared__ float s_coef[kMaxTopK], s_scoef[kMaxTopK];
  __shared__ int s_n;
  const int t = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int s = warp; s < top_k; s += kThreads / 32) {
    const int p = pair_row[t * top_k + s];
    float coef = 0.f;
    if (p >= 0) coef = post_norm_coef(ssq + (size_t)p * (H >> 5), H, topk_weights[t * top_k + s]);
    if (lane == 0) {
      s_row[s] = p;
      s_key[s] = ids[t * top_k + s];
      s_coef[s] = coef;
    }
  }
  __syncthreads();
  if (tid == 0) s_n = sort_local_slots(s_row, s_key, s_coef, top_k, s_order, s_srow, s_scoef);
  __syncthreads();
  for (int h4 = blockIdx.y * kThreads + tid; h4 * 4 < H; h4 += gridDim.y * kThreads) {  // float4 groups
    const float4 acc = weighted_rows(ypart, H, s_srow, s_scoef, s_n, h4);
    if (kF32Out)
      reinterpret_cast<float4*>(static_cast<float*>(out) + (size_t)t * H)[h4] = acc;
    else
      reinterpret_cast<uint2*>(static_cast<uint16_t*>(out) + (size_t)t * H)[h4] = pack_bf16x4(acc);
  }
}

// out[i] = bf16(in[i]), 8 elements per thread (n a multiple of 8).
__global__ void __launch_bounds__(256)
cast_bf16_kernel(const float4* __restrict__ in, uint4* __restrict__ out, size_t n8) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n8; i += (size_t)gridDim.x * blockDim.x) {
    const float4 a = in[2 * i], b = in[2 * i + 1];
    __nv_bfloat162 v[4] = {__floats2bfloat162_rn(a.x, a.y), __floats2bfloat162_rn(a.z, a.w),
                           __floats2bfloat162_rn(b.x, b.y), __floats2bfloat162_rn(b.z, b.w)};
    out[i] = *reinterpret_cast<const uint4*>(v);
  }
}

}  // namespace

int launch_combine(const LayerDims& d, const int32_t* ids, const float* topk_weights,
                   const Scratch& s, void* out, bool f32_out, cudaStream_t stream) {
  // small batches spread a row over CTAs (latency); from 1024 tokens on, one CTA per token
  // (its coefficients -- K rows of H/32 slice sums -- are read once, not once per column block)
  dim3 grid(d.tokens, d.tokens >= 1024 ? 1 : (d.hidden + kColsPerCta - 1) / kColsPerCta);
  if (f32_out)
    combine_kernel<true><<<grid, kThreads, 0, stream>>>(ids, topk_weights, s.pair_row, s.ypart,
                                                         s.ssq, d.top_k, d.hidden, out);
  else
    combine_kernel<false><<<grid, kThreads, 0, stream>>>(ids, topk_weights, s.pair_row, s.ypart,
                                                          s.ssq, d.top_k, d.hidden, out);
  return last_launch_status();
}

int launch_cast_bf16(const float* in, uint16_t* out, size_t n, cudaStream_t stream) {
  const size_t n8 = n / 8;
  if (n8 == 0) return MUSE_OK;
  const size_t blocks = (n8 + 255) / 256;
  cast_bf16_kernel<<<blocks < 1184 ? (unsigned)blocks : 1184u, 256, 0, stream>>>(
      reinterpret_cast<const float4*>(in), reinterpret_cast<uint4*>(out), n8);
  return last_launch_status();
}

}  // namespace muse
