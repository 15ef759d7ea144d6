// Expert GEMMs on the CUDA cores: W4A16 dot products with fp32 accumulation.
//
// GEMM1 (w13) computes h = x[tok] . W13^T for the gate row j and the up row I+j together and
// writes silu(gate) * up as bf16 (reference.py:103-104; SGLang keeps this cache in bf16,
// baseline.py:132). GEMM2 (w2) computes y = inter . W2^T, applies the post-norm weight
// (1 + w) and accumulates each pair's sum of squares (reference.py:88-90, 105).
// Weights are decoded on the fly: e2m1 code * e4m3 block scale in fp32, the global scale
// applied to the finished dot product.
#include "common.cuh"
#include "kernels.cuh"

namespace muse {

namespace {

constexpr int kThreads = 256;
constexpr int kRowsPerCta = 32;   // output rows per CTA: 8 warps x 4 rows
constexpr int kTok = 8;           // tokens per pass

// Decode the 8 codes of one packed word (element 2i in the low nibble) times `scale`.
__device__ __forceinline__ void decode8(uint32_t w, float scale, float (&v)[8]) {
#pragma unroll
  for (int q = 0; q < 8; ++q) v[q] = e2m1_to_float((w >> (4 * q)) & 0xF) * scale;
}

__device__ __forceinline__ void bf16x8_to_float(uint4 p, float (&v)[8]) {
  const uint32_t w[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    v[2 * q] = __uint_as_float(w[q] << 16);
    v[2 * q + 1] = __uint_as_float(w[q] & 0xFFFF0000u);
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ uint16_t float_to_bf16_bits(float f) {
  const __nv_bfloat16 b = __float2bfloat16_rn(f);
  return *reinterpret_cast<const uint16_t*>(&b);
}

// Stage rows of a bf16 matrix (row i of the chunk = src row `row_of(i)`) into shared memory;
// rows past `nt` are zero.
template <typename RowOf>
__device__ __forceinline__ void stage_rows(uint4* dst, const uint16_t* src, int width, int nt,
                                           RowOf row_of) {
  const int vec_per_row = width / 8;
  for (int idx = threadIdx.x; idx < kTok * vec_per_row; idx += kThreads) {
    const int r = idx / vec_per_row, c = idx - r * vec_per_row;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (r < nt) val = reinterpret_cast<const uint4*>(src + (size_t)row_of(r) * width)[c];
    dst[idx] = val;
  }
}

__global__ void __launch_bounds__(kThreads)
gemm1_silu_simt(const uint16_t* __restrict__ x, const int32_t* __restrict__ offsets,
                const int32_t* __restrict__ pair_order, int top_k,
                const uint8_t* __restrict__ w13, const uint8_t* __restrict__ w13_sf,
                const float* __restrict__ gs13, int H, int I, uint16_t* __restrict__ inter) {
  extern __shared__ uint4 smem_x[];  // [kTok][H/8]
  const int e = blockIdx.y;
  const int begin = offsets[e], n = offsets[e + 1] - begin;
  if (n == 0) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float gs = gs13[e];
  const size_t row_bytes = H / 2, sf_bytes = H / kBlock;
  const uint8_t* w_e = w13 + (size_t)e * 2 * I * row_bytes;
  const uint8_t* s_e = w13_sf + (size_t)e * 2 * I * sf_bytes;
  const int words = H / 8;

  for (int c0 = 0; c0 < n; c0 += kTok) {
    const int nt = min(kTok, n - c0);
    __syncthreads();
    stage_rows(smem_x, x, H, nt, [&](int r) { return pair_order[begin + c0 + r] / top_k; });
    __syncthreads();
    for (int jj = 0; jj < kRowsPerCta / 8; ++jj) {
      const int j = blockIdx.x * kRowsPerCta + warp * (kRowsPerCta / 8) + jj;
      if (j >= I) break;
      const uint32_t* g_row = reinterpret_cast<const uint32_t*>(w_e + (size_t)j * row_bytes);
      const uint32_t* u_row = reinterpret_cast<const uint32_t*>(w_e + (size_t)(I + j) * row_bytes);
      const uint8_t* g_sf = s_e + (size_t)j * sf_bytes;
      const uint8_t* u_sf = s_e + (size_t)(I + j) * sf_bytes;
      float acc_g[kTok], acc_u[kTok];
#pragma unroll
      for (int t = 0; t < kTok; ++t) acc_g[t] = acc_u[t] = 0.f;
      for (int wd = lane; wd < words; wd += 32) {
        float fg[8], fu[8];
        decode8(g_row[wd], e4m3_to_float(g_sf[wd >> 1]), fg);
        decode8(u_row[wd], e4m3_to_float(u_sf[wd >> 1]), fu);
#pragma unroll
        for (int t = 0; t < kTok; ++t) {
          float fx[8];
          bf16x8_to_float(smem_x[t * words + wd], fx);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            acc_g[t] = fmaf(fg[q], fx[q], acc_g[t]);
            acc_u[t] = fmaf(fu[q], fx[q], acc_u[t]);
          }
        }
      }
#pragma unroll
      for (int t = 0; t < kTok; ++t) {
        const float g = warp_sum(acc_g[t]) * gs;
        const float u = warp_sum(acc_u[t]) * gs;
        if (lane == t && t < nt) {
          const float silu = g / (1.0f + __expf(-g));
          inter[(size_t)(begin + c0 + t) * I + j] = float_to_bf16_bits(silu * u);
        }
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads)
gemm2_norm_simt(const uint16_t* __restrict__ inter, const int32_t* __restrict__ offsets,
                const uint8_t* __restrict__ w2, const uint8_t* __restrict__ w2_sf,
                const float* __restrict__ gs2, const uint16_t* __restrict__ post_norm_w,
                int H, int I, float* __restrict__ ypart, float* __restrict__ ssq) {
  extern __shared__ uint4 smem_in[];  // [kTok][I/8]
  __shared__ float ssq_cta[kTok];
  const int e = blockIdx.y;
  const int begin = offsets[e], n = offsets[e + 1] - begin;
  if (n == 0) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float gs = gs2[e];
  const size_t row_bytes = I / 2, sf_bytes = I / kBlock;
  const uint8_t* w_e = w2 + (size_t)e * H * row_bytes;
  const uint8_t* s_e = w2_sf + (size_t)e * H * sf_bytes;
  const int words = I / 8;

  for (int c0 = 0; c0 < n; c0 += kTok) {
    const int nt = min(kTok, n - c0);
    __syncthreads();
    if (threadIdx.x < kTok) ssq_cta[threadIdx.x] = 0.f;
    stage_rows(smem_in, inter, I, nt, [&](int r) { return begin + c0 + r; });
    __syncthreads();
    float my_ssq = 0.f;  // lane t accumulates token t's partial sum of squares
    for (int jj = 0; jj < kRowsPerCta / 8; ++jj) {
      const int h = blockIdx.x * kRowsPerCta + warp * (kRowsPerCta / 8) + jj;
      if (h >= H) break;
      const uint32_t* row = reinterpret_cast<const uint32_t*>(w_e + (size_t)h * row_bytes);
      const uint8_t* sf = s_e + (size_t)h * sf_bytes;
      float acc[kTok];
#pragma unroll
      for (int t = 0; t < kTok; ++t) acc[t] = 0.f;
      for (int wd = lane; wd < words; wd += 32) {
        float fw[8];
        decode8(row[wd], e4m3_to_float(sf[wd >> 1]), fw);
#pragma unroll
        for (int t = 0; t < kTok; ++t) {
          float fx[8];
          bf16x8_to_float(smem_in[t * words + wd], fx);
#pragma unroll
          for (int q = 0; q < 8; ++q) acc[t] = fmaf(fw[q], fx[q], acc[t]);
        }
      }
      const float wn = 1.0f + bf16_bits_to_float(post_norm_w[h]);
#pragma unroll
      for (int t = 0; t < kTok; ++t) {
        const float y = warp_sum(acc[t]) * gs * wn;
        if (lane == t && t < nt) {
          ypart[(size_t)(begin + c0 + t) * H + h] = y;
          my_ssq = fmaf(y, y, my_ssq);
        }
      }
    }
    if (lane < nt) atomicAdd(&ssq_cta[lane], my_ssq);
    __syncthreads();
    if (threadIdx.x < nt) atomicAdd(&ssq[begin + c0 + threadIdx.x], ssq_cta[threadIdx.x]);
  }
}

}  // namespace

int launch_gemm1_silu(const LayerDims& d, const uint16_t* x, const ExpertWeights& w,
                      const Scratch& s, cudaStream_t stream) {
  const size_t smem = (size_t)kTok * d.hidden * 2;
  static bool attr_set = false;  // one process, attribute is per function
  if (!attr_set) {
    cudaFuncSetAttribute(gemm1_silu_simt, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    attr_set = true;
  }
  dim3 grid((d.inter + kRowsPerCta - 1) / kRowsPerCta, d.local_count);
  gemm1_silu_simt<<<grid, kThreads, smem, stream>>>(
      x, s.offsets, s.pair_order, d.top_k, w.w13, w.w13_sf, w.w13_gs, d.hidden, d.inter,
      reinterpret_cast<uint16_t*>(s.inter));
  return last_launch_status();
}

int launch_gemm2_norm(const LayerDims& d, const ExpertWeights& w, const Scratch& s,
                      cudaStream_t stream) {
  const size_t smem = (size_t)kTok * d.inter * 2;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(gemm2_norm_simt, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    attr_set = true;
  }
  dim3 grid((d.hidden + kRowsPerCta - 1) / kRowsPerCta, d.local_count);
  gemm2_norm_simt<<<grid, kThreads, smem, stream>>>(
      reinterpret_cast<const uint16_t*>(s.inter), s.offsets, w.w2, w.w2_sf, w.w2_gs,
      w.post_norm_w, d.hidden, d.inter, s.ypart, s.ssq);
  return last_launch_status();
}

}  // namespace muse
