// prepare(): lossless repack of NVFP4 expert weights into the tiled layout of layout.cuh
// (replaces the Marlin repack of baseline.py:62-79,82-103). One CTA of 128 threads per
// (expert, 128-row tile, 128-element K chunk); thread = tile row.
#include "common.cuh"
#include "kernels.cuh"
#include "layout.cuh"

namespace muse {

namespace {

__global__ void __launch_bounds__(kTileM)
prepare_tiles_kernel(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ scales,
                     int rows, int k, int gate_up_inter, uint8_t* __restrict__ codes_out,
                     uint8_t* __restrict__ scales_out) {
  const int k_chunks = k / kChunkK;
  const int m_tiles = rows / kTileM;
  const int kc = blockIdx.x, m = blockIdx.y, e = blockIdx.z;
  const int r = threadIdx.x;
  const int src_row = gate_up_inter > 0 ? w13_tile_source_row(m, r, gate_up_inter) : m * kTileM + r;
  const size_t row_code_bytes = (size_t)k / 2, row_scale_bytes = (size_t)k / kBlock;
  const uint8_t* src = codes + ((size_t)e * rows + src_row) * row_code_bytes + (size_t)kc * kRowCodeBytes;
  const uint8_t* ssrc = scales + ((size_t)e * rows + src_row) * row_scale_bytes + (size_t)kc * kRowScaleBytes;
  const size_t tile = ((size_t)e * m_tiles + m) * k_chunks + kc;
  uint8_t* dst = codes_out + tile * kTileCodeBytes + (size_t)r * kRowCodeBytes;
  uint8_t* sdst = scales_out + tile * kTileScaleBytes + (size_t)r * kRowScaleBytes;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint4 v = reinterpret_cast<const uint4*>(src)[c];
    v.x = permute_codes(v.x);
    v.y = permute_codes(v.y);
    v.z = permute_codes(v.z);
    v.w = permute_codes(v.w);
    reinterpret_cast<uint4*>(dst)[code_slot(r, c)] = v;
  }
  *reinterpret_cast<uint2*>(sdst) = *reinterpret_cast<const uint2*>(ssrc);
}

}  // namespace

int launch_prepare_tiles(const uint8_t* codes, const uint8_t* scales, int n_experts, int rows,
                         int k, int gate_up_inter, uint8_t* codes_out, uint8_t* scales_out,
                         cudaStream_t stream) {
  dim3 grid(k / kChunkK, rows / kTileM, n_experts);
  prepare_tiles_kernel<<<grid, kTileM, 0, stream>>>(codes, scales, rows, k, gate_up_inter, codes_out,
                                                    scales_out);
  return last_launch_status();
}

}  // namespace muse
