// The prepared ("tiled") NVFP4 weight layout shared by the repack kernel (prepare.cu) and the
// expert GEMM kernel (gemm_tc.cu). It is a lossless permutation of the original bytes, the
// same size as the original tensors (the repack that baseline.py:82-103 and
// submission_v6.py:138-246 do for their kernels, with this kernel's own order):
//
//   codes  [E][m_tiles][k_chunks][kTileM rows][kChunkK/2 bytes]   (8 KiB per tile)
//   scales [E][m_tiles][k_chunks][kTileM rows][kChunkK/16 bytes]  (1 KiB per tile)
//
// * One tile = 128 weight rows x 128 K elements; one bulk copy moves it into shared memory.
// * Row order inside a w13 tile pairs gate and up rows: in each 32-row group (one TMEM lane
//   quarter, one epilogue warp) rows 0-15 are gate rows and rows 16-31 the matching up rows,
//   so the SiLU(gate)*up epilogue pairs lane i with lane i^16. w2 tiles keep natural order.
// * The four 16-byte chunks of a row are stored at slot (chunk ^ ((row >> 1) & 3)), so the
//   dequant threads' 16-byte shared loads (thread = row) are free of bank conflicts.
// * Inside each 32-bit word the 8 E2M1 codes are bit-permuted (permute_codes) so that a
//   mask, or a rotate and a mask, drops each pair of codes into the bit positions of a bf16x2
//   whose value is the code's value times 2^-126 (see dequant8 in gemm_tc.cu).
#pragma once

#include <stdint.h>

namespace muse {

constexpr int kTileM = 128;                           // weight rows per tile (= MMA M)
constexpr int kChunkK = 128;                          // K elements per tile / pipeline stage
constexpr int kTileCodeBytes = kTileM * kChunkK / 2;  // 8192
constexpr int kTileScaleBytes = kTileM * kChunkK / 16;  // 1024
constexpr int kRowCodeBytes = kChunkK / 2;            // 64
constexpr int kRowScaleBytes = kChunkK / 16;          // 8

// Source row (within one expert's [2I] rows) of row r of w13 tile `m_tile`.
__host__ __device__ inline int w13_tile_source_row(int m_tile, int r, int inter) {
  const int q = r >> 5, i = r & 31;
  const int j = 64 * m_tile + 16 * q + (i & 15);  // intermediate index
  return i < 16 ? j : inter + j;
}

__host__ __device__ inline int code_slot(int row, int chunk) { return chunk ^ ((row >> 1) & 3); }

// Bit positions (m, e0, e1, sign) of element k's code in the permuted word. Element k's
// nibble in the original word holds (m, e0, e1, sign) in bits 0..3 (nvfp4.py:5-6,40-47).
//   k0,k1 -> bf16x2 #0 by mask          (positions 6,7,8,15 / 22,23,24,31)
//   k2,k3 -> bf16x2 #1 by rotl 4 + mask
//   k4,k5 -> bf16x2 #2 by rotl 10 + mask
//   k6,k7 -> bf16x2 #3 by (<<6 & mask) | (>>2 & mask)
__host__ __device__ inline uint32_t permute_codes(uint32_t w) {
  const uint8_t pos[8][4] = {{6, 7, 8, 15},   {22, 23, 24, 31}, {2, 3, 4, 11},   {18, 19, 20, 27},
                             {28, 29, 30, 5}, {12, 13, 14, 21}, {0, 1, 10, 9},   {16, 17, 26, 25}};
  uint32_t out = 0;
  for (int k = 0; k < 8; ++k) {
    const uint32_t nib = (w >> (4 * k)) & 0xF;
    for (int b = 0; b < 4; ++b) out |= ((nib >> b) & 1u) << pos[k][b];
  }
  return out;
}

}  // namespace muse
