// Internal launch interface between the kernel files and the C ABI (abi.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace muse {

// Geometry of one layer call, validated by the ABI before any launch.
struct LayerDims {
  int tokens, top_k, local_start, local_count, hidden, inter;
  int n_pairs() const { return tokens * top_k; }
};

// Scratch buffers carved from the caller's workspace (see workspace_layout in abi.cu).
struct Scratch {
  int32_t* offsets;     // [local_count + 1]
  int32_t* pair_order;  // [T*K]
  int32_t* pair_row;    // [T*K]
  void* inter;          // bf16 [T*K, I]   SiLU(gate)*up per pair, expert-grouped rows
  float* ypart;         // fp32 [T*K, H]   y * (1 + post_norm_w) per pair
  float* ssq;           // fp32 [T*K]      sum over H of ypart^2 per pair
};

// Weights of the local experts, already in the kernels' layout.
struct ExpertWeights {
  const uint8_t* w13;
  const uint8_t* w13_sf;
  const float* w13_gs;
  const uint8_t* w2;
  const uint8_t* w2_sf;
  const float* w2_gs;
  const uint16_t* post_norm_w;  // bf16 bits
};

int launch_route(const int32_t* ids, int tokens, int top_k, int local_start, int local_count,
                 int32_t* offsets, int32_t* pair_order, int32_t* pair_row, cudaStream_t stream);

int launch_gemm1_silu(const LayerDims& d, const uint16_t* x, const ExpertWeights& w,
                      const Scratch& s, cudaStream_t stream);

int launch_gemm2_norm(const LayerDims& d, const ExpertWeights& w, const Scratch& s,
                      cudaStream_t stream);

int launch_combine(const LayerDims& d, const int32_t* ids, const float* topk_weights,
                   const Scratch& s, uint16_t* out, cudaStream_t stream);

}  // namespace muse
