// Internal launch interface between the kernel files and the C ABI (abi.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
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
  uint16_t* xs;         // bf16 [T*K, H]  hidden states gathered into expert-grouped pair order
  uint16_t* inter;      // bf16 [T*K, I]  SiLU(gate)*up per pair, expert-grouped rows
  float* ypart;         // fp32 [T*K, H]  y * (1 + post_norm_w) per pair
  float* ssq;           // fp32 [T*K, H/32] sum of ypart^2 over each 32-column slice
  int* error_flag;      // set by a kernel whose bounded wait expired
};

// Weights of the local experts in the prepared (tiled) layout of layout.cuh.
struct ExpertWeights {
  const uint8_t* w13;
  const uint8_t* w13_sf;
  const float* w13_gs;
  const uint8_t* w2;
  const uint8_t* w2_sf;
  const float* w2_gs;
  const uint16_t* post_norm_w;  // bf16 bits
};

// One GEMM of a launch (gemm_tc.cu): its weights, its B operand and its epilogue.
struct PhaseArgs {
  int m_tiles;             // weight rows per expert / 128
  int k_chunks;            // K / 128
  const uint8_t* wq;       // prepared codes
  const uint8_t* wsf;      // prepared scales
  const float* gs;         // [n_local] global scales
  int mode;                // 1: SiLU(gate)*up -> inter; 2: post-norm partials -> ypart, ssq
  int ld_out;              // row length of the output (I in mode 1, H in mode 2)
  int split_k;             // split each item's chunks over the pipelines (else one pipeline per item;
                           // the kernel also splits any phase with fewer than 4 items per CTA)
  int b_source;            // B operand: 0 tmap_b boxes at the tile's rows (expert-grouped rows),
                           // 1 four-row gathers of x by token (tmap_x), 2 tmap_b2 boxes
  int* signal;             // single launch: GEMM1 -- per-token-tile counters, each epilogue warp
                           // adds 1 per item of the tile; GEMM2 -- one completion counter, each
                           // epilogue warp adds 1 after its last item (else null)
  const int* wait_for;     // counters that must reach wait_target before B is loaded (or null)
  int wait_target;
};

// Ranks of an expert-parallel exchange.
constexpr int kMaxPeers = 8;

// Expert-parallel decode in the single launch: after the combine has written this rank's fp32
// share (the launch's `out`), the one-round exchange of peer.cuh sums every rank's share into
// bf16 `out` here. Pointers of other ranks are peer mappings of their symmetric buffers.
struct ExchangeArgs {
  const float* share[2][kMaxPeers];  // share buffers of parity 0 / 1 of rank r
  uint32_t* flags[kMaxPeers];        // flag array of rank r
  uint16_t* out;                     // bf16 [n], this rank's memory
  size_t n4;                         // elements of a share / 4
  unsigned long long timeout_ns;
  int ranks;                         // 0: no exchange
  int rank, expect_parity;
};

// Arguments of one expert-GEMM launch. A launch runs one phase (a plain GEMM) or, for small
// batches, both GEMMs and the combine of the whole layer call (`fused`).
struct GemmArgs {
  int32_t* offsets;        // [n_local + 1] expert ranges of the pair rows (written if route_inline)
  int n_local;
  int n_box;               // token tile = MMA N (16, 32, 64 or 128)
  int pair_tiles;          // items cover two token tiles (one pipeline; n_box 128, separate launches)
  int stages;              // weight-tile ring depth (shared memory)
  int b_stages;            // activation-box ring depth (shared memory)
  int n_phases;            // 1 or 2
  PhaseArgs ph[2];
  uint16_t* inter;
  const uint16_t* post_norm_w;
  float* ypart;
  float* ssq;
  int* error_flag;
  uint32_t mul16, mul64;   // 16 and 64, passed at run time (see dequant8 in gemm_tc.cu)
  // Small batches: every CTA groups the pairs itself in its prologue (CTA 0 publishes
  // offsets / pair_order / pair_row) and phase 0 gathers activation rows straight from x.
  int route_inline;
  const int32_t* ids;      // [n_pairs] expert ids (route_inline)
  int n_pairs, local_start, top_k;
  int32_t* pair_order;
  int32_t* pair_row;
  // fused: after the GEMMs, each CTA combines tokens blockIdx.x, blockIdx.x + G, ... once the
  // GEMM2 completion counter ph[1].signal has every epilogue warp's increment (4 per CTA).
  int fused;
  int tokens, hidden;
  const float* topk_weights;
  void* out;
  int out_f32;
  ExchangeArgs ex;         // fused: the decode exchange after the combine (ex.ranks 0: none)
};

// Largest batch (tokens x top_k) whose routing the first GEMM does in its own prologue, and
// the largest token tile it gathers row by row.
constexpr int kMaxInlinePairs = 1024;
constexpr int kMaxInlineBox = 32;

int launch_route(const int32_t* ids, int tokens, int top_k, int local_start, int local_count,
                 int32_t* offsets, int32_t* pair_order, int32_t* pair_row, cudaStream_t stream);

// The same routing by several CTAs for large batches; `scratch` holds route_scratch_bytes().
size_t route_scratch_bytes(int n_pairs, int local_count);
int launch_route_multi(const int32_t* ids, int tokens, int top_k, int local_start, int local_count,
                       int32_t* offsets, int32_t* pair_order, int32_t* pair_row, int32_t* scratch,
                       cudaStream_t stream);

int launch_gather(const uint16_t* x, const int32_t* offsets, const int32_t* pair_order, int n_local,
                  int top_k, int max_rows, int hidden, uint16_t* xs, cudaStream_t stream);

size_t gemm_smem_bytes(int n_box, bool pair, int w_stages, int b_stages);
// Weight-ring depth for a token tile (pair: items of two token tiles); *b_stages receives the
// activation-ring depth.
int pick_stages(int n_box, bool pair, int* b_stages);
// tmap_b / tmap_b2: bf16 row buffers read as n_box-row boxes; tmap_x: x read by four-row gathers.
// A fused launch is cooperative (all CTAs resident) and needs its counters zeroed beforehand.
int launch_expert_gemm(const CUtensorMap& tmap_b, const CUtensorMap& tmap_x, const CUtensorMap& tmap_b2,
                       const GemmArgs& args, cudaStream_t stream);

// Address of the sticky device status word (current device) and a synchronous read of it.
int device_status_ptr(int** ptr);
int read_device_status(int* status, int reset);

int launch_combine(const LayerDims& d, const int32_t* ids, const float* topk_weights,
                   const Scratch& s, void* out, bool f32_out, cudaStream_t stream);

// out[i] = bf16(in[i]) for n elements (n a multiple of 8, both 16-byte aligned).
int launch_cast_bf16(const float* in, uint16_t* out, size_t n, cudaStream_t stream);

int launch_prepare_tiles(const uint8_t* codes, const uint8_t* scales, int n_experts, int rows,
                         int k, int gate_up_inter, uint8_t* codes_out, uint8_t* scales_out,
                         cudaStream_t stream);

// 2-D bf16 tensor map over a row-major [rows, cols] matrix, box = 64 columns x box_rows,
// 128-byte swizzle, zero fill out of bounds (box_rows = 1 for four-row gathers).
int make_bf16_tmap(CUtensorMap* map, const void* base, int rows, int cols, int box_rows);

}  // namespace muse
