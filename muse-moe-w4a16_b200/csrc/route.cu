// Token -> local-expert grouping: histogram, exclusive scan, stable scatter.
//
// Restates the pair order of ref_kernel (reference.py:99-102): experts ascending, and within
// an expert the (token, slot) pairs in ascending flat index t*K+s -- i.e. a stable counting
// sort of the flat pair list by local expert id. Plays the role of moe_align_block_size
// (baseline.py:121-130) without padding: GEMM tiles index the expert ranges directly.
#include "common.cuh"
#include "kernels.cuh"

namespace muse {

namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;

// One CTA. The pair list is walked in chunks of 1024 in flat order; inside a chunk a pair's
// position is  (expert base) + (pairs of the same expert in lower warps) + (rank in its warp),
// the warp rank coming from __match_any_sync. Chunks are processed in order, so the scatter
// is stable.
__global__ void __launch_bounds__(kThreads)
route_kernel(const int32_t* __restrict__ ids, int n_pairs, int lo, int n_local,
             int32_t* __restrict__ offsets, int32_t* __restrict__ pair_order,
             int32_t* __restrict__ pair_row) {
  __shared__ int hist[kMaxLocalExperts];
  __shared__ int base[kMaxLocalExperts];
  __shared__ int wcnt[kWarps][kMaxLocalExperts];
  __shared__ int wsum[8];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = tid; e < kMaxLocalExperts; e += kThreads) hist[e] = 0;
  for (int j = tid; j < kWarps * kMaxLocalExperts; j += kThreads) (&wcnt[0][0])[j] = 0;
  __syncthreads();

  for (int i = tid; i < n_pairs; i += kThreads) {
    const int e = ids[i] - lo;
    if ((unsigned)e < (unsigned)n_local) atomicAdd(&hist[e], 1);
  }
  __syncthreads();

  // Exclusive scan of hist[0, 256) by the first 8 warps.
  int v = 0, incl = 0;
  if (tid < kMaxLocalExperts) {
    v = hist[tid];
    incl = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += o;
    }
    if (lane == 31) wsum[warp] = incl;
  }
  __syncthreads();
  if (tid < kMaxLocalExperts) {
    int before = 0;
    for (int w = 0; w < warp; ++w) before += wsum[w];
    const int excl = before + incl - v;
    if (tid < n_local) {
      offsets[tid] = excl;
      base[tid] = excl;
    }
    if (tid == n_local - 1) offsets[n_local] = excl + v;
  }
  __syncthreads();

  const unsigned lt_mask = (1u << lane) - 1u;
  for (int chunk = 0; chunk < n_pairs; chunk += kThreads) {
    const int i = chunk + tid;
    const int e = (i < n_pairs) ? ids[i] - lo : -1;
    const bool local = (unsigned)e < (unsigned)n_local;
    const unsigned key = local ? (unsigned)e : 0xffffffffu;
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    const int rank = __popc(peers & lt_mask);
    if (local && lane == __ffs(peers) - 1) wcnt[warp][e] = __popc(peers);
    __syncthreads();
    if (local) {
      int pos = base[e] + rank;
      for (int w = 0; w < warp; ++w) pos += wcnt[w][e];
      pair_order[pos] = i;
      pair_row[i] = pos;
    } else if (i < n_pairs) {
      pair_row[i] = -1;
    }
    __syncthreads();
    for (int x = tid; x < n_local; x += kThreads) {
      int s = 0;
      for (int w = 0; w < kWarps; ++w) {
        s += wcnt[w][x];
        wcnt[w][x] = 0;
      }
      base[x] += s;
    }
    __syncthreads();
  }
  // Unused tail of pair_order is -1, so the buffer is fully determined by the input.
  const int total = base[n_local - 1];
  for (int r = total + tid; r < n_pairs; r += kThreads) pair_order[r] = -1;
}

// xs[r] = x[pair_order[r] / top_k] for the P = offsets[n_local] routed pairs: the GEMM1 B
// operand in expert-grouped order, so each token tile is a plain 2-D TMA box.
__global__ void __launch_bounds__(256)
gather_rows_kernel(const uint16_t* __restrict__ x, const int32_t* __restrict__ offsets,
                   const int32_t* __restrict__ pair_order, int n_local, int top_k, int hidden,
                   uint16_t* __restrict__ xs) {
  const int P = offsets[n_local];
  const int vec = hidden / 8;
  for (int r = blockIdx.x; r < P; r += gridDim.x) {
    const int tok = pair_order[r] / top_k;
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)tok * hidden);
    uint4* dst = reinterpret_cast<uint4*>(xs + (size_t)r * hidden);
    for (int i = threadIdx.x; i < vec; i += blockDim.x) dst[i] = src[i];
  }
}

}  // namespace

int launch_gather(const uint16_t* x, const int32_t* offsets, const int32_t* pair_order, int n_local,
                  int top_k, int max_rows, int hidden, uint16_t* xs, cudaStream_t stream) {
  const int grid = max_rows < 296 ? max_rows : 296;
  gather_rows_kernel<<<grid, 256, 0, stream>>>(x, offsets, pair_order, n_local, top_k, hidden, xs);
  return last_launch_status();
}

int launch_route(const int32_t* ids, int tokens, int top_k, int local_start, int local_count,
                 int32_t* offsets, int32_t* pair_order, int32_t* pair_row, cudaStream_t stream) {
  route_kernel<<<1, kThreads, 0, stream>>>(ids, tokens * top_k, local_start, local_count, offsets,
                                           pair_order, pair_row);
  return last_launch_status();
}

}  // namespace muse

extern "C" int muse_moe_route(const int32_t* topk_ids, int tokens, int top_k, int local_start,
                              int local_count, int32_t* expert_offsets, int32_t* pair_order,
                              int32_t* pair_row, muse_stream_t stream) {
  if (tokens < 0 || top_k <= 0 || local_count <= 0 || local_start < 0) return MUSE_ERR_INVALID_ARGUMENT;
  if (top_k > muse::kMaxTopK || local_count > muse::kMaxLocalExperts) return MUSE_ERR_UNSUPPORTED_SHAPE;
  if (!expert_offsets || (tokens > 0 && (!topk_ids || !pair_order || !pair_row)))
    return MUSE_ERR_INVALID_ARGUMENT;
  return muse::launch_route(topk_ids, tokens, top_k, local_start, local_count, expert_offsets,
                            pair_order, pair_row, (cudaStream_t)stream);
}
