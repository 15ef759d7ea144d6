// Standalone routing kernel (the grouping itself is route_block in route.cuh) and the
// activation-row gather that the larger batches use.
#include "common.cuh"
#include "kernels.cuh"
#include "route.cuh"

namespace muse {

namespace {

constexpr int kThreads = 1024;

// One CTA of 1024 threads sorts the whole pair list.
__global__ void __launch_bounds__(kThreads)
route_kernel(const int32_t* __restrict__ ids, int n_pairs, int lo, int n_local,
             int32_t* __restrict__ offsets, int32_t* __restrict__ pair_order,
             int32_t* __restrict__ pair_row) {
  __shared__ int scratch[route_scratch_ints(kThreads)];
  route_block(ids, n_pairs, lo, n_local, scratch, offsets, pair_order, pair_row);
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
