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

// Multi-CTA routing of large batches (the same stable order as route_block): CTA b owns pairs
// [b * kRouteBlockPairs, (b + 1) * kRouteBlockPairs). Pass 1 counts each CTA's pairs per local
// expert; pass 2 (one CTA) turns the counts into each CTA's first row per expert -- expert
// ranges ascending, and inside an expert the CTAs in order -- and writes the expert offsets;
// pass 3 places each CTA's pairs from those bases in flat order.
constexpr int kRouteBlockPairs = 4096;

__global__ void __launch_bounds__(kThreads)
route_count_kernel(const int32_t* __restrict__ ids, int n_pairs, int lo, int n_local, int32_t* __restrict__ counts) {
  __shared__ int hist[kMaxLocalExperts];
  for (int e = threadIdx.x; e < kMaxLocalExperts; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int begin = blockIdx.x * kRouteBlockPairs, end = min(begin + kRouteBlockPairs, n_pairs);
  for (int i = begin + threadIdx.x; i < end; i += blockDim.x) {
    const int e = ids[i] - lo;
    if ((unsigned)e < (unsigned)n_local) atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < n_local; e += blockDim.x) counts[blockIdx.x * n_local + e] = hist[e];
}

// counts[b][e] -> first pair row of CTA b's pairs of expert e; offsets[0..n_local]; the unused
// tail of pair_order is set to -1.
__global__ void __launch_bounds__(kThreads)
route_bases_kernel(int32_t* __restrict__ counts, int nb, int n_pairs, int n_local, int32_t* __restrict__ offsets,
                   int32_t* __restrict__ pair_order) {
  __shared__ int wsum[kThreads / 32];
  __shared__ int s_total;
  const int e = threadIdx.x, lane = e & 31, warp = e >> 5;
  int total = 0;  // pairs of expert e over all CTAs
  if (e < n_local)
    for (int b = 0; b < nb; ++b) total += counts[b * n_local + e];
  // exclusive scan of the totals over experts (n_local <= 256 < kThreads)
  int incl = total;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += o;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  int before = 0;
  for (int w = 0; w < warp; ++w) before += wsum[w];
  const int excl = before + incl - total;
  if (e < n_local) {
    offsets[e] = excl;
    int run = excl;
    for (int b = 0; b < nb; ++b) {
      const int c = counts[b * n_local + e];
      counts[b * n_local + e] = run;
      run += c;
    }
    if (e == n_local - 1) {
      offsets[n_local] = run;
      s_total = run;
    }
  }
  __syncthreads();
  for (int r = s_total + threadIdx.x; r < n_pairs; r += blockDim.x) pair_order[r] = -1;
}

__global__ void __launch_bounds__(kThreads)
route_place_kernel(const int32_t* __restrict__ ids, int n_pairs, int lo, int n_local, const int32_t* __restrict__ bases,
                   int32_t* __restrict__ pair_order, int32_t* __restrict__ pair_row) {
  __shared__ int base[kMaxLocalExperts];
  __shared__ int wcnt[(kThreads / 32) * kMaxLocalExperts];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, warps = kThreads / 32;
  for (int e = tid; e < n_local; e += kThreads) base[e] = bases[blockIdx.x * n_local + e];
  for (int j = tid; j < warps * kMaxLocalExperts; j += kThreads) wcnt[j] = 0;
  __syncthreads();
  const int begin = blockIdx.x * kRouteBlockPairs, end = min(begin + kRouteBlockPairs, n_pairs);
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int chunk = begin; chunk < end; chunk += kThreads) {
    const int i = chunk + tid;
    const int e = (i < end) ? ids[i] - lo : -1;
    const bool local = (unsigned)e < (unsigned)n_local;
    const unsigned key = local ? (unsigned)e : 0xffffffffu;
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    const int rank = __popc(peers & lt_mask);
    if (local && lane == __ffs(peers) - 1) wcnt[warp * kMaxLocalExperts + e] = __popc(peers);
    __syncthreads();
    if (local) {
      int pos = base[e] + rank;
      for (int w = 0; w < warp; ++w) pos += wcnt[w * kMaxLocalExperts + e];
      pair_order[pos] = i;
      pair_row[i] = pos;
    } else if (i < end) {
      pair_row[i] = -1;
    }
    __syncthreads();
    for (int x = tid; x < n_local; x += kThreads) {
      int sum = 0;
      for (int w = 0; w < warps; ++w) {
        sum += wcnt[w * kMaxLocalExperts + x];
        wcnt[w * kMaxLocalExperts + x] = 0;
      }
      base[x] += sum;
    }
    __syncthreads();
  }
}

}  // namespace

size_t route_scratch_bytes(int n_pairs, int local_count) {
  const int nb = (n_pairs + kRouteBlockPairs - 1) / kRouteBlockPairs;
  return sizeof(int32_t) * (size_t)nb * local_count;
}

int launch_route_multi(const int32_t* ids, int tokens, int top_k, int local_start, int local_count,
                       int32_t* offsets, int32_t* pair_order, int32_t* pair_row, int32_t* scratch,
                       cudaStream_t stream) {
  const int n_pairs = tokens * top_k;
  const int nb = (n_pairs + kRouteBlockPairs - 1) / kRouteBlockPairs;
  if (nb <= 1)
    return launch_route(ids, tokens, top_k, local_start, local_count, offsets, pair_order, pair_row, stream);
  route_count_kernel<<<nb, kThreads, 0, stream>>>(ids, n_pairs, local_start, local_count, scratch);
  route_bases_kernel<<<1, kThreads, 0, stream>>>(scratch, nb, n_pairs, local_count, offsets, pair_order);
  route_place_kernel<<<nb, kThreads, 0, stream>>>(ids, n_pairs, local_start, local_count, scratch, pair_order,
                                                  pair_row);
  return last_launch_status();
}

int launch_gather(const uint16_t* x, const int32_t* offsets, const int32_t* pair_order, int n_local,
                  int top_k, int max_rows, int hidden, uint16_t* xs, cudaStream_t stream) {
  // up to 8 CTAs of 256 threads per SM (148 SMs): enough rows in flight to stream at HBM speed
  const int grid = max_rows < 1184 ? max_rows : 1184;
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
