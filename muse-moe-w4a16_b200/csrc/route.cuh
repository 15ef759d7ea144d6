// Token -> local-expert grouping by one CTA: histogram, exclusive scan, stable scatter.
//
// Restates the pair order of ref_kernel (reference.py:99-102): experts ascending, and within
// an expert the (token, slot) pairs in ascending flat index t*K+s -- a stable counting sort of
// the flat pair list by local expert id (the role of moe_align_block_size, baseline.py:121-130,
// without padding: GEMM tiles index the expert ranges directly). Used by the standalone route
// kernel and, for small batches, inside the first expert GEMM's prologue.
#pragma once

#include "common.cuh"

namespace muse {

// Shared-memory ints route_block needs for `threads` threads.
__host__ __device__ constexpr int route_scratch_ints(int threads) {
  return 2 * kMaxLocalExperts + 8 + (threads / 32) * kMaxLocalExperts;
}

// All threads of the CTA call this (blockDim.x >= 256, a multiple of 32). The pair list is
// walked in chunks of blockDim.x in flat order; inside a chunk a pair's position is (expert
// base) + (pairs of the same expert in lower warps) + (rank in its warp, from
// __match_any_sync). Chunks go in order, so the scatter is stable. Writes offsets[n_local+1],
// pair_order[n_pairs] (tail -1) and, when non-null, pair_row[n_pairs] (-1 for non-local).
// Ends with __syncthreads().
// Small lists (n_pairs <= kRouteDirectMax, blockDim.x > n_local): thread i places pair i directly --
// its position is (pairs of smaller local expert) + (pairs of its expert with smaller flat
// index), both counted over the list in shared memory -- one pass instead of a histogram,
// scan and per-warp scatter. Same output as the general path.
constexpr int kRouteDirectMax = 128;

__device__ inline void route_block_direct(const int32_t* __restrict__ ids, int n_pairs, int lo,
                                          int n_local, int* scratch, int32_t* offsets,
                                          int32_t* pair_order, int32_t* pair_row) {
  int* le = scratch;  // [n_pairs] local expert of each pair, or -1
  const int tid = threadIdx.x;
  if (tid < n_pairs) {
    const int e = ids[tid] - lo;
    le[tid] = (unsigned)e < (unsigned)n_local ? e : -1;
  }
  __syncthreads();
  int total = 0;  // local pairs (every thread counts them; used for the tail below)
  if (tid < n_pairs) {
    const int e = le[tid];
    int before = 0, rank = 0;
    for (int j = 0; j < n_pairs; ++j) {
      const int ej = le[j];
      total += ej >= 0;
      before += (unsigned)ej < (unsigned)e;  // 0 <= ej < e
      rank += (ej == e) & (j < tid);
    }
    if (e >= 0) {
      pair_order[before + rank] = tid;
      if (pair_row) pair_row[tid] = before + rank;
    } else {
      if (pair_row) pair_row[tid] = -1;
    }
    if (tid >= total) pair_order[tid] = -1;  // unused tail
  }
  if (tid <= n_local) {  // offsets[e] = local pairs of experts below e
    int c = 0;
    for (int j = 0; j < n_pairs; ++j) c += (unsigned)le[j] < (unsigned)tid;
    offsets[tid] = c;
  }
  __syncthreads();
}

__device__ inline void route_block(const int32_t* __restrict__ ids, int n_pairs, int lo, int n_local,
                                   int* scratch, int32_t* offsets, int32_t* pair_order,
                                   int32_t* pair_row) {
  // (the pass costs every thread O(n_pairs); at 256 pairs it is no faster than the general path)
  if (n_pairs <= kRouteDirectMax && (int)blockDim.x >= kRouteDirectMax && (int)blockDim.x > n_local) {
    route_block_direct(ids, n_pairs, lo, n_local, scratch, offsets, pair_order, pair_row);
    return;
  }
  int* hist = scratch;
  int* base = hist + kMaxLocalExperts;
  int* wsum = base + kMaxLocalExperts;
  int* wcnt = wsum + 8;  // [warps][kMaxLocalExperts]
  const int nthreads = blockDim.x, warps = nthreads >> 5;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = tid; e < kMaxLocalExperts; e += nthreads) hist[e] = 0;
  for (int j = tid; j < warps * kMaxLocalExperts; j += nthreads) wcnt[j] = 0;
  __syncthreads();

  for (int i = tid; i < n_pairs; i += nthreads) {
    const int e = ids[i] - lo;
    if ((unsigned)e < (unsigned)n_local) atomicAdd(&hist[e], 1);
  }
  __syncthreads();

  // exclusive scan of hist[0, 256) by the first 8 warps
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
  for (int chunk = 0; chunk < n_pairs; chunk += nthreads) {
    const int i = chunk + tid;
    const int e = (i < n_pairs) ? ids[i] - lo : -1;
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
      if (pair_row) pair_row[i] = pos;
    } else if (i < n_pairs && pair_row) {
      pair_row[i] = -1;
    }
    __syncthreads();
    for (int x = tid; x < n_local; x += nthreads) {
      int s = 0;
      for (int w = 0; w < warps; ++w) {
        s += wcnt[w * kMaxLocalExperts + x];
        wcnt[w * kMaxLocalExperts + x] = 0;
      }
      base[x] += s;
    }
    __syncthreads();
  }
  // unused tail of pair_order is -1, so the buffer is fully determined by the input
  const int total = base[n_local - 1];
  for (int r = total + tid; r < n_pairs; r += nthreads) pair_order[r] = -1;
  __syncthreads();
}

}  // namespace muse
