// Expert-parallel exchange over NVLink peer memory: the sum of every rank's fp32 share of the
// layer output, cast to bf16 -- on every rank for all elements (the all-reduce of the decode
// layout), or on each rank for its own slice of the elements (the reduce-scatter of the
// prefill layout) -- done by this kernel instead of a collective library.
//
// Each rank's share lives in its own symmetric buffer; the buffers of all ranks are mapped
// into every rank's address space (peer pointers). Every rank keeps, in its own flag array
// (kFlagWords uint32, zero before the first call), one round-1 and one round-2 slot per peer,
// its generation counter (calls completed) and three bookkeeping words. A call with generation
// g = counter + 1 (the same on every rank):
//   1. block 0 publishes "my share of call g is complete" by writing g into round-1 slot `rank`
//      of every rank's flag array (system-scope release after a system fence, so the share's
//      bytes -- written by the previous kernel on this stream -- are visible first);
//   2. every block waits (acquire, bounded) until all round-1 slots of its own array hold g;
//   3. reduce: element i of this rank's slice = bf16(sum over r = 0 .. R-1, in that order, of
//      share_r[i]) from the share buffers of parity g & 1. The slice is the whole share (one-round
//      all-reduce), this rank's 1/R of it (reduce-scatter), or, for the two-round all-reduce,
//      this rank's 1/R written both to the output and to its bf16 staging buffer;
//   4. two-round all-reduce only: the last block of this rank to finish step 3 publishes round 2
//      to every rank; every block waits (bounded) for all round-2 slots and then copies every
//      other rank's slice from that rank's staging buffer (gather);
//   5. the last block to finish stores g as the new counter -- unless a wait expired.
// Every element is summed by exactly one rank in rank order, so all ranks hold identical bits.
// The generation lives on the device, so a captured graph of the call stays valid across
// replays. Callers write call g's share into buffer g & 1: a rank rewrites a buffer only two
// calls later, after every peer has signalled the call in between (which it does only after
// finishing its reads of this rank's older share). A staging buffer is rewritten by its owner
// in the next call, after every peer's round-1 signal of that call, i.e. after their gathers.
//
// Prefill (tokens split over the ranks, T_r per rank) adds a dispatch before the layer and a
// routed mode of step 3 after it:
//   dispatch (ep_dispatch_kernel): rank s sends row t of its x to rank d's receive buffer, slot
//      s * T_r + t, only when d owns one of the token's experts (the token's destination mask,
//      also kept in this rank's `masks`), and the token's ids and weights to every rank (the
//      others route it nowhere). The last block then signals dispatch slot s of every rank and
//      waits, bounded, for all ranks' dispatch signals of the same generation: the receive
//      buffer is complete when the kernel ends. A rank rewrites a peer's receive buffer only in
//      the next call, after that peer's round-1 signal of this call, which follows its layer.
//   mode 3 (routed reduce-scatter): element (t, h) of this rank's slice = sum over the ranks in
//      the token's mask, in rank order, of their share's row rank * T_r + t -- the other ranks'
//      rows of that token are all zero and are never read over NVLink.
//
// Failure: a wait that runs past the caller's limit sets the sticky device status to 6 and
// this rank's call stops without advancing its generation (the output is then unspecified); a
// call whose generation parity differs from the caller's expectation does nothing and sets 7.
// Either way the exchange is out of step: re-create its flag arrays (zeroed, then a barrier of
// all ranks) before the next call.
#include "common.cuh"
#include "kernels.cuh"
#include "peer.cuh"
#include "ptx.cuh"

namespace muse {
namespace {

enum Mode { kAllReduce1 = 0, kReduceScatter = 1, kAllReduce2 = 2, kRoutedScatter = 3 };

struct PeerArgs {
  const float* share[2][kMaxPeers];  // share buffers of parity 0 / 1 of rank r (peer pointers)
  uint32_t* flags[kMaxPeers];        // flag array of rank r
  uint16_t* staging[kMaxPeers];      // bf16 staging buffer of rank r (two-round all-reduce)
  int ranks, rank, mode, expect_parity;
  unsigned long long timeout_ns;
  size_t slice4;                     // elements of one rank's slice / 4
  size_t n4;                         // elements of a share / 4
  uint16_t* out;                     // bf16, this rank's memory
  int* error_flag;
  const uint32_t* masks;             // mode 3: destination ranks of each of this rank's tokens
  int h4;                            // mode 3: float4 groups per token row
};

__device__ __forceinline__ uint2 sum_bf16x4(const PeerArgs& a, int par, size_t i4) {
  return rank_sum_bf16x4(a.share[par], a.ranks, i4);
}

// Mode 3: this rank's token t, float4 group c: the sum over the ranks in the token's mask.
__device__ __forceinline__ uint2 routed_sum_bf16x4(const PeerArgs& a, int par, size_t row, int c, uint32_t mask) {
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int r = 0; r < a.ranks; ++r) {
    if (!((mask >> r) & 1u)) continue;
    const float4 v = __ldcv(reinterpret_cast<const float4*>(a.share[par][r]) + row * a.h4 + c);
    acc.x += v.x;
    acc.y += v.y;
    acc.z += v.z;
    acc.w += v.w;
  }
  __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y);
  __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z, acc.w);
  uint2 packed;
  packed.x = *reinterpret_cast<uint32_t*>(&lo);
  packed.y = *reinterpret_cast<uint32_t*>(&hi);
  return packed;
}

__global__ void __launch_bounds__(256) peer_exchange_kernel(const PeerArgs a) {
  __shared__ int s_ok, s_last;
  __shared__ uint32_t s_gen;
  uint32_t* mine = a.flags[a.rank];
  if (threadIdx.x == 0) s_gen = *reinterpret_cast<volatile uint32_t*>(mine + kGenSlot) + 1u;
  __syncthreads();
  const uint32_t gen = s_gen;
  if (a.expect_parity >= 0 && (int)(gen & 1u) != a.expect_parity) {
    // the caller's share went to the other buffer: touch nothing, say so
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(a.error_flag, 7);
    return;
  }
  if (blockIdx.x == 0 && threadIdx.x < a.ranks) {
    __threadfence_system();
    st_release_sys(a.flags[threadIdx.x] + a.rank, gen);
  }
  if (threadIdx.x == 0) {
    s_ok = wait_slots(mine, 0, a.ranks, gen, a.timeout_ns);
    if (!s_ok) {
      atomicExch(mine + kFail, 1u);
      atomicExch(a.error_flag, 6);
    }
  }
  __syncthreads();
  const int par = gen & 1u;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (s_ok) {
    // step 3: this rank's slice (all of it for the one-round all-reduce)
    const size_t lo = a.mode == kAllReduce1 ? 0 : (size_t)a.rank * a.slice4;
    const size_t hi = a.mode == kAllReduce1 ? a.n4 : min(lo + a.slice4, a.n4);
    uint2* out = reinterpret_cast<uint2*>(a.out);
    uint2* stage = a.mode == kAllReduce2 ? reinterpret_cast<uint2*>(a.staging[a.rank]) : nullptr;
    if (a.mode == kRoutedScatter) {
      for (size_t i = lo + tid; i < hi; i += stride) {
        const size_t t = (i - lo) / a.h4;
        const int c = (int)(i - lo - t * a.h4);
        out[i - lo] = routed_sum_bf16x4(a, par, i / a.h4, c, __ldg(a.masks + t));
      }
    } else {
      for (size_t i = lo + tid; i < hi; i += stride) {
        const uint2 v = sum_bf16x4(a, par, i);
        out[a.mode == kReduceScatter ? i - lo : i] = v;
        if (stage) stage[i] = v;
      }
    }
  }
  if (a.mode == kAllReduce2) {
    // step 4: once every block of this rank has written its part of the slice, the last one
    // tells the peers (one thread per rank, so the signals go out in parallel)
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();
      s_last = 0;
      if (atomicAdd(mine + kDoneA, 1u) == gridDim.x - 1) {
        mine[kDoneA] = 0;
        __threadfence();
        s_last = !*reinterpret_cast<volatile uint32_t*>(mine + kFail);
      }
    }
    __syncthreads();
    if (s_last && threadIdx.x < a.ranks) {
      __threadfence_system();
      st_release_sys(a.flags[threadIdx.x] + kRound2 + a.rank, gen);
    }
    if (threadIdx.x == 0) {
      if (s_ok) {
        s_ok = wait_slots(mine, kRound2, a.ranks, gen, a.timeout_ns);
        if (!s_ok) {
          atomicExch(mine + kFail, 1u);
          atomicExch(a.error_flag, 6);
        }
      }
    }
    __syncthreads();
    if (s_ok) {
      uint4* out = reinterpret_cast<uint4*>(a.out);
      const size_t slice8 = a.slice4 / 2, n8 = a.n4 / 2;
      for (int k = 1; k < a.ranks; ++k) {
        const int r = (a.rank + k) % a.ranks;   // start with a different peer on every rank
        const size_t lo = (size_t)r * slice8, hi = min(lo + slice8, n8);
        const uint4* src = reinterpret_cast<const uint4*>(a.staging[r]);
        for (size_t i = lo + tid; i < hi; i += stride) out[i] = __ldcv(src + i);
      }
    }
  }
  // step 5: the last block out advances the generation (every block has read it by now)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(mine + kDoneB, 1u) == gridDim.x - 1) {
      mine[kDoneB] = 0;
      const bool failed = *reinterpret_cast<volatile uint32_t*>(mine + kFail) != 0;
      mine[kFail] = 0;
      __threadfence();
      if (!failed) *reinterpret_cast<volatile uint32_t*>(mine + kGenSlot) = gen;
    }
  }
}

struct DispatchArgs {
  const uint16_t* x;                 // bf16 [T_r, H], this rank's tokens
  const int32_t* ids;                // [T_r, K]
  const float* wts;                  // [T_r, K]
  uint16_t* recv_x[kMaxPeers];       // rank r's receive buffers (peer pointers): bf16 [R * T_r, H]
  int32_t* recv_ids[kMaxPeers];      // [R * T_r, K]
  float* recv_wts[kMaxPeers];        // [R * T_r, K]
  uint32_t* flags[kMaxPeers];
  int expert_start[kMaxPeers + 1];   // rank r owns experts [expert_start[r], expert_start[r + 1])
  uint32_t* masks;                   // [T_r], this rank's memory: destination ranks of each token
  int tokens, top_k, h8, ranks, rank;
  unsigned long long timeout_ns;
  int* error_flag;
};

// One block per token (grid-stride): its destination mask, the row to the destinations, the ids
// and weights to every rank; then the last block signals and waits for every rank's dispatch.
__global__ void __launch_bounds__(256) ep_dispatch_kernel(const DispatchArgs a) {
  __shared__ uint32_t s_mask;
  __shared__ uint32_t s_gen;
  __shared__ int s_last;
  uint32_t* mine = a.flags[a.rank];
  if (threadIdx.x == 0) s_gen = *reinterpret_cast<volatile uint32_t*>(mine + kGenSlot) + 1u;
  for (int t = blockIdx.x; t < a.tokens; t += gridDim.x) {
    if (threadIdx.x == 0) s_mask = 0;
    __syncthreads();
    if (threadIdx.x < a.top_k) {
      const int e = a.ids[(size_t)t * a.top_k + threadIdx.x];
      for (int r = 0; r < a.ranks; ++r)
        if (e >= a.expert_start[r] && e < a.expert_start[r + 1]) atomicOr(&s_mask, 1u << r);
    }
    __syncthreads();
    const uint32_t mask = s_mask;
    if (threadIdx.x == 0) a.masks[t] = mask;
    const size_t slot = (size_t)a.rank * a.tokens + t;
    const uint4* src = reinterpret_cast<const uint4*>(a.x + (size_t)t * a.h8 * 8);
    for (int r = 0; r < a.ranks; ++r) {
      if ((mask >> r) & 1u) {
        uint4* dst = reinterpret_cast<uint4*>(a.recv_x[r] + slot * a.h8 * 8);
        for (int i = threadIdx.x; i < a.h8; i += blockDim.x) dst[i] = __ldg(src + i);
      }
      if (threadIdx.x < a.top_k) {
        a.recv_ids[r][slot * a.top_k + threadIdx.x] = a.ids[(size_t)t * a.top_k + threadIdx.x];
        a.recv_wts[r][slot * a.top_k + threadIdx.x] = a.wts[(size_t)t * a.top_k + threadIdx.x];
      }
    }
  }
  __syncthreads();
  const uint32_t gen = s_gen;
  if (threadIdx.x == 0) {
    __threadfence_system();
    s_last = 0;
    if (atomicAdd(mine + kDispDone, 1u) == gridDim.x - 1) {
      mine[kDispDone] = 0;
      __threadfence();
      s_last = 1;
    }
  }
  __syncthreads();
  if (!s_last) return;
  if (threadIdx.x < a.ranks) {   // the last block: one thread per rank signals, in parallel
    __threadfence_system();
    st_release_sys(a.flags[threadIdx.x] + kDispatch + a.rank, gen);
  }
  if (threadIdx.x == 0 && !wait_slots(mine, kDispatch, a.ranks, gen, a.timeout_ns)) {
    atomicExch(mine + kFail, 1u);
    atomicExch(a.error_flag, 6);
  }
}

}  // namespace
}  // namespace muse

namespace muse {
namespace {

int launch_peer(const uint64_t* shares0, const uint64_t* shares1, const uint64_t* flags,
                const uint64_t* staging, int ranks, int rank, size_t n, int mode, int expect_parity,
                long long timeout_us, void* out, cudaStream_t stream, const uint32_t* masks = nullptr,
                int hidden = 0) {
  if (!shares0 || !shares1 || !flags || !out || ranks < 1 || ranks > kMaxPeers || rank < 0 ||
      rank >= ranks || n % 8 || expect_parity < -1 || expect_parity > 1 || timeout_us < 0)
    return MUSE_ERR_INVALID_ARGUMENT;
  if (mode == kAllReduce2 && !staging) return MUSE_ERR_INVALID_ARGUMENT;
  if (mode == kRoutedScatter && (!masks || hidden <= 0 || hidden % 8 || n % ((size_t)hidden * ranks)))
    return MUSE_ERR_INVALID_ARGUMENT;
  PeerArgs a{};
  for (int r = 0; r < ranks; ++r) {
    if (!shares0[r] || !shares1[r] || !flags[r] || shares0[r] % 16 || shares1[r] % 16 || flags[r] % 4)
      return MUSE_ERR_INVALID_ARGUMENT;
    a.share[0][r] = reinterpret_cast<const float*>(shares0[r]);
    a.share[1][r] = reinterpret_cast<const float*>(shares1[r]);
    a.flags[r] = reinterpret_cast<uint32_t*>(flags[r]);
    if (mode == kAllReduce2) {
      if (!staging[r] || staging[r] % 16) return MUSE_ERR_INVALID_ARGUMENT;
      a.staging[r] = reinterpret_cast<uint16_t*>(staging[r]);
    }
  }
  if (reinterpret_cast<uintptr_t>(out) % 16) return MUSE_ERR_INVALID_ARGUMENT;
  a.ranks = ranks;
  a.rank = rank;
  a.mode = mode;
  a.expect_parity = expect_parity;
  a.timeout_ns = timeout_us ? (unsigned long long)timeout_us * 1000ull : kDefaultTimeoutNs;
  a.n4 = n / 4;
  // a rank's slice: n / ranks rounded up to 8 elements (16-byte pieces of bf16)
  const size_t slice = mode == kAllReduce1 ? n : (n / ranks + 7) / 8 * 8;
  if ((mode == kReduceScatter || mode == kRoutedScatter) && slice * ranks != n) return MUSE_ERR_INVALID_ARGUMENT;
  a.masks = masks;
  a.h4 = hidden / 4;
  a.slice4 = slice / 4;
  a.out = static_cast<uint16_t*>(out);
  int rc = device_status_ptr(&a.error_flag);
  if (rc) return rc;
  // at least one block: an empty exchange (no tokens) still signals the peers and advances the
  // generation, so every rank's count -- and the share buffer its caller writes next -- stays in
  // step. The two-round all-reduce waits across its own blocks (step 4), so it is launched
  // cooperatively: all of its blocks are resident at once, or the launch fails.
  const size_t work4 = mode == kAllReduce1 ? a.n4 : a.slice4;
  size_t blocks = work4 == 0 ? 1 : (work4 + 255) / 256;
  if (blocks > 296) blocks = 296;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = mode == kAllReduce2 ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, peer_exchange_kernel, a);
  if (e != cudaSuccess) return e;
  return last_launch_status();
}

}  // namespace
}  // namespace muse

extern "C" int muse_moe_peer_exchange_bf16(const uint64_t* shares0, const uint64_t* shares1,
                                           const uint64_t* flags, const uint64_t* staging, int ranks,
                                           int rank, size_t n, int mode, int expect_parity,
                                           long long timeout_us, void* out, muse_stream_t stream) {
  if (mode < 0 || mode > 2) return MUSE_ERR_INVALID_ARGUMENT;
  return muse::launch_peer(shares0, shares1, flags, staging, ranks, rank, n, mode, expect_parity,
                           timeout_us, out, (cudaStream_t)stream);
}

extern "C" int muse_moe_peer_routed_reduce_scatter_bf16(const uint64_t* shares0, const uint64_t* shares1,
                                                        const uint64_t* flags, int ranks, int rank,
                                                        int tokens_per_rank, int hidden,
                                                        const uint32_t* masks, int expect_parity,
                                                        long long timeout_us, void* out,
                                                        muse_stream_t stream) {
  if (tokens_per_rank < 0) return MUSE_ERR_INVALID_ARGUMENT;
  return muse::launch_peer(shares0, shares1, flags, nullptr, ranks, rank,
                           (size_t)ranks * tokens_per_rank * hidden, muse::kRoutedScatter, expect_parity,
                           timeout_us, out, (cudaStream_t)stream, masks, hidden);
}

extern "C" int muse_moe_ep_dispatch(const void* x, const int32_t* topk_ids, const float* topk_weights,
                                    int tokens_per_rank, int top_k, int hidden, int ranks, int rank,
                                    const int* expert_start, const uint64_t* recv_x,
                                    const uint64_t* recv_ids, const uint64_t* recv_weights,
                                    const uint64_t* flags, uint32_t* masks, long long timeout_us,
                                    muse_stream_t stream) {
  using namespace muse;
  if (!expert_start || !recv_x || !recv_ids || !recv_weights || !flags || !masks || ranks < 1 ||
      ranks > kMaxPeers || rank < 0 || rank >= ranks || tokens_per_rank < 0 || top_k < 1 ||
      top_k > kMaxTopK || hidden <= 0 || hidden % 8 || timeout_us < 0)
    return MUSE_ERR_INVALID_ARGUMENT;
  if (tokens_per_rank > 0 && (!x || !topk_ids || !topk_weights || reinterpret_cast<uintptr_t>(x) % 16))
    return MUSE_ERR_INVALID_ARGUMENT;
  DispatchArgs a{};
  a.x = static_cast<const uint16_t*>(x);
  a.ids = topk_ids;
  a.wts = topk_weights;
  for (int r = 0; r < ranks; ++r) {
    if (!recv_x[r] || !recv_ids[r] || !recv_weights[r] || !flags[r] || recv_x[r] % 16 || recv_ids[r] % 4 ||
        recv_weights[r] % 4 || flags[r] % 4)
      return MUSE_ERR_INVALID_ARGUMENT;
    a.recv_x[r] = reinterpret_cast<uint16_t*>(recv_x[r]);
    a.recv_ids[r] = reinterpret_cast<int32_t*>(recv_ids[r]);
    a.recv_wts[r] = reinterpret_cast<float*>(recv_weights[r]);
    a.flags[r] = reinterpret_cast<uint32_t*>(flags[r]);
  }
  for (int r = 0; r <= ranks; ++r) {
    if (r > 0 && expert_start[r] < expert_start[r - 1]) return MUSE_ERR_INVALID_ARGUMENT;
    a.expert_start[r] = expert_start[r];
  }
  a.masks = masks;
  a.tokens = tokens_per_rank;
  a.top_k = top_k;
  a.h8 = hidden / 8;
  a.ranks = ranks;
  a.rank = rank;
  a.timeout_ns = timeout_us ? (unsigned long long)timeout_us * 1000ull : kDefaultTimeoutNs;
  int rc = device_status_ptr(&a.error_flag);
  if (rc) return rc;
  // one block per token up to 1184 blocks; at least one, so an empty batch still signals
  const int blocks = tokens_per_rank == 0 ? 1 : (tokens_per_rank < 1184 ? tokens_per_rank : 1184);
  ep_dispatch_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(a);
  return last_launch_status();
}

extern "C" int muse_moe_peer_allreduce_bf16(const uint64_t* shares0, const uint64_t* shares1,
                                            const uint64_t* flags, int ranks, int rank, size_t n,
                                            void* out, muse_stream_t stream) {
  return muse::launch_peer(shares0, shares1, flags, nullptr, ranks, rank, n, muse::kAllReduce1, -1, 0,
                           out, (cudaStream_t)stream);
}

extern "C" int muse_moe_peer_reduce_scatter_bf16(const uint64_t* shares0, const uint64_t* shares1,
                                                 const uint64_t* flags, int ranks, int rank,
                                                 size_t n_per_rank, void* out, muse_stream_t stream) {
  return muse::launch_peer(shares0, shares1, flags, nullptr, ranks, rank, n_per_rank * ranks,
                           muse::kReduceScatter, -1, 0, out, (cudaStream_t)stream);
}
