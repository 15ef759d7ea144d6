// Flag protocol of the expert-parallel exchange, shared by the exchange kernels (peer.cu) and
// the single-launch layer kernel, which runs the one-round exchange after its combine
// (gemm_tc.cu). The protocol itself is described at the top of peer.cu.
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

#include "kernels.cuh"

namespace muse {

// Words of a rank's flag array (kFlagWords uint32, zero before the first call).
constexpr int kRound2 = 8;          // slots [8, 16): round-2 signals ([0, 8): round 1)
constexpr int kGenSlot = 16;        // calls completed
constexpr int kDoneA = 17;          // blocks past their part of the call's first stage
constexpr int kDoneB = 18;          // blocks finished in the current call
constexpr int kFail = 19;           // a wait of the current call expired
constexpr int kDispatch = 20;       // slots [20, 28): prefill dispatch signals
constexpr int kDispDone = 28;       // dispatch blocks finished in the current call
constexpr unsigned long long kDefaultTimeoutNs = 1000000000ull;  // 1 s

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait (one thread) until slots [base, base + ranks) of `mine` hold at least gen. Gives up after
// timeout_ns, or as soon as another block of this rank has recorded a failure.
__device__ __forceinline__ bool wait_slots(const uint32_t* mine, int base, int ranks, uint32_t gen,
                                           unsigned long long timeout_ns) {
  const unsigned long long t0 = global_ns();
  for (int r = 0; r < ranks; ++r) {
    unsigned ns = 32;
    while (ld_acquire_sys(mine + base + r) < gen) {
      if (global_ns() - t0 > timeout_ns) return false;
      if (*reinterpret_cast<const volatile uint32_t*>(mine + kFail)) return false;
      __nanosleep(ns);
      if (ns < 256) ns <<= 1;
    }
  }
  return true;
}

// bf16x4 of the sum over r = 0 .. ranks - 1, in that order from 0, of float4 group i4 of
// share[r] (read through to the owner's memory: the shares of other ranks are peer mappings).
__device__ __forceinline__ uint2 rank_sum_bf16x4(const float* const* share, int ranks, size_t i4) {
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int r = 0; r < ranks; ++r) {
    const float4 v = __ldcv(reinterpret_cast<const float4*>(share[r]) + i4);
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

// The one-round exchange run by every block of a cooperative grid after the grid has written
// this rank's share (ex.share[p][ex.rank], p = the call's parity): every block counts itself in
// once its share stores are visible on this GPU, and the last one signals round 1 to every
// rank, one thread per rank, each after a system-scope fence. Only as many blocks as the sum needs (one float4 group per
// thread) then wait (bounded) for all ranks' signals, sum their part of the elements into ex.out
// and count themselves out; the last of them advances the generation. The others return. The
// same sums as peer_exchange_kernel in mode 0, so the bits are the same as the layer launch
// followed by that kernel. s_gen, s_ok[2]: shared-memory words of the block.
// Not inlined: it runs once, at the end of the layer kernel, and kept out of line it leaves the
// register allocation of the kernel's loops alone.
static __device__ __noinline__ void grid_exchange_one_round(const ExchangeArgs& ex, int* error_flag,
                                                               uint32_t* s_gen, int* s_ok) {
  uint32_t* mine = ex.flags[ex.rank];
  const size_t want = (ex.n4 + blockDim.x - 1) / blockDim.x;
  const unsigned summers = want == 0 ? 1u : (want < gridDim.x ? (unsigned)want : gridDim.x);
  __syncthreads();  // this block's share stores are issued
  if (threadIdx.x == 0) {
    // read before this block counts itself in: the generation advances only after the summing
    // blocks have counted themselves out, which follows every block's count-in
    const uint32_t gen = *reinterpret_cast<volatile uint32_t*>(mine + kGenSlot) + 1u;
    *s_gen = gen;
    int ok = (int)(gen & 1u) == ex.expect_parity;
    if (!ok) {
      if (blockIdx.x == 0) atomicExch(error_flag, 7);   // the share went to the other buffer
    } else {
      __threadfence();
      if (atomicAdd(mine + kDoneA, 1u) == gridDim.x - 1) {   // the last block in signals
        mine[kDoneA] = 0;
        __threadfence();
        ok |= 4;
      }
    }
    s_ok[0] = ok;
  }
  __syncthreads();
  if ((s_ok[0] & 4) && threadIdx.x < ex.ranks) {
    // one thread per rank: the signals go out in parallel
    __threadfence_system();   // every block's share stores before the peers hear of them
    st_release_sys(ex.flags[threadIdx.x] + ex.rank, *s_gen);
  }
  if (threadIdx.x == 0) {
    int ok = s_ok[0] & 3;
    if (ok == 1) {
      if (blockIdx.x < summers) {
        ok = wait_slots(mine, 0, ex.ranks, *s_gen, ex.timeout_ns) ? 1 : 2;
        if (ok == 2) {
          atomicExch(mine + kFail, 1u);
          atomicExch(error_flag, 6);
        }
      } else {
        ok = 3;   // counted in; takes no part in the sum
      }
    }
    s_ok[1] = ok;   // 0: parity mismatch (nothing done), 1: sum, 2: a wait expired, 3: done
  }
  __syncthreads();
  const uint32_t gen = *s_gen;
  const int ok = s_ok[1];
  if (ok == 1) {
    const float* const* share = ex.share[gen & 1u];
    uint2* out = reinterpret_cast<uint2*>(ex.out);
    const size_t stride = (size_t)summers * blockDim.x;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < ex.n4; i += stride)
      out[i] = rank_sum_bf16x4(share, ex.ranks, i);
  }
  __syncthreads();
  if (threadIdx.x == 0 && (ok == 1 || ok == 2)) {
    __threadfence();
    if (atomicAdd(mine + kDoneB, 1u) == summers - 1) {
      mine[kDoneB] = 0;
      const bool failed = *reinterpret_cast<volatile uint32_t*>(mine + kFail) != 0;
      mine[kFail] = 0;
      __threadfence();
      if (!failed) *reinterpret_cast<volatile uint32_t*>(mine + kGenSlot) = gen;
    }
  }
}

}  // namespace muse
