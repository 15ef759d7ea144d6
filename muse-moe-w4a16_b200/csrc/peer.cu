// Expert-parallel exchange over NVLink peer memory: the sum of every rank's fp32 share of the
// layer output, cast to bf16 -- on every rank for all elements (the all-reduce of the decode
// layout), or on each rank for its own slice of the elements (the reduce-scatter of the
// prefill layout) -- done by this kernel instead of a collective library.
//
// Each rank's share lives in its own symmetric buffer; the buffers of all ranks are mapped
// into every rank's address space (peer pointers). Every rank keeps, in its own flag array,
// 8 peer slots, its generation counter (slot 8: calls completed) and a finished-block count
// (slot 9). A call with generation g = counter + 1 (the same on every rank):
//   1. block 0 publishes "my share of call g is complete" by writing g into slot `rank` of
//      every rank's flag array (system-scope release after a system fence, so the share's
//      bytes -- written by the previous kernel on this stream -- are visible first);
//   2. every block waits (acquire, bounded) until all R peer slots of its own array hold g;
//   3. out[i] = bf16(sum over r = 0 .. R-1 of share_r[offset + i]) from the share buffers of
//      parity g & 1, in the same order on every rank, so all ranks produce identical bits;
//   4. the last block to finish stores g as the new counter.
// The generation lives on the device, so a captured graph of the call stays valid across
// replays. Callers write call g's share into buffer g & 1: a rank rewrites a buffer only two
// calls later, after every peer has signalled the call in between (which it does only after
// finishing its reads of this rank's older share).
#include "common.cuh"
#include "kernels.cuh"
#include "ptx.cuh"

namespace muse {
namespace {

constexpr int kMaxPeers = 8;
constexpr int kGenSlot = 8, kDoneSlot = 9;

struct PeerArgs {
  const float* share[2][kMaxPeers];  // share buffers of parity 0 / 1 of rank r (peer pointers)
  uint32_t* flags[kMaxPeers];        // flag array of rank r
  int ranks, rank;
  size_t n4;                         // elements / 4
  size_t offset4;                    // first element / 4 (0, or this rank's slice)
  uint16_t* out;                     // bf16 [n], this rank's memory
  int* error_flag;
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__global__ void __launch_bounds__(256) peer_allreduce_kernel(const PeerArgs a) {
  __shared__ int s_ok;
  __shared__ uint32_t s_gen;
  uint32_t* mine = a.flags[a.rank];
  if (threadIdx.x == 0) s_gen = *reinterpret_cast<volatile uint32_t*>(mine + kGenSlot) + 1u;
  __syncthreads();
  const uint32_t gen = s_gen;
  if (blockIdx.x == 0 && threadIdx.x < a.ranks) {
    __threadfence_system();
    st_release_sys(a.flags[threadIdx.x] + a.rank, gen);
  }
  if (threadIdx.x == 0) {
    bool ok = true;
    const long long t0 = clock64();
    for (int r = 0; r < a.ranks && ok; ++r) {
      unsigned ns = 32;
      while (ld_acquire_sys(mine + r) < gen) {
        if (clock64() - t0 > ptx::kWaitCycles) {
          ok = false;
          break;
        }
        __nanosleep(ns);
        if (ns < 256) ns <<= 1;
      }
    }
    if (!ok) atomicExch(a.error_flag, 6);
    s_ok = ok;
  }
  __syncthreads();
  if (s_ok) {  // else a peer never signalled: the output is left alone, the status says why
    const int par = gen & 1u;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < a.n4; i += (size_t)gridDim.x * blockDim.x) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int r = 0; r < a.ranks; ++r) {
        const float4 v = __ldcv(reinterpret_cast<const float4*>(a.share[par][r]) + a.offset4 + i);
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
      reinterpret_cast<uint2*>(a.out)[i] = packed;
    }
  }
  // the last block out advances the generation (every block has read it by now)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(mine + kDoneSlot, 1u) == gridDim.x - 1) {
      mine[kDoneSlot] = 0;
      __threadfence();
      *reinterpret_cast<volatile uint32_t*>(mine + kGenSlot) = gen;
    }
  }
}

}  // namespace
}  // namespace muse

namespace muse {
namespace {

int launch_peer_sum(const uint64_t* shares0, const uint64_t* shares1, const uint64_t* flags, int ranks,
                    int rank, size_t offset, size_t n, void* out, cudaStream_t stream) {
  if (!shares0 || !shares1 || !flags || !out || ranks < 1 || ranks > kMaxPeers || rank < 0 ||
      rank >= ranks || n % 8 || offset % 8)
    return MUSE_ERR_INVALID_ARGUMENT;
  PeerArgs a{};
  for (int r = 0; r < ranks; ++r) {
    if (!shares0[r] || !shares1[r] || !flags[r] || shares0[r] % 16 || shares1[r] % 16 || flags[r] % 4)
      return MUSE_ERR_INVALID_ARGUMENT;
    a.share[0][r] = reinterpret_cast<const float*>(shares0[r]);
    a.share[1][r] = reinterpret_cast<const float*>(shares1[r]);
    a.flags[r] = reinterpret_cast<uint32_t*>(flags[r]);
  }
  if (reinterpret_cast<uintptr_t>(out) % 16) return MUSE_ERR_INVALID_ARGUMENT;
  a.ranks = ranks;
  a.rank = rank;
  a.n4 = n / 4;
  a.offset4 = offset / 4;
  a.out = static_cast<uint16_t*>(out);
  int rc = device_status_ptr(&a.error_flag);
  if (rc) return rc;
  // at least one block: an empty exchange (no tokens) still signals the peers and advances the
  // generation, so every rank's count -- and the share buffer its caller writes next -- stays in step
  const size_t blocks = a.n4 == 0 ? 1 : (a.n4 + 255) / 256;
  peer_allreduce_kernel<<<blocks < 296 ? (unsigned)blocks : 296u, 256, 0, stream>>>(a);
  return last_launch_status();
}

}  // namespace
}  // namespace muse

extern "C" int muse_moe_peer_allreduce_bf16(const uint64_t* shares0, const uint64_t* shares1,
                                            const uint64_t* flags, int ranks, int rank, size_t n,
                                            void* out, muse_stream_t stream) {
  return muse::launch_peer_sum(shares0, shares1, flags, ranks, rank, 0, n, out, (cudaStream_t)stream);
}

extern "C" int muse_moe_peer_reduce_scatter_bf16(const uint64_t* shares0, const uint64_t* shares1,
                                                 const uint64_t* flags, int ranks, int rank,
                                                 size_t n_per_rank, void* out, muse_stream_t stream) {
  return muse::launch_peer_sum(shares0, shares1, flags, ranks, rank, (size_t)rank * n_per_rank, n_per_rank,
                               out, (cudaStream_t)stream);
}
