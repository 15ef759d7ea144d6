// Optional per-role timestamps of the expert GEMM (compiled in only with -DMUSE_TRACE).
//
// A traced build records clock64() stamps of each role's steps into a caller-attached device
// buffer: per CTA a block of kTraceStride u64 values. The default build compiles every
// MUSE_TRACE_* macro to nothing, so the product kernels carry no tracing code.
//
//   [0] globaltimer at kernel entry (thread 0), [1] clock64 at entry, [2] set-up done,
//   [3] every role done (before the tensor-memory release), [4] combine done,
//   set-up steps: [5] barriers initialised (last warp), [6] routing done, [7] scale table and
//   tile scan issued, [8] first set-up barrier passed (thread 0), [9] producer 0 starts
//   producer p, chunk c: [kTrW + p*kTrC + c] weight tile issued, [kTrB + ...] activation issued
//   dequant warp (lane quarter 0) of pipeline p: [kTrF + ...] weight tile landed,
//                                                [kTrA + ...] A buffer handed to the MMA
//   MMA issuer p: [kTrM + ...] chunk's MMAs issued
//   epilogue (lane quarter 0), item j: [kTrE + j] accumulators ready, [kTrE + kTrJ + j] stored
#pragma once

#include <stdint.h>

namespace muse {
namespace trace {

constexpr int kTrC = 128;  // chunks recorded per pipeline
constexpr int kTrJ = 64;   // items recorded per CTA
constexpr int kTrW = 16;
constexpr int kTrF = kTrW + 3 * kTrC;
constexpr int kTrA = kTrF + 3 * kTrC;
constexpr int kTrM = kTrA + 3 * kTrC;
constexpr int kTrB = kTrM + 3 * kTrC;
constexpr int kTrE = kTrB + 3 * kTrC;
constexpr int kTrWait = kTrE + 2 * kTrJ;   // per warp: wait-loop iterations (32), waits entered (32)
constexpr int kTraceStride = kTrWait + 64;

}  // namespace trace
}  // namespace muse

#ifdef MUSE_TRACE
namespace muse {
namespace trace {
// defined here: only the expert GEMM's translation unit includes this header
__device__ unsigned long long* g_trace_buf = nullptr;
// host side: the attached buffer, its launch blocks and the next block to use
inline unsigned long long* g_host_buf = nullptr;
inline int g_host_slots = 1, g_host_next = 0;
__device__ __forceinline__ void stamp(int slot) {
  if (g_trace_buf) g_trace_buf[(size_t)blockIdx.x * kTraceStride + slot] = clock64();
}
__device__ __forceinline__ void stamp_global_entry() {
  if (g_trace_buf) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    g_trace_buf[(size_t)blockIdx.x * kTraceStride + 0] = t;
    g_trace_buf[(size_t)blockIdx.x * kTraceStride + 1] = clock64();
  }
}
__device__ __forceinline__ void count_wait(int which) {
  if (g_trace_buf && (threadIdx.x & 31) == 0)
    atomicAdd(&g_trace_buf[(size_t)blockIdx.x * kTraceStride + kTrWait + 32 * which + (threadIdx.x >> 5)], 1ull);
}
}  // namespace trace
}  // namespace muse
#define MUSE_TRACE_WAIT_ITER() ::muse::trace::count_wait(0)
#define MUSE_TRACE_WAIT_ENTER() ::muse::trace::count_wait(1)
#define MUSE_TRACE_ENTRY() ::muse::trace::stamp_global_entry()
#define MUSE_TRACE_AT(slot) ::muse::trace::stamp(slot)
#define MUSE_TRACE_SEQ(base, p, c)                                              \
  do {                                                                          \
    if ((c) < ::muse::trace::kTrC) ::muse::trace::stamp((base) + (p) * ::muse::trace::kTrC + (c)); \
  } while (0)
#define MUSE_TRACE_ITEM(base, j)                                                \
  do {                                                                          \
    if ((j) < ::muse::trace::kTrJ) ::muse::trace::stamp((base) + (j));          \
  } while (0)
#else
#define MUSE_TRACE_WAIT_ITER() ((void)0)
#define MUSE_TRACE_WAIT_ENTER() ((void)0)
#define MUSE_TRACE_ENTRY() ((void)0)
#define MUSE_TRACE_AT(slot) ((void)0)
#define MUSE_TRACE_SEQ(base, p, c) ((void)0)
#define MUSE_TRACE_ITEM(base, j) ((void)0)
#endif
