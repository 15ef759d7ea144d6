// muse_moe_forward_noalloc: the layer call for callers that cannot allocate device memory.
//
// Some callers have no way to hand the layer a workspace: code that runs inside another
// runtime's execution callback (an inference server's plugin or custom-op hook) where the
// host framework owns every device allocation and forbids new ones, or a latency-critical
// serving loop that must not call cudaMalloc / cudaFree because they can synchronise the
// device and stall every stream on it. This entry point takes the same inputs and output as
// muse_moe_forward but carves its scratch from a fixed array in device global memory that
// belongs to the library, so the call allocates nothing.
//
// Limits and sharing:
//   * the array holds kStaticScratchBytes (32 MiB); a call whose muse_moe_workspace_size is
//     larger is refused with MUSE_ERR_SCRATCH_LIMIT before anything is launched;
//   * a device holds the array from the first call on it until the process exits;
//   * every call on a device uses the same array, so calls that overlap on the GPU (two
//     streams, or two host threads) race on it and must be serialised by the caller;
//   * the array keeps whatever the last call left in it. No part of it has to start at zero:
//     every value the layer reads from its scratch was written earlier in the same call;
//   * every call looks the array's device address up on the current device (cheap once the
//     library's module is loaded), so a device reset or a re-created primary context, which
//     may move the array, is followed; a call made while its stream is being captured cannot
//     do the lookup and uses the address of the last call on that device -- make one call on
//     the device before capturing, and capture again after a device reset.
#include <mutex>

#include "common.cuh"

namespace muse {
namespace {

constexpr size_t kStaticScratchBytes = size_t(32) << 20;
constexpr int kMaxDevices = 64;

// The scratch itself. In host code this name is only a stand-in for the symbol: its device
// address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_addr[kMaxDevices] = {nullptr};

// Device address of g_static_scratch on the current device: looked up on every call, and
// remembered per device for calls made while `stream` is being captured.
int static_scratch(cudaStream_t stream, void** addr) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return MUSE_ERR_NO_DEVICE;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  e = cudaStreamIsCapturing(stream, &cap);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (cap == cudaStreamCaptureStatusNone) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return e;
    if (!p) return MUSE_ERR_NO_DEVICE;
    g_scratch_addr[dev] = p;
  } else if (!g_scratch_addr[dev]) {
    return MUSE_ERR_INVALID_ARGUMENT;   // first call on this device inside a capture
  }
  *addr = g_scratch_addr[dev];
  return MUSE_OK;
}

}  // namespace
}  // namespace muse

extern "C" int muse_moe_forward_noalloc(const void* x, const int32_t* topk_ids,
                                        const float* topk_weights, int tokens, int top_k,
                                        int local_start, int local_count, int hidden, int inter,
                                        const uint8_t* w13p, const uint8_t* w13_sfp,
                                        const float* w13_gs, const uint8_t* w2p,
                                        const uint8_t* w2_sfp, const float* w2_gs,
                                        const void* post_norm_w, void* out, muse_stream_t stream) {
  size_t need = 0;
  int rc = muse_moe_workspace_size(tokens, top_k, local_count, hidden, inter, &need);
  if (rc) return rc;
  if (need > muse::kStaticScratchBytes) return MUSE_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  if ((rc = muse::static_scratch((cudaStream_t)stream, &scratch))) return rc;
  return muse_moe_forward(x, topk_ids, topk_weights, tokens, top_k, local_start, local_count,
                          hidden, inter, w13p, w13_sfp, w13_gs, w2p, w2_sfp, w2_gs, post_norm_w,
                          out, scratch, muse::kStaticScratchBytes, stream);
}
