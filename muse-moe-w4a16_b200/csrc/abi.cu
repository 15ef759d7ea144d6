// C ABI entry points (include/muse_moe.h): argument validation, workspace carving and the
// launch sequence of one layer call.
#include "common.cuh"
#include "kernels.cuh"

namespace muse {
namespace {

constexpr size_t kAlign = 256;

// Workspace layout for one call; every buffer 256-byte aligned.
struct WorkspaceLayout {
  size_t offsets, pair_order, pair_row, inter, ypart, ssq, total;
};

WorkspaceLayout workspace_layout(int tokens, int top_k, int local_count, int hidden, int inter) {
  const size_t P = (size_t)tokens * top_k;
  WorkspaceLayout l;
  size_t at = 0;
  auto take = [&](size_t bytes) {
    const size_t o = at;
    at = align_up(at + bytes, kAlign);
    return o;
  };
  l.offsets = take(sizeof(int32_t) * (local_count + 1));
  l.pair_order = take(sizeof(int32_t) * P);
  l.pair_row = take(sizeof(int32_t) * P);
  l.inter = take(2 * P * inter);
  l.ypart = take(4 * P * hidden);
  l.ssq = take(4 * P);
  l.total = at;
  return l;
}

int check_dims(int tokens, int top_k, int local_start, int local_count, int hidden, int inter) {
  if (tokens < 0 || top_k <= 0 || local_start < 0 || local_count <= 0 || hidden <= 0 || inter <= 0)
    return MUSE_ERR_INVALID_ARGUMENT;
  if (top_k > kMaxTopK || local_count > kMaxLocalExperts || hidden % 128 || inter % 128)
    return MUSE_ERR_UNSUPPORTED_SHAPE;
  return MUSE_OK;
}

}  // namespace
}  // namespace muse

using namespace muse;

extern "C" int muse_moe_version(void) { return (0 << 16) | 1; }

extern "C" const char* muse_moe_error_string(int code) {
  switch (code) {
    case MUSE_OK: return "success";
    case MUSE_ERR_INVALID_ARGUMENT: return "invalid argument (null pointer or bad size)";
    case MUSE_ERR_UNSUPPORTED_SHAPE:
      return "unsupported shape (hidden and inter must be multiples of 128, top_k <= 16, "
             "local_count <= 256)";
    case MUSE_ERR_WORKSPACE_TOO_SMALL: return "workspace smaller than muse_moe_workspace_size()";
    case MUSE_ERR_NO_DEVICE: return "no sm_100 CUDA device is current";
    case MUSE_ERR_DEVICE_TIMEOUT: return "a bounded device-side wait expired";
    default: break;
  }
  if (code > 0) return cudaGetErrorString((cudaError_t)code);
  return "unknown muse_moe error code";
}

extern "C" int muse_moe_workspace_size(int tokens, int top_k, int local_count, int hidden,
                                       int inter, size_t* bytes) {
  if (!bytes) return MUSE_ERR_INVALID_ARGUMENT;
  const int rc = check_dims(tokens, top_k, 0, local_count, hidden, inter);
  if (rc) return rc;
  *bytes = workspace_layout(tokens, top_k, local_count, hidden, inter).total;
  return MUSE_OK;
}

extern "C" int muse_moe_prepare_weights(const uint8_t* w13, const uint8_t* w13_sf,
                                        const uint8_t* w2, const uint8_t* w2_sf, int n_experts,
                                        int hidden, int inter, uint8_t* w13_out,
                                        uint8_t* w13_sf_out, uint8_t* w2_out, uint8_t* w2_sf_out,
                                        muse_stream_t stream) {
  if (n_experts <= 0 || hidden <= 0 || inter <= 0) return MUSE_ERR_INVALID_ARGUMENT;
  if (hidden % 128 || inter % 128) return MUSE_ERR_UNSUPPORTED_SHAPE;
  if (!w13 || !w13_sf || !w2 || !w2_sf || !w13_out || !w13_sf_out || !w2_out || !w2_sf_out)
    return MUSE_ERR_INVALID_ARGUMENT;
  const size_t E = n_experts, H = hidden, I = inter;
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e;
  if ((e = cudaMemcpyAsync(w13_out, w13, E * 2 * I * H / 2, cudaMemcpyDeviceToDevice, s))) return e;
  if ((e = cudaMemcpyAsync(w13_sf_out, w13_sf, E * 2 * I * H / 16, cudaMemcpyDeviceToDevice, s))) return e;
  if ((e = cudaMemcpyAsync(w2_out, w2, E * H * I / 2, cudaMemcpyDeviceToDevice, s))) return e;
  if ((e = cudaMemcpyAsync(w2_sf_out, w2_sf, E * H * I / 16, cudaMemcpyDeviceToDevice, s))) return e;
  return MUSE_OK;
}

extern "C" int muse_moe_forward(const void* x, const int32_t* topk_ids, const float* topk_weights,
                                int tokens, int top_k, int local_start, int local_count,
                                int hidden, int inter, const uint8_t* w13p,
                                const uint8_t* w13_sfp, const float* w13_gs, const uint8_t* w2p,
                                const uint8_t* w2_sfp, const float* w2_gs,
                                const void* post_norm_w, void* out, void* workspace,
                                size_t workspace_bytes, muse_stream_t stream) {
  int rc = check_dims(tokens, top_k, local_start, local_count, hidden, inter);
  if (rc) return rc;
  if (tokens == 0) return MUSE_OK;
  if (!x || !topk_ids || !topk_weights || !w13p || !w13_sfp || !w13_gs || !w2p || !w2_sfp ||
      !w2_gs || !post_norm_w || !out || !workspace)
    return MUSE_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(workspace) % kAlign) return MUSE_ERR_INVALID_ARGUMENT;
  const WorkspaceLayout l = workspace_layout(tokens, top_k, local_count, hidden, inter);
  if (workspace_bytes < l.total) return MUSE_ERR_WORKSPACE_TOO_SMALL;

  char* ws = static_cast<char*>(workspace);
  Scratch s;
  s.offsets = reinterpret_cast<int32_t*>(ws + l.offsets);
  s.pair_order = reinterpret_cast<int32_t*>(ws + l.pair_order);
  s.pair_row = reinterpret_cast<int32_t*>(ws + l.pair_row);
  s.inter = ws + l.inter;
  s.ypart = reinterpret_cast<float*>(ws + l.ypart);
  s.ssq = reinterpret_cast<float*>(ws + l.ssq);
  const LayerDims d{tokens, top_k, local_start, local_count, hidden, inter};
  const ExpertWeights w{w13p, w13_sfp, w13_gs, w2p, w2_sfp, w2_gs,
                        static_cast<const uint16_t*>(post_norm_w)};
  cudaStream_t st = (cudaStream_t)stream;

  cudaError_t ce = cudaMemsetAsync(s.ssq, 0, sizeof(float) * d.n_pairs(), st);
  if (ce != cudaSuccess) return ce;
  if ((rc = launch_route(topk_ids, tokens, top_k, local_start, local_count, s.offsets,
                         s.pair_order, s.pair_row, st)))
    return rc;
  if ((rc = launch_gemm1_silu(d, static_cast<const uint16_t*>(x), w, s, st))) return rc;
  if ((rc = launch_gemm2_norm(d, w, s, st))) return rc;
  return launch_combine(d, topk_ids, topk_weights, s, static_cast<uint16_t*>(out), st);
}
