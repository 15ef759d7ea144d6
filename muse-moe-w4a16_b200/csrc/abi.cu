// C ABI entry points (include/muse_moe.h): argument validation, workspace carving, tensor
// maps and the launch sequence of one layer call.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.cuh"
#include "layout.cuh"
#include "peer.cuh"

namespace muse {
namespace {

constexpr size_t kAlign = 256;

// Workspace layout for one call; every buffer 256-byte aligned. Order of the offsets is the
// order muse_moe_workspace_offsets reports them in.
struct WorkspaceLayout {
  size_t offsets, pair_order, pair_row, xs, inter, ypart, ssq, sync, total;
};

// Token-tile completion counters of a fused call: GEMM1 tiles, then GEMM2 tiles. A batch has
// at most one tile per pair plus one partial tile per expert.
size_t tile_capacity(int tokens, int top_k, int local_count) {
  return (size_t)tokens * top_k + local_count;
}

// Pair-row capacity of the row buffers: at least one full token tile (128 rows), so a TMA box
// never spans more rows than the tensor map describes.
size_t pair_rows(int tokens, int top_k) {
  const size_t p = (size_t)tokens * top_k;
  return p < 128 ? 128 : p;
}

WorkspaceLayout workspace_layout(int tokens, int top_k, int local_count, int hidden, int inter) {
  const size_t P = pair_rows(tokens, top_k);
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
  l.xs = take(2 * P * hidden);
  l.inter = take(2 * P * inter);
  l.ypart = take(4 * P * hidden);
  l.ssq = take(4 * P * (hidden / 32));
  l.sync = take(sizeof(int) * 2 * tile_capacity(tokens, top_k, local_count));
  l.total = at;
  return l;
}

int check_dims(int tokens, int top_k, int local_start, int local_count, int hidden, int inter) {
  if (tokens < 0 || top_k <= 0 || local_start < 0 || local_count <= 0 || hidden <= 0 || inter <= 0)
    return MUSE_ERR_INVALID_ARGUMENT;
  if (top_k > kMaxTopK || local_count > kMaxLocalExperts || hidden % 128 || inter % 128)
    return MUSE_ERR_UNSUPPORTED_SHAPE;
  if ((long long)tokens * top_k > (1LL << 30)) return MUSE_ERR_UNSUPPORTED_SHAPE;
  return MUSE_OK;
}

// Token tile (the MMA's N) from the expected pairs per local expert (twice the mean, so that
// most experts fit one tile); shapes only. The batch's T*K pairs spread over the model's
// n_experts experts, of which this call computes local_count, so a local expert expects
// T*K / n_experts of them -- on an expert-parallel slice (n_experts = R * local_count) R times
// fewer than T*K / local_count.
int pick_n_box(int tokens, int top_k, int n_experts) {
  const long long per_expert = 2LL * tokens * top_k / n_experts;
  int n = 16;
  while (n < 128 && n < per_expert) n <<= 1;
  return n;
}

// Pair-tile items (one dequantised weight chunk feeds two 128-token tiles): when the batch
// averages at least 128 pairs per local expert, i.e. most of its pairs sit in experts with two
// or more full tiles (prefill); shapes only.
bool use_pair_tiles(int tokens, int top_k, int n_experts) {
  return pick_n_box(tokens, top_k, n_experts) == 128 && (long long)tokens * top_k >= 128LL * n_experts;
}

// The single-launch (fused) path: decode batches of at most kMaxFusedPairs pairs with a small
// token tile. Above that the separate route / gather / GEMM1 / GEMM2 / combine launches are
// faster on B200 (measured at 256 pairs, E=128, H=2048, I=768: 116.7 vs 120.8 us).
constexpr int kMaxFusedPairs = 128;

// Launch plan of a call: 2 = the whole layer in one cooperative launch, 1 = GEMM1 routes in
// its prologue and gathers x itself (then GEMM2, combine), 0 = route, gather, GEMM1, GEMM2,
// combine.
int path_of(int tokens, int top_k, int n_experts) {
  const long long pairs = (long long)tokens * top_k;
  if (pick_n_box(tokens, top_k, n_experts) > kMaxInlineBox || pairs > kMaxInlinePairs) return 0;
  return pairs <= kMaxFusedPairs ? 2 : 1;
}

// Phases with more K chunks than this split each item over the pipelines; shorter ones give
// each item to one pipeline (unless the kernel finds fewer than 4 items per CTA). The single
// launch splits from 9 chunks on, the separate GEMM launches from 17 (measured on one B200,
// L2 flushed: 16 instead of 8 for the separate launches takes cfg4 T=32 / 256 from 917 / 1422
// to 909 / 1409 us -- GEMM2's 16-chunk items stay whole -- and leaves cfg2, cfg3 and cfg0
// unchanged; for the single launch it costs cfg2 T=16 2.5 %; 64 slows cfg0's 32-chunk items).
constexpr int kSplitKMinChunksFused = 8;
constexpr int kSplitKMinChunks = 16;

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

}  // namespace

int make_bf16_tmap(CUtensorMap* map, const void* base, int rows, int cols, int box_rows) {
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess) return e;
    if (q != cudaDriverEntryPointSuccess || !fn) return MUSE_ERR_NO_DEVICE;
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                              strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MUSE_OK : MUSE_ERR_INVALID_ARGUMENT;
}

}  // namespace muse

using namespace muse;

extern "C" int muse_moe_version(void) { return (0 << 16) | 2; }

extern "C" const char* muse_moe_error_string(int code) {
  switch (code) {
    case MUSE_OK: return "success";
    case MUSE_ERR_INVALID_ARGUMENT: return "invalid argument (null pointer or bad size)";
    case MUSE_ERR_UNSUPPORTED_SHAPE:
      return "unsupported shape (hidden and inter must be multiples of 128, top_k <= 16, "
             "local_count <= 256)";
    case MUSE_ERR_WORKSPACE_TOO_SMALL: return "workspace smaller than muse_moe_workspace_size()";
    case MUSE_ERR_NO_DEVICE: return "no sm_100 CUDA device / driver entry point available";
    case MUSE_ERR_DEVICE_TIMEOUT: return "a bounded device-side wait expired";
    case MUSE_ERR_SCRATCH_LIMIT:
      return "muse_moe_forward_noalloc: the call needs more scratch than its fixed 32 MiB array "
             "(use muse_moe_forward with a caller-supplied workspace)";
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

extern "C" int muse_moe_workspace_offsets(int tokens, int top_k, int local_count, int hidden,
                                          int inter, size_t* offsets) {
  if (!offsets) return MUSE_ERR_INVALID_ARGUMENT;
  const int rc = check_dims(tokens, top_k, 0, local_count, hidden, inter);
  if (rc) return rc;
  const WorkspaceLayout l = workspace_layout(tokens, top_k, local_count, hidden, inter);
  const size_t v[9] = {l.offsets, l.pair_order, l.pair_row, l.xs, l.inter, l.ypart, l.ssq, l.sync, l.total};
  for (int i = 0; i < 9; ++i) offsets[i] = v[i];
  return MUSE_OK;
}

extern "C" int muse_moe_device_status(int* status, int reset) {
  if (!status) return MUSE_ERR_INVALID_ARGUMENT;
  return read_device_status(status, reset);
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
  for (const void* p : {(const void*)w13, (const void*)w13_sf, (const void*)w2, (const void*)w2_sf,
                        (const void*)w13_out, (const void*)w13_sf_out, (const void*)w2_out,
                        (const void*)w2_sf_out})
    if (reinterpret_cast<uintptr_t>(p) % 16) return MUSE_ERR_INVALID_ARGUMENT;
  cudaStream_t s = (cudaStream_t)stream;
  int rc = launch_prepare_tiles(w13, w13_sf, n_experts, 2 * inter, hidden, inter, w13_out, w13_sf_out, s);
  if (rc) return rc;
  return launch_prepare_tiles(w2, w2_sf, n_experts, hidden, inter, 0, w2_out, w2_sf_out, s);
}

namespace {

// The launch sequence of one layer call. `ev` (optional) receives five event records on the
// stream: start, before GEMM1, after GEMM1, after GEMM2, after the combine. n_experts: the
// model's expert count (for the tile choice; local_count when unknown).
int forward_impl(const void* x, const int32_t* topk_ids, const float* topk_weights, int tokens,
                 int top_k, int local_start, int local_count, int hidden, int inter,
                 const uint8_t* w13p, const uint8_t* w13_sfp, const float* w13_gs,
                 const uint8_t* w2p, const uint8_t* w2_sfp, const float* w2_gs,
                 const void* post_norm_w, void* out, void* workspace, size_t workspace_bytes,
                 cudaStream_t st, cudaEvent_t* ev, bool f32_out = false, int n_experts = 0,
                 const ExchangeArgs* ex = nullptr) {
  int rc = check_dims(tokens, top_k, local_start, local_count, hidden, inter);
  if (rc) return rc;
  if (n_experts == 0) n_experts = local_count;
  if (n_experts < local_count) return MUSE_ERR_INVALID_ARGUMENT;
  if (tokens == 0) return MUSE_OK;
  if (!x || !topk_ids || !topk_weights || !w13p || !w13_sfp || !w13_gs || !w2p || !w2_sfp ||
      !w2_gs || !post_norm_w || !out || !workspace)
    return MUSE_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(workspace) % kAlign || reinterpret_cast<uintptr_t>(x) % 16 ||
      reinterpret_cast<uintptr_t>(w13p) % 16 || reinterpret_cast<uintptr_t>(w13_sfp) % 16 ||
      reinterpret_cast<uintptr_t>(w2p) % 16 || reinterpret_cast<uintptr_t>(w2_sfp) % 16 ||
      reinterpret_cast<uintptr_t>(out) % 16)
    return MUSE_ERR_INVALID_ARGUMENT;
  const WorkspaceLayout l = workspace_layout(tokens, top_k, local_count, hidden, inter);
  if (workspace_bytes < l.total) return MUSE_ERR_WORKSPACE_TOO_SMALL;

  char* ws = static_cast<char*>(workspace);
  Scratch s;
  s.offsets = reinterpret_cast<int32_t*>(ws + l.offsets);
  s.pair_order = reinterpret_cast<int32_t*>(ws + l.pair_order);
  s.pair_row = reinterpret_cast<int32_t*>(ws + l.pair_row);
  s.xs = reinterpret_cast<uint16_t*>(ws + l.xs);
  s.inter = reinterpret_cast<uint16_t*>(ws + l.inter);
  s.ypart = reinterpret_cast<float*>(ws + l.ypart);
  s.ssq = reinterpret_cast<float*>(ws + l.ssq);
  if ((rc = device_status_ptr(&s.error_flag))) return rc;
  const LayerDims d{tokens, top_k, local_start, local_count, hidden, inter};
  const int P = d.n_pairs();
  const int rows = (int)pair_rows(tokens, top_k);
  const int n_box = pick_n_box(tokens, top_k, n_experts);
  const int path = path_of(tokens, top_k, n_experts);
  const bool pair = path == 0 && use_pair_tiles(tokens, top_k, n_experts);
  int b_stages = 0;
  const int stages = pick_stages(n_box, pair, &b_stages);
  auto mark = [&](int i) -> int { return ev ? (int)cudaEventRecord(ev[i], st) : 0; };

  // Smallest batches: one cooperative launch does the whole layer -- routing in every CTA's
  // prologue, GEMM1 with x rows gathered straight from x, GEMM2 as soon as each token tile's
  // GEMM1 rows are in, and the combine. Decode batches up to kMaxInlinePairs: GEMM1 routes and
  // gathers x itself, then GEMM2 and the combine. Larger: all five kernels (pair-tile items
  // for prefill-sized batches).

  CUtensorMap tmap_xs, tmap_x, tmap_i;
  if ((rc = make_bf16_tmap(&tmap_xs, s.xs, rows, hidden, n_box))) return rc;
  if ((rc = make_bf16_tmap(&tmap_x, x, tokens, hidden, 1))) return rc;
  if ((rc = make_bf16_tmap(&tmap_i, s.inter, rows, inter, n_box))) return rc;

  GemmArgs g{};
  g.offsets = s.offsets;
  g.n_local = local_count;
  g.n_box = n_box;
  g.pair_tiles = pair;
  g.stages = stages;
  g.b_stages = b_stages;
  g.inter = s.inter;
  g.post_norm_w = static_cast<const uint16_t*>(post_norm_w);
  g.ypart = s.ypart;
  g.ssq = s.ssq;
  g.error_flag = s.error_flag;
  g.mul16 = 16;
  g.mul64 = 64;
  g.ids = topk_ids;
  g.n_pairs = P;
  g.local_start = local_start;
  g.top_k = top_k;
  g.pair_order = s.pair_order;
  g.pair_row = s.pair_row;
  PhaseArgs gemm1{};
  gemm1.m_tiles = 2 * inter / kTileM;
  gemm1.k_chunks = hidden / kChunkK;
  gemm1.wq = w13p;
  gemm1.wsf = w13_sfp;
  gemm1.gs = w13_gs;
  gemm1.mode = 1;
  gemm1.ld_out = inter;
  const int split_min = path == 2 ? kSplitKMinChunksFused : kSplitKMinChunks;
  gemm1.split_k = gemm1.k_chunks > split_min;
  PhaseArgs gemm2{};
  gemm2.m_tiles = hidden / kTileM;
  gemm2.k_chunks = inter / kChunkK;
  gemm2.wq = w2p;
  gemm2.wsf = w2_sfp;
  gemm2.gs = w2_gs;
  gemm2.mode = 2;
  gemm2.ld_out = hidden;
  gemm2.split_k = gemm2.k_chunks > split_min;

  if ((rc = mark(0))) return rc;
  if (path == 2) {
    int* counters = reinterpret_cast<int*>(ws + l.sync);
    const size_t cap = tile_capacity(tokens, top_k, local_count);
    cudaError_t ce = cudaMemsetAsync(counters, 0, sizeof(int) * 2 * cap, st);
    if (ce != cudaSuccess) return ce;
    gemm1.b_source = 1;
    gemm1.signal = counters;
    gemm2.b_source = 2;
    gemm2.signal = counters + cap;
    gemm2.wait_for = counters;
    gemm2.wait_target = 4 * gemm1.m_tiles;  // 4 epilogue warps per GEMM1 item
    g.n_phases = 2;
    g.ph[0] = gemm1;
    g.ph[1] = gemm2;
    g.route_inline = 1;
    g.fused = 1;
    g.tokens = tokens;
    g.hidden = hidden;
    g.topk_weights = topk_weights;
    g.out = out;
    g.out_f32 = f32_out;
    if (ex) g.ex = *ex;
    if ((rc = mark(1))) return rc;
    if ((rc = launch_expert_gemm(tmap_xs, tmap_x, tmap_i, g, st))) return rc;
    if ((rc = mark(2))) return rc;
    if ((rc = mark(3))) return rc;
    return mark(4);
  }

  if (path == 1) {
    g.route_inline = 1;
    gemm1.b_source = 1;  // four-row gathers of x
  } else {
    // large batches: the multi-CTA routing, its per-CTA counts in the head of ypart (written only
    // later, by GEMM2)
    if ((rc = launch_route_multi(topk_ids, tokens, top_k, local_start, local_count, s.offsets,
                                 s.pair_order, s.pair_row, reinterpret_cast<int32_t*>(s.ypart), st)))
      return rc;
    if ((rc = launch_gather(static_cast<const uint16_t*>(x), s.offsets, s.pair_order, local_count,
                            top_k, P, hidden, s.xs, st)))
      return rc;
  }
  g.n_phases = 1;
  g.ph[0] = gemm1;  // b_source 0: the gathered rows xs
  if ((rc = mark(1))) return rc;
  if ((rc = launch_expert_gemm(tmap_xs, tmap_x, tmap_xs, g, st))) return rc;
  if ((rc = mark(2))) return rc;
  g.ph[0] = gemm2;  // b_source 0: the inter rows
  g.route_inline = 0;
  if ((rc = launch_expert_gemm(tmap_i, tmap_x, tmap_i, g, st))) return rc;
  if ((rc = mark(3))) return rc;
  if ((rc = launch_combine(d, topk_ids, topk_weights, s, out, f32_out, st))) return rc;
  return mark(4);
}

}  // namespace

extern "C" int muse_moe_forward(const void* x, const int32_t* topk_ids, const float* topk_weights,
                                int tokens, int top_k, int local_start, int local_count,
                                int hidden, int inter, const uint8_t* w13p,
                                const uint8_t* w13_sfp, const float* w13_gs, const uint8_t* w2p,
                                const uint8_t* w2_sfp, const float* w2_gs,
                                const void* post_norm_w, void* out, void* workspace,
                                size_t workspace_bytes, muse_stream_t stream) {
  return forward_impl(x, topk_ids, topk_weights, tokens, top_k, local_start, local_count, hidden,
                      inter, w13p, w13_sfp, w13_gs, w2p, w2_sfp, w2_gs, post_norm_w, out, workspace,
                      workspace_bytes, (cudaStream_t)stream, nullptr);
}

extern "C" int muse_moe_forward_profiled(const void* x, const int32_t* topk_ids,
                                         const float* topk_weights, int tokens, int top_k,
                                         int local_start, int local_count, int hidden, int inter,
                                         const uint8_t* w13p, const uint8_t* w13_sfp,
                                         const float* w13_gs, const uint8_t* w2p,
                                         const uint8_t* w2_sfp, const float* w2_gs,
                                         const void* post_norm_w, void* out, void* workspace,
                                         size_t workspace_bytes, muse_stream_t stream,
                                         void* const* stage_events) {
  if (!stage_events) return MUSE_ERR_INVALID_ARGUMENT;
  cudaEvent_t ev[5];
  for (int i = 0; i < 5; ++i) {
    if (!stage_events[i]) return MUSE_ERR_INVALID_ARGUMENT;
    ev[i] = static_cast<cudaEvent_t>(stage_events[i]);
  }
  return forward_impl(x, topk_ids, topk_weights, tokens, top_k, local_start, local_count, hidden,
                      inter, w13p, w13_sfp, w13_gs, w2p, w2_sfp, w2_gs, post_norm_w, out, workspace,
                      workspace_bytes, (cudaStream_t)stream, ev);
}

extern "C" int muse_moe_forward_partial(const void* x, const int32_t* topk_ids,
                                        const float* topk_weights, int tokens, int top_k,
                                        int local_start, int local_count, int hidden, int inter,
                                        const uint8_t* w13p, const uint8_t* w13_sfp,
                                        const float* w13_gs, const uint8_t* w2p,
                                        const uint8_t* w2_sfp, const float* w2_gs,
                                        const void* post_norm_w, float* out_f32, void* workspace,
                                        size_t workspace_bytes, muse_stream_t stream) {
  return forward_impl(x, topk_ids, topk_weights, tokens, top_k, local_start, local_count, hidden,
                      inter, w13p, w13_sfp, w13_gs, w2p, w2_sfp, w2_gs, post_norm_w, out_f32,
                      workspace, workspace_bytes, (cudaStream_t)stream, nullptr, true);
}

// Ranks up to which the decode exchange runs inside the layer's single launch. Measured with
// CUDA graphs at cfg4 T=1 (max over ranks): 2 ranks 78 us inside against 83 us as a second
// launch; 4 ranks 65.6 against 62.1 (the exchange kernel's 7 blocks start as soon as the layer
// launch ends, while in the fused tail every block of the grid counts in before the peers are
// signalled, and a few blocks make all the peer reads).
constexpr int kMaxFusedExchangeRanks = 2;

extern "C" int muse_moe_forward_exchange_bf16(
    const void* x, const int32_t* topk_ids, const float* topk_weights, int tokens, int top_k,
    int local_start, int local_count, int n_experts, int hidden, int inter, const uint8_t* w13p,
    const uint8_t* w13_sfp, const float* w13_gs, const uint8_t* w2p, const uint8_t* w2_sfp,
    const float* w2_gs, const void* post_norm_w, void* workspace, size_t workspace_bytes,
    const uint64_t* shares0, const uint64_t* shares1, const uint64_t* flags, const uint64_t* staging,
    int ranks, int rank, int mode, int expect_parity, long long timeout_us, void* out,
    muse_stream_t stream) {
  if (!shares0 || !shares1 || !flags || !out || ranks < 1 || ranks > kMaxPeers || rank < 0 ||
      rank >= ranks || (mode != 0 && mode != 2) || (expect_parity != 0 && expect_parity != 1) ||
      timeout_us < 0 || tokens < 0 || hidden <= 0 || reinterpret_cast<uintptr_t>(out) % 16)
    return MUSE_ERR_INVALID_ARGUMENT;
  ExchangeArgs ex{};
  for (int r = 0; r < ranks; ++r) {
    if (!shares0[r] || !shares1[r] || !flags[r] || shares0[r] % 16 || shares1[r] % 16 || flags[r] % 4)
      return MUSE_ERR_INVALID_ARGUMENT;
    ex.share[0][r] = reinterpret_cast<const float*>(shares0[r]);
    ex.share[1][r] = reinterpret_cast<const float*>(shares1[r]);
    ex.flags[r] = reinterpret_cast<uint32_t*>(flags[r]);
  }
  float* share = const_cast<float*>(ex.share[expect_parity][rank]);
  const size_t n = (size_t)tokens * hidden;
  const int n_eff = n_experts == 0 ? local_count : n_experts;
  // One launch when the layer is the single cooperative launch, the one-round sum is asked for
  // and at most kMaxFusedExchangeRanks ranks take part: the exchange follows the combine inside
  // it. Otherwise the layer, then the exchange kernel.
  const bool fused = mode == 0 && ranks <= kMaxFusedExchangeRanks && tokens > 0 && local_count > 0 &&
                     n_eff >= local_count &&
                     check_dims(tokens, top_k, local_start, local_count, hidden, inter) == MUSE_OK &&
                     path_of(tokens, top_k, n_eff) == 2;
  if (fused) {
    ex.out = static_cast<uint16_t*>(out);
    ex.n4 = n / 4;
    ex.timeout_ns = timeout_us ? (unsigned long long)timeout_us * 1000ull : kDefaultTimeoutNs;
    ex.ranks = ranks;
    ex.rank = rank;
    ex.expect_parity = expect_parity;
    return forward_impl(x, topk_ids, topk_weights, tokens, top_k, local_start, local_count, hidden,
                        inter, w13p, w13_sfp, w13_gs, w2p, w2_sfp, w2_gs, post_norm_w, share, workspace,
                        workspace_bytes, (cudaStream_t)stream, nullptr, true, n_experts, &ex);
  }
  const int rc = forward_impl(x, topk_ids, topk_weights, tokens, top_k, local_start, local_count,
                              hidden, inter, w13p, w13_sfp, w13_gs, w2p, w2_sfp, w2_gs, post_norm_w,
                              share, workspace, workspace_bytes, (cudaStream_t)stream, nullptr, true,
                              n_experts);
  if (rc) return rc;
  return muse_moe_peer_exchange_bf16(shares0, shares1, flags, staging, ranks, rank, n, mode,
                                     expect_parity, timeout_us, out, stream);
}

extern "C" int muse_moe_cast_bf16(const float* in, void* out, size_t n, muse_stream_t stream) {
  if (n == 0) return MUSE_OK;
  if (!in || !out || n % 8 || reinterpret_cast<uintptr_t>(in) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
    return MUSE_ERR_INVALID_ARGUMENT;
  return launch_cast_bf16(in, static_cast<uint16_t*>(out), n, (cudaStream_t)stream);
}

extern "C" int muse_moe_launch_plan_ex(int tokens, int top_k, int local_count, int n_experts, int hidden,
                                       int inter, int* plan) {
  if (!plan) return MUSE_ERR_INVALID_ARGUMENT;
  const int rc = check_dims(tokens, top_k, 0, local_count, hidden, inter);
  if (rc) return rc;
  if (n_experts == 0) n_experts = local_count;
  if (n_experts < local_count) return MUSE_ERR_INVALID_ARGUMENT;
  const int n_box = pick_n_box(tokens, top_k, n_experts);
  const int path = path_of(tokens, top_k, n_experts);
  const bool pair = path == 0 && use_pair_tiles(tokens, top_k, n_experts);
  plan[0] = tokens == 0 ? 0 : (path == 2 ? 1 : path == 1 ? 3 : 5);
  plan[1] = n_box;
  int b_stages = 0;
  plan[2] = pick_stages(n_box, pair, &b_stages);
  plan[3] = path;
  plan[4] = pair;
  return MUSE_OK;
}

extern "C" int muse_moe_launch_plan(int tokens, int top_k, int local_count, int hidden, int inter,
                                    int* plan) {
  return muse_moe_launch_plan_ex(tokens, top_k, local_count, local_count, hidden, inter, plan);
}

extern "C" int muse_moe_forward_ex(const void* x, const int32_t* topk_ids, const float* topk_weights,
                                   int tokens, int top_k, int local_start, int local_count,
                                   int n_experts, int hidden, int inter, const uint8_t* w13p,
                                   const uint8_t* w13_sfp, const float* w13_gs, const uint8_t* w2p,
                                   const uint8_t* w2_sfp, const float* w2_gs,
                                   const void* post_norm_w, void* out, int out_f32, void* workspace,
                                   size_t workspace_bytes, muse_stream_t stream,
                                   void* const* stage_events) {
  cudaEvent_t ev[5];
  if (stage_events) {
    for (int i = 0; i < 5; ++i) {
      if (!stage_events[i]) return MUSE_ERR_INVALID_ARGUMENT;
      ev[i] = static_cast<cudaEvent_t>(stage_events[i]);
    }
  }
  return forward_impl(x, topk_ids, topk_weights, tokens, top_k, local_start, local_count, hidden,
                      inter, w13p, w13_sfp, w13_gs, w2p, w2_sfp, w2_gs, post_norm_w, out, workspace,
                      workspace_bytes, (cudaStream_t)stream, stage_events ? ev : nullptr, out_f32 != 0,
                      n_experts);
}
