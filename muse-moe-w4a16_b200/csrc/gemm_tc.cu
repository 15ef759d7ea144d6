// Expert GEMMs on the 5th-generation tensor cores (tcgen05, sm_100a), swap-AB:
// the weight rows are the MMA's M = 128 side, the tokens of one expert its N side.
//
//   GEMM1 (mode 1): h = xs . W13^T over K = H, epilogue silu(gate) * up -> inter (bf16)
//                   (reference.py:103-104; SGLang keeps inter in bf16, baseline.py:132)
//   GEMM2 (mode 2): y = inter . W2^T over K = I, epilogue y * gs * (1 + post_norm_w) -> ypart
//                   (fp32) and, per pair, the sum of squares of each 32-row slice -> ssq
//                   (reference.py:88-90, 105); every value is written exactly once, in a fixed
//                   order, so the layer's output is bit-reproducible
//
// One persistent CTA per SM walks a static list of (expert, 128-row tile, token tile) items.
// A tcgen05.mma costs its issuing thread ~44 cycles however small N is (measured on B200), so
// a CTA runs P independent pipelines (P = 3 for the 16-token decode tile, else 2) that split
// the K chunks of each tile between them (split-K, one partial accumulator per pipeline,
// summed by the epilogue). Warp roles:
//
//   warps [0, P)        producers: 1-D bulk copies of the prepared fp4 code and scale tiles,
//                       2-D TMA boxes of the activations (128-byte swizzle)
//   warps [P, 2P)       MMA issuers: tcgen05.mma, A in tensor memory, B in shared memory,
//                       fp32 accumulators in tensor memory; warp P also owns the allocation
//   warps [2P, 2P+4)    epilogue for all pipelines (items in list order): tcgen05.ld, fused
//                       activation / post-norm, stores
//   4 warps per pipeline dequantisers. Thread = weight row: e2m1 x e4m3 -> exact bf16 in
//                       registers, tcgen05.st into an A buffer
//
// Tensor memory: pipeline p owns a column range of 512/P (rounded to 32): n_a A buffers of
// 64 columns (128 K elements as bf16 pairs) followed by n_acc accumulators of n_box columns.
// Every mbarrier wait is bounded; on timeout the CTA records an error flag and unwinds.
#include "common.cuh"
#include "combine.cuh"
#include "kernels.cuh"
#include "layout.cuh"
#include "peer.cuh"
#include "ptx.cuh"
#include "route.cuh"
#include "trace.cuh"

namespace muse {

namespace {

constexpr int kMaxPipes = 3;
// The 16-token (decode) tile's layout: pipelines x dequant warps per pipeline. Measured on
// B200 (cfg2 / cfg4 decode sweeps): 3 x 4 beats 2 x 8 (two warps per lane quarter) by 2-10 %.
constexpr int kDecodePipes = 3;
constexpr int kDecodeDW = 4;
constexpr int kACols = kChunkK / 2;   // TMEM columns per A buffer (bf16 pairs)
constexpr int kTmemCols = 512;

// P pipelines, DW dequant warps per pipeline (4: one per TMEM lane quarter, each converting a
// whole 128-element row slice of a chunk; 8: two per quarter, each converting one half).
template <int P, int DW> struct Roles {
  static_assert(DW == 4 || DW == 8, "dequant warps per pipeline");
  static constexpr int kMmaWarp0 = P;
  static constexpr int kEpiWarp0 = 2 * P;
  static constexpr int kDeqWarp0 = 2 * P + 4;  // a multiple of 4 for P = 2: warp % 4 = quarter
  static constexpr int kWarps = 2 * P + 4 + DW * P;
  static constexpr int kThreads = 32 * kWarps;
  static constexpr int kPipeCols = (kTmemCols / P) / 32 * 32;
};
constexpr int kMaxStages = 8;
constexpr int kMaxABuf = 3;
constexpr int kMaxExperts = kMaxLocalExperts;
// raw code value = e2m1 * 2^-126; scales held as sf * 2^60; product = e2m1 * sf * 2^-66.
constexpr float kUnscale = 73786976294838206464.0f;  // 2^66

// Two rings per pipeline: weight tiles (freed by the dequantisers as soon as they have read
// them) and activation boxes (freed when the MMAs that read them complete), so a weight slot
// is refilled without waiting for the tensor core.
struct PipeCtl {
  uint64_t w_full[kMaxStages];
  uint64_t w_empty[kMaxStages];
  uint64_t b_full[kMaxStages];
  uint64_t b_empty[kMaxStages];
  uint64_t a_full[kMaxABuf];
  uint64_t a_empty[kMaxABuf];
  uint64_t acc_full[3];
  uint64_t acc_empty[3];
  uint64_t drain;
};

struct SharedCtl {
  PipeCtl pipe[kMaxPipes];
  uint32_t tmem_base;
  int tile_warp_sum[8];              // token tiles of experts [32w, 32w + 32)
  int tile_prefix[kMaxExperts + 1];  // cumulative item columns per expert (token tiles, or pairs of them)
  int ntiles[kMaxExperts];           // token tiles per expert
  uint32_t scale_lut[256];           // e4m3 byte -> bf16x2 (sf * 2^60, sf * 2^60)
  int offs[kMaxExperts + 1];         // route_inline: expert ranges of the pair rows
  int order[kMaxInlinePairs];        // route_inline: token of each expert-grouped pair row
  uint8_t slot_of_row[kMaxInlinePairs];  // route_inline: top-k slot of each pair row
  int c_row[kMaxTopK], c_key[kMaxTopK], c_order[kMaxTopK], c_srow[kMaxTopK], c_n;  // combine of one token
  float c_coef[kMaxTopK], c_scoef[kMaxTopK];
  ExchangeArgs ex;                   // the decode exchange after the combine: its arguments,
  uint32_t ex_gen;                   // its generation
  int ex_ok[2];                      // and this block's go / no-go (count-in, then sum)
};

// Per-launch geometry shared by all roles.
struct Geo {
  int Sw, Sb;         // weight / activation ring depths per pipeline
  int n_box;          // token tile = MMA N
  int n_a, n_acc;     // A buffers and accumulators per pipeline
  uint32_t b_bytes;   // one activation slot: two 64-column boxes of n_box rows per token tile
  uint32_t pipe_bytes;
};
// Items of the pair-tile variant cover up to two token tiles of one expert: every dequantised
// A chunk feeds two MMAs (one per tile), so the in-register conversion is done once per 2 x
// n_box tokens. One pipeline, three accumulator slots of n_box columns (an item takes one or
// two of them, so the epilogue of one tile overlaps the next item's MMAs), two A buffers.
constexpr int kPairAccSlots = 3;
constexpr uint32_t kWStageBytes = kTileCodeBytes + kTileScaleBytes;  // 9 KiB, 1 KiB multiple

__host__ __device__ inline Geo make_geo(int pipe_cols, int n_box, int w_stages, int b_stages, bool pair) {
  Geo g;
  g.Sw = w_stages;
  g.Sb = b_stages;
  g.n_box = n_box;
  g.n_acc = pair ? kPairAccSlots : (2 * n_box <= pipe_cols / 2 ? 2 : 1);
  g.n_a = (pipe_cols - g.n_acc * n_box) / kACols;
  if (g.n_a > kMaxABuf) g.n_a = kMaxABuf;
  g.b_bytes = (pair ? 4u : 2u) * n_box * 128u;
  g.pipe_bytes = w_stages * kWStageBytes + b_stages * g.b_bytes;
  return g;
}

// One work item: phase (GEMM), expert, 128-row weight tile m, token tile n (rows row0 ..
// row0 + nvalid of the expert-grouped pairs), and the token tile's index over all experts; in
// the pair-tile variant nt = 2 when the item also covers tile n + 1 (nvalid1 rows from
// row0 + n_box), else 1.
struct Item {
  int ph, e, m, n, row0, nvalid, tile, nt, nvalid1;
};

// Position in a ring of `size` slots: slot index and the parity of the slot's current use.
// Advanced incrementally, so the hot loops do no division.
struct Ring {
  int slot = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void next(int size) {
    if (++slot == size) { slot = 0; phase ^= 1u; }
  }
};

// Items are numbered phase by phase: phase 0 has cols x ph[0].m_tiles items (n0), then phase
// 1. Inside a phase, expert e owns items [tile_prefix[e] * m_tiles, tile_prefix[e + 1] * m_tiles),
// m-tile major: item column c of weight tile m is token tile c (or tiles 2c, 2c + 1 with kPair).
template <bool kPair = false>
__device__ __forceinline__ Item decode_item(const SharedCtl& c, const int32_t* offsets, int it, int n0,
                                            int n_local, int n_box, int mt0, int mt1) {
  Item r;
  r.ph = it >= n0;
  if (r.ph) it -= n0;
  const int mt = r.ph ? mt1 : mt0;
  int lo = 0, hi = n_local;  // largest e with tile_prefix[e] * mt <= it (a non-empty expert)
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (c.tile_prefix[mid] * mt <= it) lo = mid; else hi = mid;
  }
  r.e = lo;
  const int local = it - c.tile_prefix[lo] * mt;
  const int cols = c.tile_prefix[lo + 1] - c.tile_prefix[lo];
  r.m = local / cols;
  const int col = local - r.m * cols;
  r.n = kPair ? 2 * col : col;
  r.tile = c.tile_prefix[lo] + col;
  const int begin = offsets[lo], cnt = offsets[lo + 1] - begin;
  r.row0 = begin + r.n * n_box;
  r.nvalid = min(n_box, cnt - r.n * n_box);
  r.nt = kPair && (r.n + 1) * n_box < cnt ? 2 : 1;
  r.nvalid1 = r.nt == 2 ? min(n_box, cnt - (r.n + 1) * n_box) : 0;
  return r;
}

// bf16x2 multiply (round to nearest); exact here: both factors have <= 4 significant bits.
__device__ __forceinline__ uint32_t hmul2_bf16(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// One permuted code word (8 elements) -> 4 bf16x2 of e2m1 * sf * 2^-66 (layout.cuh).
// The integer logic pipe and the multiply pipe each run these ops at half rate, so the two
// left shifts that never need wrapped bits (rotl 4, and the << 6 of the last pair) are done
// as multiplies by m16 = 16 and m64 = 64 -- values the compiler cannot see, so they stay on
// the multiply pipe -- leaving 5 logic ops and 2 funnel shifts per word on the logic pipe.
__device__ __forceinline__ void dequant8(uint32_t w, uint32_t scale2, uint32_t m16, uint32_t m64,
                                         uint32_t* out) {
  constexpr uint32_t kMask = 0x81C081C0u;
  out[0] = hmul2_bf16(w & kMask, scale2);
  out[1] = hmul2_bf16((w * m16) & kMask, scale2);
  out[2] = hmul2_bf16(ptx::rotl(w, 10) & kMask, scale2);
  out[3] = hmul2_bf16(((w * m64) & 0x80C080C0u) | ((w >> 2) & 0x01000100u), scale2);
}

__device__ __forceinline__ void record_error(int* flag, int code) {
  if (flag) atomicExch(flag, code);
}

// The layer's combine (fused launches): out[t] = sum over t's local slots, in ascending expert
// order, of topk_weight * rsqrt(mean(ypart^2) + eps) * ypart, fp32, then bf16 (or fp32 for an
// expert-parallel share). Restates reference.py:88-90,106-107 with combine.cu's arithmetic.
// The work is (token, column range) pieces, piece i to CTA i % G: with fewer tokens than CTAs a
// token's columns are cut into ranges so that the whole grid combines it (each piece recomputes
// the token's coefficients, which are read from the rows' slice sums of squares). A token's
// slots are found and ordered from the routing tables before the rows exist; then one wait on
// the GEMM2 completion counter (every epilogue warp of every CTA adds 1 after its last item),
// and the rows' sums of squares and values are read together.
__device__ __forceinline__ void combine_tokens(SharedCtl& ctl, const GemmArgs& a, int n_local) {
  const int K = a.top_k, H = a.hidden, H4 = H >> 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total_rows = ctl.offs[n_local];
  const int G = gridDim.x;
  // column ranges per token (at least 8 float4 columns each) and their width in float4 columns
  const int ranges = a.tokens >= G ? 1 : max(1, min(G / a.tokens, H4 / 8));
  const int width = (H4 + ranges - 1) / ranges;
  bool waited = false;
  for (int piece = blockIdx.x; piece < a.tokens * ranges; piece += G) {
    const int t = piece / ranges;
    const int h4_begin = (piece - t * ranges) * width, h4_end = min(H4, h4_begin + width);
    if (threadIdx.x < K) {
      ctl.c_row[threadIdx.x] = -1;
      ctl.c_key[threadIdx.x] = a.ids[t * K + threadIdx.x];
      ctl.c_scoef[threadIdx.x] = a.topk_weights[t * K + threadIdx.x];   // slot weights for now
    }
    __syncthreads();
    for (int r = threadIdx.x; r < total_rows; r += blockDim.x)
      if (ctl.order[r] == t) ctl.c_row[ctl.slot_of_row[r]] = r;
    __syncthreads();
    if (threadIdx.x == 0) {
      ctl.c_n = sort_local_slots(ctl.c_row, ctl.c_key, ctl.c_scoef, K, ctl.c_order, ctl.c_srow, ctl.c_coef);
      if (!waited && !ptx::wait_counter(a.ph[1].signal, 4 * (int)gridDim.x)) record_error(a.error_flag, 5);
    }
    waited = true;
    __syncthreads();
    const int n = ctl.c_n;
    if (warp < n) {   // sorted slot `warp`: its post-norm coefficient (c_coef holds its weight)
      const float c = post_norm_coef(a.ssq + (size_t)ctl.c_srow[warp] * (H >> 5), H, ctl.c_coef[warp]);
      if (lane == 0) ctl.c_scoef[warp] = c;
    }
    // The rows' values are loaded while the coefficients are being computed. Every thread makes
    // the same number of passes (the barrier inside), and only those with a column group work.
    for (int base4 = h4_begin; base4 < h4_end; base4 += blockDim.x) {
      const int h4 = base4 + threadIdx.x;
      const bool mine = h4 < h4_end;
      // the first eight rows are in flight across the barrier; more slots (top_k > 8) follow
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (mine && u < n) v[u] = __ldcg(reinterpret_cast<const float4*>(a.ypart + (size_t)ctl.c_srow[u] * H) + h4);
      __syncthreads();
      if (!mine) continue;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int u0 = 0; u0 < n; u0 += 8) {
        if (u0 > 0) {
#pragma unroll
          for (int u = 0; u < 8; ++u)
            if (u0 + u < n) v[u] = __ldcg(reinterpret_cast<const float4*>(a.ypart + (size_t)ctl.c_srow[u0 + u] * H) + h4);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (u0 + u < n) {
            const float c = ctl.c_scoef[u0 + u];
            acc.x = fmaf(c, v[u].x, acc.x);
            acc.y = fmaf(c, v[u].y, acc.y);
            acc.z = fmaf(c, v[u].z, acc.z);
            acc.w = fmaf(c, v[u].w, acc.w);
          }
        }
      }
      if (a.out_f32)
        reinterpret_cast<float4*>(static_cast<float*>(a.out) + (size_t)t * H)[h4] = acc;
      else
        reinterpret_cast<uint2*>(static_cast<uint16_t*>(a.out) + (size_t)t * H)[h4] = pack_bf16x4(acc);
    }
    __syncthreads();
  }
}

// kFused: the single-launch variant (two phases with cross-CTA tile counters, then the
// combine). The plain variant leaves that code out of its loops. kPair: items of up to two
// token tiles (P = 1; see kPairAccSlots).
template <int P, int DW, bool kFused, bool kPair>
__global__ void __launch_bounds__(Roles<P, DW>::kThreads, 1)
expert_gemm_tc(const __grid_constant__ CUtensorMap tmap_b, const __grid_constant__ CUtensorMap tmap_x,
               const __grid_constant__ CUtensorMap tmap_b2, const GemmArgs a) {
  static_assert(!kPair || (P == 1 && !kFused), "pair-tile items: one pipeline, separate launches");
  using R = Roles<P, DW>;
  constexpr int kPipes = P;
  constexpr int kMmaWarp0 = R::kMmaWarp0, kEpiWarp0 = R::kEpiWarp0, kDeqWarp0 = R::kDeqWarp0;
  constexpr int kPipeCols = R::kPipeCols;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Geo geo = make_geo(kPipeCols, a.n_box, a.stages, a.b_stages, kPair);
  const int Sw = geo.Sw, Sb = geo.Sb, n_box = geo.n_box;
  SharedCtl& ctl = *reinterpret_cast<SharedCtl*>(smem + (size_t)kPipes * geo.pipe_bytes);
  // pipeline p: Sw weight slots [fp4 codes | scales], then Sb activation slots [box | box]
  auto w_slot = [&](int p, int s) { return smem + (size_t)p * geo.pipe_bytes + (size_t)s * kWStageBytes; };
  auto b_slot = [&](int p, int s) {
    return smem + (size_t)p * geo.pipe_bytes + (size_t)Sw * kWStageBytes + (size_t)s * geo.b_bytes;
  };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_local = a.n_local;
  if (threadIdx.x == 0) MUSE_TRACE_ENTRY();

  // ---- set-up: barriers, scale table, work list, tensor memory
  auto init_barrier = [&](int p, int r) {  // barrier r of pipeline p's control block (single launch)
    PipeCtl& pc = ctl.pipe[p];
    if (r < Sw) return ptx::mbar_init(&pc.w_full[r], 1);
    if ((r -= Sw) < Sw) return ptx::mbar_init(&pc.w_empty[r], DW);  // the dequant warps
    if ((r -= Sw) < Sb) return ptx::mbar_init(&pc.b_full[r], 1);
    if ((r -= Sb) < Sb) return ptx::mbar_init(&pc.b_empty[r], 1);  // MMA commit
    if ((r -= Sb) < geo.n_a) return ptx::mbar_init(&pc.a_full[r], DW);
    if ((r -= geo.n_a) < geo.n_a) return ptx::mbar_init(&pc.a_empty[r], 1);
    if ((r -= geo.n_a) < geo.n_acc) return ptx::mbar_init(&pc.acc_full[r], 1);
    if ((r -= geo.n_acc) < geo.n_acc) return ptx::mbar_init(&pc.acc_empty[r], 4);
    ptx::mbar_init(&pc.drain, 1);
  };
  const int per_pipe = 2 * Sw + 2 * Sb + 2 * geo.n_a + 2 * geo.n_acc + 1;
  if (kFused) {
    // Single launch (latency-bound): the last warp initialises the barriers, one lane per
    // barrier, while the first warps already load the routing ids.
    if (warp == R::kWarps - 1) {
      for (int i = lane; i < kPipes * per_pipe; i += 32) init_barrier(i / per_pipe, i % per_pipe);
      ptx::fence_barrier_init();
      if (lane == 0) MUSE_TRACE_AT(5);
    }
  } else if (threadIdx.x == 0) {
    for (int p = 0; p < kPipes; ++p) {
      PipeCtl& pc = ctl.pipe[p];
      for (int s = 0; s < Sw; ++s) {
        ptx::mbar_init(&pc.w_full[s], 1);
        ptx::mbar_init(&pc.w_empty[s], DW);  // the dequant warps
      }
      for (int s = 0; s < Sb; ++s) {
        ptx::mbar_init(&pc.b_full[s], 1);
        ptx::mbar_init(&pc.b_empty[s], 1);  // MMA commit
      }
      for (int b = 0; b < geo.n_a; ++b) {
        ptx::mbar_init(&pc.a_full[b], DW);
        ptx::mbar_init(&pc.a_empty[b], 1);
      }
      for (int b = 0; b < geo.n_acc; ++b) {
        ptx::mbar_init(&pc.acc_full[b], 1);
        ptx::mbar_init(&pc.acc_empty[b], 4);
      }
      ptx::mbar_init(&pc.drain, 1);
    }
    ptx::fence_barrier_init();
    MUSE_TRACE_AT(5);
  }
  if (warp < kPipes && lane == 0) {
    ptx::prefetch_tensormap(a.route_inline ? &tmap_x : &tmap_b);
    if (kFused && a.n_phases > 1) ptx::prefetch_tensormap(&tmap_b2);
  }
  // Expert ranges: from the route kernel, or (small batches) computed here by every CTA, with
  // the stage buffers as scratch -- nothing is copied into them before the prologue ends.
  const int32_t* offs = a.offsets;
  if (a.route_inline) {
    route_block(a.ids, a.n_pairs, a.local_start, n_local, reinterpret_cast<int*>(smem), ctl.offs,
                ctl.order, blockIdx.x == 0 ? a.pair_row : nullptr);
    if (blockIdx.x == 0) {
      for (int i = threadIdx.x; i <= n_local; i += R::kThreads) a.offsets[i] = ctl.offs[i];
      for (int i = threadIdx.x; i < a.n_pairs; i += R::kThreads) a.pair_order[i] = ctl.order[i];
    }
    offs = ctl.offs;
  }
  if (threadIdx.x == 0) MUSE_TRACE_AT(6);
  int incl = 0;  // item columns of experts [32 * warp, threadIdx.x], threads < 256
  if (threadIdx.x < 256) {
    const float f = e4m3_to_float(threadIdx.x) * 1152921504606846976.0f;  // * 2^60
    const __nv_bfloat16 h = __float2bfloat16_rn(f);
    const uint32_t u = *reinterpret_cast<const uint16_t*>(&h);
    ctl.scale_lut[threadIdx.x] = u | (u << 16);
    // token tiles per expert, warp-inclusive scan (completed across warps below)
    const int e = threadIdx.x;
    int cnt = 0;
    if (e < n_local) cnt = offs[e + 1] - offs[e];
    const int nt = (cnt + n_box - 1) / n_box;
    if (e < n_local) ctl.ntiles[e] = nt;
    incl = kPair ? (nt + 1) >> 1 : nt;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += o;
    }
    if (lane == 31) ctl.tile_warp_sum[warp] = incl;
  }
  if (warp == kMmaWarp0) {
    ptx::tmem_alloc(&ctl.tmem_base, kTmemCols);
    ptx::tmem_relinquish();
  }
  if (threadIdx.x == 0) MUSE_TRACE_AT(7);
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (threadIdx.x == 0) MUSE_TRACE_AT(8);
  if (a.route_inline) {  // pair index -> token and slot (CTA 0 has published the pair indices)
    for (int i = threadIdx.x; i < a.n_pairs; i += R::kThreads) {
      const int pr = ctl.order[i];
      if (pr >= 0) {
        ctl.order[i] = pr / a.top_k;
        ctl.slot_of_row[i] = (uint8_t)(pr - ctl.order[i] * a.top_k);
      }
    }
  }
  if (threadIdx.x < 256) {  // complete the scan across the 8 warps
    int before = 0;
    for (int w = 0; w < warp; ++w) before += ctl.tile_warp_sum[w];
    ctl.tile_prefix[threadIdx.x + 1] = before + incl;
    if (threadIdx.x == 0) ctl.tile_prefix[0] = 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) MUSE_TRACE_AT(2);

  const uint32_t tbase = ctl.tmem_base;
  const int tiles = ctl.tile_prefix[n_local];       // item columns (token tiles, or pairs)
  const int mt0 = a.ph[0].m_tiles, mt1 = kFused && a.n_phases > 1 ? a.ph[1].m_tiles : 0;
  const int n0 = tiles * mt0;                       // items of phase 0
  const int total = n0 + tiles * mt1;               // all items of this launch
  const int G = gridDim.x;
  // Item j of this CTA is blockIdx.x + j * G (phase 0 items first, so a CTA finishes its GEMM1
  // items before any GEMM2 item). In a split-K phase its K chunks are split over the
  // pipelines: pipeline p takes the chunks kc with (kc + j) % P == p, into its own accumulator,
  // and the epilogue sums the partial accumulators (rotating with j balances the pipelines
  // when P does not divide the chunk count). Otherwise (few chunks per item) item j goes whole
  // to pipeline j % P, so each item costs one accumulator hand-off instead of P.
  // A phase is split when the host asks for it (many chunks per item) and also whenever it has
  // fewer than 4 items per CTA: with 1-2 items a CTA would leave pipelines idle, and splitting
  // never gives a pipeline more chunks than whole items would, so the CTA's longest pipeline
  // -- the decode critical path -- gets shorter.
  const bool split0 = a.ph[0].split_k || (a.ph[0].k_chunks > 1 && n0 < 4 * G);
  const bool split1 = kFused && a.n_phases > 1 && (a.ph[1].split_k || (a.ph[1].k_chunks > 1 && total - n0 < 4 * G));
  // jm = j % P; returns the first chunk of pipeline p (k_chunks if it has none).
  auto chunk_begin = [&](int p, int jm, const PhaseArgs& f, bool split) {
    return split ? (p - jm + kPipes) % kPipes : (p == jm ? 0 : f.k_chunks);
  };
  auto phase_of = [&](int it) { return kFused && it >= n0 ? 1 : 0; };

  if (warp < kMmaWarp0) {
    // ------------------------------------------------------------------ producers
    const int p = warp;
    PipeCtl& pc = ctl.pipe[p];
    {
      // The whole warp walks the loop (warp-uniform values stay in uniform registers); the
      // elected leader issues the copies.
      const bool leader = ptx::elect_one();
      bool ok = true;
      Ring ws, bs;
      int w_issued = 0, b_issued = 0;
      // Dependency readiness of this CTA's items j0 .. j0 + 31 (bit j - j0), read 32 counters at
      // a time so that a satisfied dependency costs no round trip to L2.
      uint32_t dep_ready = 0;
      int dep_j0 = -64;
      if (p == 0 && lane == 0) MUSE_TRACE_AT(9);
      int jm = 0;
      for (int j = 0; ok && blockIdx.x + j * G < total; ++j, jm = (jm + 1 == kPipes ? 0 : jm + 1)) {
        const int it = blockIdx.x + j * G;
        const int ph = phase_of(it);
        const PhaseArgs& f = a.ph[ph];
        const bool split = ph ? split1 : split0;
        const int kcn = f.k_chunks, kstep = split ? kPipes : 1;
        const int kc0 = chunk_begin(p, jm, f, split);
        if (kc0 >= kcn) continue;
        const Item t = decode_item<kPair>(ctl, offs, it, n0, n_local, n_box, mt0, mt1);
        const size_t tile0 = ((size_t)t.e * f.m_tiles + t.m) * kcn;
        bool dep_ok = !kFused || f.wait_for == nullptr;
        for (int kc = kc0; kc < kcn; kc += kstep) {
          if (!__all_sync(0xffffffffu, ptx::mbar_wait_sleep(&pc.w_empty[ws.slot], ws.phase ^ 1))) {
            ok = false;
            break;
          }
          uint8_t* wp = w_slot(p, ws.slot);
          if (leader) {
            ptx::mbar_arrive_expect_tx(&pc.w_full[ws.slot], kWStageBytes);
            ptx::bulk_g2s(wp, f.wq + (tile0 + kc) * kTileCodeBytes, kTileCodeBytes, &pc.w_full[ws.slot]);
            ptx::bulk_g2s(wp + kTileCodeBytes, f.wsf + (tile0 + kc) * kTileScaleBytes, kTileScaleBytes,
                          &pc.w_full[ws.slot]);
            MUSE_TRACE_SEQ(trace::kTrW, p, w_issued);
          }
          ++w_issued;
          ws.next(Sw);
          if (!dep_ok) {
            // the B rows of this item are written by other CTAs' epilogues (the previous phase):
            // the weight tile is already on its way, the activation box waits for the counter
            if (j - dep_j0 >= 32 || !((dep_ready >> (j - dep_j0)) & 1u)) {
              const int itl = blockIdx.x + (j + lane) * G;
              bool rdy = false;
              if (itl < total && itl >= n0) {
                const Item tl = decode_item<kPair>(ctl, offs, itl, n0, n_local, n_box, mt0, mt1);
                rdy = ptx::ld_acquire_gpu(f.wait_for + tl.tile) >= f.wait_target;
              }
              dep_ready = __ballot_sync(0xffffffffu, rdy);
              dep_j0 = j;
            }
            dep_ok = (dep_ready >> (j - dep_j0)) & 1u;
            if (!dep_ok)
              dep_ok = __all_sync(0xffffffffu, leader ? ptx::wait_counter(f.wait_for + t.tile, f.wait_target) : true);
            if (!dep_ok) {
              ok = false;
              break;
            }
            __syncwarp();
            if (leader) ptx::fence_proxy_async_global();
          }
          if (!__all_sync(0xffffffffu, ptx::mbar_wait_sleep(&pc.b_empty[bs.slot], bs.phase ^ 1))) {
            ok = false;
            break;
          }
          uint8_t* bp = b_slot(p, bs.slot);
          uint64_t* bb = &pc.b_full[bs.slot];
          if (f.b_source == 1) {
            // Activation rows straight from x[token], four rows per gather; only the groups that
            // hold the tile's pairs are loaded (the MMA columns of the rest are never read).
            const int groups = (t.nvalid + 3) >> 2;
            const int* tok = ctl.order + t.row0;
            const int last = t.nvalid - 1;
            if (leader) {
              ptx::mbar_arrive_expect_tx(bb, groups * 1024);
              for (int g4 = 0; g4 < groups; ++g4) {
                const int i = 4 * g4;
                const int r0 = tok[i], r1 = tok[min(i + 1, last)], r2 = tok[min(i + 2, last)],
                          r3 = tok[min(i + 3, last)];
                ptx::tma_gather4_2d(bp + i * 128, &tmap_x, kc * kChunkK, r0, r1, r2, r3, bb);
                ptx::tma_gather4_2d(bp + (n_box + i) * 128, &tmap_x, kc * kChunkK + 64, r0, r1, r2, r3, bb);
              }
            }
          } else if (leader) {
            // [tile 0: box | box][tile 1: box | box] (pair items), each box 64 columns x n_box rows
            const CUtensorMap* tm = f.b_source == 2 ? &tmap_b2 : &tmap_b;
            const uint32_t tile_bytes = 2u * n_box * 128u;
            ptx::mbar_arrive_expect_tx(bb, t.nt * tile_bytes);
            for (int h = 0; h < t.nt; ++h) {
              ptx::tma_load_2d(bp + h * tile_bytes, tm, kc * kChunkK, t.row0 + h * n_box, bb);
              ptx::tma_load_2d(bp + h * tile_bytes + n_box * 128, tm, kc * kChunkK + 64, t.row0 + h * n_box, bb);
            }
          }
          if (leader) MUSE_TRACE_SEQ(trace::kTrB, p, b_issued);
          ++b_issued;
          bs.next(Sb);
        }
      }
      if (!ok) {
        if (leader) record_error(a.error_flag, 1);
        // let copies already in flight land before the CTA can exit: walk back over the last
        // min(issued, depth) slots of each ring
        int s = ws.slot;
        uint32_t ph = ws.phase;
        for (int i = 0; i < w_issued && i < Sw; ++i) {
          if (s == 0) { s = Sw; ph ^= 1u; }
          --s;
          ptx::mbar_wait(&pc.w_full[s], ph);
        }
        s = bs.slot;
        ph = bs.phase;
        for (int i = 0; i < b_issued && i < Sb; ++i) {
          if (s == 0) { s = Sb; ph ^= 1u; }
          --s;
          ptx::mbar_wait(&pc.b_full[s], ph);
        }
      }
    }
  } else if (warp < kEpiWarp0) {
    // ------------------------------------------------------------------ MMA issuers
    const int p = warp - kMmaWarp0;
    PipeCtl& pc = ctl.pipe[p];
    {
      // The whole warp walks the loop; the elected leader issues the MMAs and the commits that
      // track them (a commit covers the MMAs of its own thread).
      const bool leader = ptx::elect_one();
      bool ok = true;
      const uint32_t col0 = tbase + p * kPipeCols;
      const uint32_t acc_col0 = col0 + geo.n_a * kACols;
      Ring st, ar, accr;
      const uint64_t desc_first = ptx::smem_desc_k_sw128(ptx::smem_u32(b_slot(p, 0)), 1024);
      const uint32_t stage_step = geo.b_bytes >> 4;              // descriptor units (16 B)
      const uint32_t atom_step = (uint32_t)(n_box * 128) >> 4;  // second 64-K box of a slot
      uint64_t desc_stage = desc_first;
#ifdef MUSE_TRACE
      int tr_c = 0;
#endif
      int jm = 0;
      for (int j = 0; ok && blockIdx.x + j * G < total; ++j, jm = (jm + 1 == kPipes ? 0 : jm + 1)) {
        const int ph = phase_of(blockIdx.x + j * G);
        const PhaseArgs& f = a.ph[ph];
        const bool split = ph ? split1 : split0;
        const int kcn = f.k_chunks, kstep = split ? kPipes : 1;
        const int kc0 = chunk_begin(p, jm, f, split);
        if (kc0 >= kcn) continue;
        // MMA width = the item's token rows rounded up to 16, not the whole tile: a partly
        // filled tile (the last of an expert, or an expert with few pairs) costs the tensor
        // core only its own columns
        const Item t = decode_item<kPair>(ctl, offs, blockIdx.x + j * G, n0, n_local, n_box, mt0, mt1);
        const uint32_t idesc = ptx::idesc_bf16_f32(kTileM, min(n_box, (t.nvalid + 15) & ~15));
        const int acc = accr.slot;
        // pair items: the second tile's accumulator is the ring's next slot
        Ring acc2 = accr;
        acc2.next(geo.n_acc);
        const bool two = kPair && t.nt == 2;
        const uint32_t idesc2 = two ? ptx::idesc_bf16_f32(kTileM, min(n_box, (t.nvalid1 + 15) & ~15)) : 0u;
        if (!__all_sync(0xffffffffu, ptx::mbar_wait_sleep(&pc.acc_empty[acc], accr.phase ^ 1) &&
                                         (!two || ptx::mbar_wait_sleep(&pc.acc_empty[acc2.slot], acc2.phase ^ 1)))) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_tmem = acc_col0 + acc * n_box;
        const uint32_t d_tmem2 = acc_col0 + acc2.slot * n_box;
        const uint32_t tile_step = (2u * n_box * 128u) >> 4;   // second tile's boxes in a slot
        for (int kc = kc0; kc < kcn; kc += kstep) {
          const int s = st.slot;
          const int ab = ar.slot;
          const bool ready = ptx::mbar_wait_sleep(&pc.a_full[ab], ar.phase) &&
                             ptx::mbar_wait_sleep(&pc.b_full[s], st.phase);
          if (!__all_sync(0xffffffffu, ready)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t a_tmem = col0 + ab * kACols;
          if (leader) {
#pragma unroll
            for (int kk = 0; kk < kChunkK / 16; ++kk) {
              const uint64_t bdesc = desc_stage + (uint64_t)((kk >> 2) * atom_step + (kk & 3) * 2);
              ptx::mma_bf16_ts(d_tmem, a_tmem + kk * 8, bdesc, idesc, (kc != kc0) | (kk != 0));
              if (two) ptx::mma_bf16_ts(d_tmem2, a_tmem + kk * 8, bdesc + tile_step, idesc2, (kc != kc0) | (kk != 0));
            }
            ptx::mma_commit(&pc.b_empty[s]);
            ptx::mma_commit(&pc.a_empty[ab]);
#ifdef MUSE_TRACE
            MUSE_TRACE_SEQ(trace::kTrM, p, tr_c);
#endif
          }
#ifdef MUSE_TRACE
          ++tr_c;
#endif
          __syncwarp();
          ar.next(geo.n_a);
          st.next(Sb);
          desc_stage = st.slot == 0 ? desc_first : desc_stage + stage_step;
        }
        if (!ok) break;
        if (leader) {
          ptx::mma_commit(&pc.acc_full[acc]);
          if (two) ptx::mma_commit(&pc.acc_full[acc2.slot]);
        }
        __syncwarp();
        accr.next(geo.n_acc);
        if (two) accr.next(geo.n_acc);
      }
      if (!ok && leader) record_error(a.error_flag, 2);
      // all issued MMAs complete before tensor memory is released
      if (leader) ptx::mma_commit(&pc.drain);
      __syncwarp();
      ptx::mbar_wait(&pc.drain, 0);
    }
  } else if (warp < kDeqWarp0) {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const uint32_t lane_base = tbase + ((uint32_t)(32 * q) << 16) + geo.n_a * kACols;
    bool ok = true;
    Ring accr[kPipes];
    // Per-item constants (the item, its global scale, this lane's post-norm weight) are loaded
    // one item ahead, so their global-memory latency overlaps the previous item.
    auto item_consts = [&](int it, Item& t, float& gs, float& pnw) {
      t = decode_item<kPair>(ctl, offs, it, n0, n_local, n_box, mt0, mt1);
      const PhaseArgs& f = a.ph[t.ph];
      gs = __ldg(f.gs + t.e);
      pnw = f.mode == 2 ? bf16_bits_to_float(__ldg(a.post_norm_w + kTileM * t.m + 32 * q + lane)) : 0.f;
    };
    Item t_next;
    float gs_next = 0.f, pnw_next = 0.f;
    if (blockIdx.x < total) item_consts(blockIdx.x, t_next, gs_next, pnw_next);
    int jm = 0;
    for (int j = 0; ok && blockIdx.x + j * G < total; ++j, jm = (jm + 1 == kPipes ? 0 : jm + 1)) {
      const Item t = t_next;
      const float gs_item = gs_next, pnw_item = pnw_next;
      if (blockIdx.x + (j + 1) * G < total) item_consts(blockIdx.x + (j + 1) * G, t_next, gs_next, pnw_next);
      const PhaseArgs& f = a.ph[t.ph];
      const bool split = t.ph ? split1 : split0;
      const int kcn = f.k_chunks;
      // a pair item's second token tile is a second accumulator, finished the same way
      for (int tt = 0; tt < (kPair ? t.nt : 1); ++tt) {
        const int row0 = t.row0 + tt * n_box;
        const int nvalid = tt ? t.nvalid1 : t.nvalid;
        // accumulators of the participating pipelines
        uint32_t taddr[kPipes];
        int used = 0;
#pragma unroll
        for (int p = 0; p < kPipes; ++p) {
          if (chunk_begin(p, jm, f, split) >= kcn) continue;
          if (!ptx::mbar_wait_sleep(&ctl.pipe[p].acc_full[accr[p].slot], accr[p].phase)) ok = false;
          taddr[used++] = lane_base + p * kPipeCols + accr[p].slot * n_box;
        }
        if (!ok) break;
        ptx::tc_fence_after();
        if (q == 0 && lane == 0) MUSE_TRACE_ITEM(trace::kTrE, j);
        const float gsc = gs_item * kUnscale;
        if (f.mode == 1) {
          const int jj = 64 * t.m + 16 * q + (lane & 15);  // intermediate index of this lane
          for (int cb = 0; cb * 16 < nvalid; ++cb) {
            float acc[16];
            uint32_t v[16];
            ptx::tmem_ld16(taddr[0] + cb * 16, v);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 16; ++c) acc[c] = __uint_as_float(v[c]);
            for (int u = 1; u < used; ++u) {
              ptx::tmem_ld16(taddr[u] + cb * 16, v);
              ptx::tmem_wait_ld();
#pragma unroll
              for (int c = 0; c < 16; ++c) acc[c] += __uint_as_float(v[c]);
            }
            // four columns at a time (independent chains the scheduler can overlap), only as many
            // groups as the item has rows: the epilogue shares the issue slots of the dequantisers
            const int ncols = min(16, nvalid - cb * 16);  // warp-uniform
#pragma unroll
            for (int c4 = 0; c4 < 16; c4 += 4) {
              if (c4 >= ncols) break;
              float act[4];
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const float mine = acc[c4 + k] * gsc;
                const float other = __shfl_xor_sync(0xffffffffu, mine, 16);
                // lanes < 16: silu(gate) * up; fast divide (2 ulp): the result is rounded to bf16
                act[k] = __fdividef(mine, 1.0f + __expf(-mine)) * other;
              }
              if (lane < 16) {
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                  if (c4 + k < ncols) {
                    const __nv_bfloat16 hb = __float2bfloat16_rn(act[k]);
                    a.inter[(size_t)(row0 + cb * 16 + c4 + k) * f.ld_out + jj] = *reinterpret_cast<const uint16_t*>(&hb);
                  }
                }
              }
            }
          }
        } else {
          const int h = kTileM * t.m + 32 * q + lane;  // output row of this lane
          const float wn = gsc * (1.0f + pnw_item);
          for (int cb = 0; cb * 16 < nvalid; ++cb) {
            float acc[16];
            uint32_t v[16];
            ptx::tmem_ld16(taddr[0] + cb * 16, v);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 16; ++c) acc[c] = __uint_as_float(v[c]);
            for (int u = 1; u < used; ++u) {
              ptx::tmem_ld16(taddr[u] + cb * 16, v);
              ptx::tmem_wait_ld();
#pragma unroll
              for (int c = 0; c < 16; ++c) acc[c] += __uint_as_float(v[c]);
            }
            const int ncols = min(16, nvalid - cb * 16);  // warp-uniform
#pragma unroll
            for (int col = 0; col < 16; ++col) {
              acc[col] *= wn;
              if (col < ncols) a.ypart[(size_t)(row0 + cb * 16 + col) * f.ld_out + h] = acc[col];
              acc[col] *= acc[col];
            }
            // Sum of squares of each column over the warp's 32 rows, all 16 columns at once: a
            // transposed butterfly (each round halves the columns a lane keeps, 16 shuffles in
            // all). It adds the same pairs as a per-column xor 16/8/4/2/1 reduction, so the sums
            // are bit-identical to it; lanes 2c and 2c + 1 end with column c.
#pragma unroll
            for (int half = 8; half >= 1; half >>= 1) {
              const bool up = lane & (2 * half);
#pragma unroll
              for (int i = 0; i < half; ++i) {
                const float keep = up ? acc[half + i] : acc[i];
                const float send = up ? acc[i] : acc[half + i];
                acc[i] = keep + __shfl_xor_sync(0xffffffffu, send, 2 * half);
              }
            }
            acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], 1);
            const int c = (lane >> 1) & 15;
            if (!(lane & 1) && c < ncols)
              a.ssq[(size_t)(row0 + cb * 16 + c) * (f.ld_out >> 5) + (h >> 5)] = acc[0];
          }
        }
        ptx::tc_fence_before();
        if (q == 0 && lane == 0) MUSE_TRACE_ITEM(trace::kTrE + trace::kTrJ, j);
        __syncwarp();
        // Single launch: this warp's rows of a GEMM1 item are published as soon as they are
        // stored (a CTA's items belong to different experts, so waiting for its last GEMM1 item
        // would hold back GEMM2 items that depend only on the first). The warp barrier orders
        // every lane's stores before lane 0's release.
        if (kFused && t.ph == 0 && a.ph[0].signal) {
          if (lane == 0) ptx::red_release_gpu_add(a.ph[0].signal + t.tile, 1);
          __syncwarp();
        }
#pragma unroll
        for (int p = 0; p < kPipes; ++p) {
          if (chunk_begin(p, jm, f, split) >= kcn) continue;
          if (lane == 0) ptx::mbar_arrive(&ctl.pipe[p].acc_empty[accr[p].slot]);
          accr[p].next(geo.n_acc);
        }
      }
    }
    // Single launch: one increment of the GEMM2 completion counter per warp, after its last item.
    if (kFused && ok && a.ph[1].signal) {
      __syncwarp();
      if (lane == 0) {
        __threadfence();
        ptx::red_relaxed_gpu_add(a.ph[1].signal, 1);
      }
    }
    if (!ok && lane == 0) record_error(a.error_flag, 3);
  } else {
    // ------------------------------------------------------------------ dequantisers
    // A chunk is converted in 16-column groups (32 elements of this thread's row). The shared-
    // memory reads of group g + 1 -- its 16 code bytes and its two scale-table entries -- are
    // issued before group g is converted, so their latency hides behind the arithmetic; the
    // reads of the next chunk's first group are issued during the last group whenever that
    // weight tile has already landed. A weight slot is handed back as soon as its last bytes
    // are in registers, and the A buffer is waited for only once the first group is converted.
    const int p = (warp - kDeqWarp0) / DW;
    PipeCtl& pc = ctl.pipe[p];
    const int q = warp & 3;                  // TMEM lane quarter
    const int hsel = DW == 8 ? ((warp - kDeqWarp0) % DW) >> 2 : 0;  // DW = 8: this warp's half
    const int row = 32 * q + lane;           // weight row of this thread
    const uint32_t lane_col0 = tbase + ((uint32_t)(32 * q) << 16) + p * kPipeCols;
    const uint32_t m16 = a.mul16, m64 = a.mul64;
    constexpr int kGroups = DW == 8 ? 2 : 4;  // 16-column groups of a chunk this warp converts
    bool ok = true;
    Ring st, ar;
    // this pipeline's chunks in order: item j (jm = j % P), chunk kc of it
    int j = -1, jm = kPipes - 1, kc = 0, kcn = 0, kstep = 1;
    auto advance = [&]() -> bool {
      kc += kstep;
      while (kc >= kcn) {
        ++j;
        jm = jm + 1 == kPipes ? 0 : jm + 1;
        if (blockIdx.x + j * G >= total) return false;
        const int ph = phase_of(blockIdx.x + j * G);
        const PhaseArgs& f = a.ph[ph];
        const bool split = ph ? split1 : split0;
        kcn = f.k_chunks;
        kstep = split ? kPipes : 1;
        kc = chunk_begin(p, jm, f, split);
      }
      return true;
    };
#ifdef MUSE_TRACE
    int tr_c = 0;
#endif
    // Group g's 16 code bytes of this row in weight slot `slot`.
    auto load_codes = [&](int slot, int g) -> uint4 {
      return *reinterpret_cast<const uint4*>(w_slot(p, slot) + row * kRowCodeBytes +
                                             16 * code_slot(row, 2 * hsel + g));
    };
    // This row's 8 scale bytes of the chunk in slot `slot` (group g uses bytes 2g, 2g + 1 of
    // its warp's half).
    auto load_scales = [&](int slot) -> uint2 {
      return *reinterpret_cast<const uint2*>(w_slot(p, slot) + kTileCodeBytes + row * kRowScaleBytes);
    };
    auto lut = [&](uint2 sfw, int g, uint32_t& s0, uint32_t& s1) {
      const uint32_t sw = (hsel + (g >> 1)) ? sfw.y : sfw.x;
      s0 = ctl.scale_lut[__byte_perm(sw, 0, 0x4440 + 2 * (g & 1))];
      s1 = ctl.scale_lut[__byte_perm(sw, 0, 0x4441 + 2 * (g & 1))];
    };
    bool more = advance();
    uint4 cg = make_uint4(0, 0, 0, 0);   // codes of the group about to be converted
    uint2 sfw = make_uint2(0, 0);        // scale bytes of the current chunk
    uint32_t s0 = 0, s1 = 0;             // its two scale-table entries
    if (more) {
      ok = ptx::mbar_wait_sleep(&pc.w_full[st.slot], st.phase);
      if (ok) {
        sfw = load_scales(st.slot);
        cg = load_codes(st.slot, 0);
        lut(sfw, 0, s0, s1);
      }
    }
    while (ok && more) {
#ifdef MUSE_TRACE
      if (q == 0 && hsel == 0 && lane == 0) MUSE_TRACE_SEQ(trace::kTrF, p, tr_c);
#endif
      const int ab = ar.slot;
      const int cur = st.slot;
      bool next_loaded = false, more_next = false;
      uint2 sfw_next = sfw;
#pragma unroll
      for (int g = 0; g < kGroups; ++g) {
        // issue the next group's reads before converting this one
        uint4 cn = cg;
        uint32_t n0 = s0, n1 = s1;
        if (g + 1 < kGroups) {
          cn = load_codes(cur, g + 1);
          lut(sfw, g + 1, n0, n1);
        } else {
          // every byte of this chunk is read: hand the slot back, then look ahead
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(&pc.w_empty[cur]);
          st.next(Sw);
          more_next = advance();
          if (more_next && __all_sync(0xffffffffu, ptx::mbar_try_wait(&pc.w_full[st.slot], st.phase))) {
            sfw_next = load_scales(st.slot);
            cn = load_codes(st.slot, 0);
            next_loaded = true;
          }
        }
        uint32_t out[16];
        dequant8(cg.x, s0, m16, m64, &out[0]);
        dequant8(cg.y, s0, m16, m64, &out[4]);
        dequant8(cg.z, s1, m16, m64, &out[8]);
        dequant8(cg.w, s1, m16, m64, &out[12]);
        if (g == 0 && !ptx::mbar_wait_sleep(&pc.a_empty[ab], ar.phase ^ 1)) {
          ok = false;
          break;
        }
        ptx::tmem_st16(lane_col0 + ab * kACols + hsel * 32 + g * 16, out);
        cg = cn;
        s0 = n0;
        s1 = n1;
      }
      if (!ok) break;
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&pc.a_full[ab]);
#ifdef MUSE_TRACE
      if (q == 0 && hsel == 0 && lane == 0) MUSE_TRACE_SEQ(trace::kTrA, p, tr_c);
      ++tr_c;
#endif
      ar.next(geo.n_a);
      more = more_next;
      if (!more) break;
      if (!next_loaded) {   // the next tile had not landed during the last group: wait for it now
        if (!ptx::mbar_wait_sleep(&pc.w_full[st.slot], st.phase)) {
          ok = false;
          break;
        }
        sfw_next = load_scales(st.slot);
        cg = load_codes(st.slot, 0);
      }
      sfw = sfw_next;
      lut(sfw, 0, s0, s1);
    }
    if (!ok && lane == 0) record_error(a.error_flag, 4);
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (threadIdx.x == 0) MUSE_TRACE_AT(3);
  if (warp == kMmaWarp0) ptx::tmem_dealloc(tbase, kTmemCols);
  if (kFused && a.fused) combine_tokens(ctl, a, n_local);
  // expert-parallel decode: every rank's share summed into this rank's bf16 output
  // (its arguments are read from shared memory: a reference into the kernel's parameters would
  // make the compiler copy all of them to the stack)
  if (kFused && a.ex.ranks > 0) {
    if (threadIdx.x == 0) ctl.ex = a.ex;
    __syncthreads();
    grid_exchange_one_round(ctl.ex, a.error_flag, &ctl.ex_gen, ctl.ex_ok);
  }
  if (threadIdx.x == 0) MUSE_TRACE_AT(4);
}

// Host-side view of one instantiation.
template <int P, int DW> struct Variant {
  static constexpr int kThreads = Roles<P, DW>::kThreads;
  static constexpr int kPipeCols = Roles<P, DW>::kPipeCols;
};

int g_num_sms[64] = {0};
bool g_attr_set[64] = {false};

}  // namespace

// Sticky per-device status word: 0, or the role code (1 producer, 2 MMA, 3 epilogue,
// 4 dequant) of the first bounded wait that expired. Read and cleared by muse_moe_device_status.
__device__ int g_device_status;

int device_status_ptr(int** ptr) {
  return (int)cudaGetSymbolAddress(reinterpret_cast<void**>(ptr), g_device_status);
}

int read_device_status(int* status, int reset) {
  cudaError_t e = cudaMemcpyFromSymbol(status, g_device_status, sizeof(int));
  if (e != cudaSuccess) return e;
  if (reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int));
  }
  return e;
}

// Pipelines per CTA for a token tile: three issuers fit the tensor memory only with N = 16.
int pick_pipes(int n_box, bool pair) { return pair ? 1 : n_box <= 16 ? kDecodePipes : 2; }
// Dequant warps per pipeline for a token tile.
int pick_dw(int n_box, bool pair) { return pair ? 8 : n_box <= 16 ? kDecodeDW : 4; }

int pipe_cols(int pipes) {
  return pipes == 1 ? Variant<1, 8>::kPipeCols : pipes == 3 ? Variant<3, 4>::kPipeCols : Variant<2, 4>::kPipeCols;
}
static_assert(kDecodePipes == 2 || kDecodePipes == 3, "decode pipelines");

size_t gemm_smem_bytes(int n_box, bool pair, int w_stages, int b_stages) {
  const Geo g = make_geo(pipe_cols(pick_pipes(n_box, pair)), n_box, w_stages, b_stages, pair);
  return 1024 + (size_t)pick_pipes(n_box, pair) * g.pipe_bytes + sizeof(SharedCtl);
}

// Ring depths for a token tile: the deepest weight ring that fits 226 KB with one activation
// slot more than weight slots (an activation slot lives until its MMAs complete, a weight slot
// only until it has been read), else equal depths; pair items (64 KiB activation slots) take
// two activation slots and the deepest weight ring beside them.
int pick_stages(int n_box, bool pair, int* b_stages) {
  const int P = pick_pipes(n_box, pair);
  const Geo g = make_geo(pipe_cols(P), n_box, 1, 1, pair);
  const size_t budget = (226u * 1024u - sizeof(SharedCtl) - 1024) / P;
  if (pair) {
    // Pair items (prefill, tensor-bound): the MMAs of a chunk read 64 KiB of activation rows,
    // refetched from L2 for every weight tile, so the activation ring gets three slots and the
    // weights what is left (measured at cfg5 T=4096 / 8192: 4368 / 8108 us against 4780 / 8824
    // with eight weight slots and two activation slots; weight tiles are few and mostly L2 hits
    // by then).
    for (int sw = kMaxStages; sw >= 2; --sw)
      if (sw * (size_t)kWStageBytes + 3 * (size_t)g.b_bytes <= budget) {
        *b_stages = 3;
        return sw;
      }
  }
  for (int sw = kMaxStages; sw >= 2; --sw) {
    for (int extra = 1; extra >= (pair ? 2 - sw : 0); --extra) {
      const int sb = sw + extra;
      if (sb >= 2 && sb <= kMaxStages && sw * (size_t)kWStageBytes + sb * (size_t)g.b_bytes <= budget) {
        *b_stages = sb;
        return sw;
      }
    }
  }
  *b_stages = 2;
  return 2;
}

template <int P, int DW, bool kFused, bool kPair = false>
cudaError_t launch_variant(int grid, size_t smem, bool cooperative, const CUtensorMap& tmap_b,
                           const CUtensorMap& tmap_x, const CUtensorMap& tmap_b2, const GemmArgs& args,
                           cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(Variant<P, DW>::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = cooperative ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, expert_gemm_tc<P, DW, kFused, kPair>, tmap_b, tmap_x, tmap_b2, args);
}

int launch_expert_gemm(const CUtensorMap& tmap_b, const CUtensorMap& tmap_x, const CUtensorMap& tmap_b2,
                       const GemmArgs& args, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return MUSE_ERR_NO_DEVICE;
  if (!g_num_sms[dev]) {
    e = cudaDeviceGetAttribute(&g_num_sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
  }
  if (!g_attr_set[dev]) {
    const void* fns[5] = {(const void*)expert_gemm_tc<2, 4, false, false>,
                          (const void*)expert_gemm_tc<2, 4, true, false>,
                          (const void*)expert_gemm_tc<kDecodePipes, kDecodeDW, false, false>,
                          (const void*)expert_gemm_tc<kDecodePipes, kDecodeDW, true, false>,
                          (const void*)expert_gemm_tc<1, 8, false, true>};
    for (int i = 0; i < 5 && e == cudaSuccess; ++i)
      e = cudaFuncSetAttribute(fns[i], cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    g_attr_set[dev] = true;
  }
  if (args.stages < 2 || args.b_stages < 2 || args.stages > kMaxStages || args.b_stages > kMaxStages)
    return MUSE_ERR_UNSUPPORTED_SHAPE;
  if (args.n_phases < 1 || args.n_phases > 2 || (args.fused && args.n_phases != 2))
    return MUSE_ERR_INVALID_ARGUMENT;
  const bool pair = args.pair_tiles != 0;
  if (pair && (args.fused || args.route_inline || args.n_box != 128)) return MUSE_ERR_INVALID_ARGUMENT;
  const Geo g = make_geo(pipe_cols(pick_pipes(args.n_box, pair)), args.n_box, args.stages, args.b_stages, pair);
  if (g.n_a < 2) return MUSE_ERR_UNSUPPORTED_SHAPE;
  if (args.route_inline &&
      (args.n_pairs > kMaxInlinePairs || args.n_box > kMaxInlineBox || !args.ids || !args.pair_order ||
       !args.pair_row))
    return MUSE_ERR_UNSUPPORTED_SHAPE;
  // a fused launch combines through the inline routing tables and the GEMM2 tile counters
  if (args.fused && (!args.route_inline || !args.ph[1].signal || !args.ph[1].wait_for || !args.out ||
                     !args.topk_weights || args.top_k > kMaxTopK || args.hidden % 128))
    return MUSE_ERR_INVALID_ARGUMENT;
  const size_t smem = gemm_smem_bytes(args.n_box, pair, args.stages, args.b_stages);
  if (smem > 227u * 1024u) return MUSE_ERR_UNSUPPORTED_SHAPE;
  const int grid = g_num_sms[dev];
#ifdef MUSE_TRACE
  if (trace::g_host_buf) {  // this launch's block of the attached stamp buffer
    unsigned long long* p = trace::g_host_buf + (size_t)(trace::g_host_next++ % trace::g_host_slots) * grid *
                                                    trace::kTraceStride;
    e = cudaMemcpyToSymbolAsync(trace::g_trace_buf, &p, sizeof(p), 0, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return e;
  }
#endif
  // A fused launch waits across CTAs (GEMM2 items on GEMM1 tiles, the combine on GEMM2 tiles):
  // it is launched cooperatively, so either every CTA is resident at once or the launch fails.
  const bool decode = args.n_box <= 16;  // the decode variant: kDecodePipes x kDecodeDW
  if (args.fused)
    e = decode ? launch_variant<kDecodePipes, kDecodeDW, true>(grid, smem, true, tmap_b, tmap_x, tmap_b2, args, stream)
               : launch_variant<2, 4, true>(grid, smem, true, tmap_b, tmap_x, tmap_b2, args, stream);
  else if (pair)
    e = launch_variant<1, 8, false, true>(grid, smem, false, tmap_b, tmap_x, tmap_b2, args, stream);
  else
    e = decode ? launch_variant<kDecodePipes, kDecodeDW, false>(grid, smem, false, tmap_b, tmap_x, tmap_b2, args, stream)
               : launch_variant<2, 4, false>(grid, smem, false, tmap_b, tmap_x, tmap_b2, args, stream);
  if (e != cudaSuccess) return e;
  return last_launch_status();
}

}  // namespace muse

#ifdef MUSE_TRACE
// Traced builds only: attach (or, with null, detach) a stamp buffer for the expert GEMM's next
// `launches` launches on the current device, each gridDim.x * kTraceStride u64 values (launch
// i writes block i; later launches wrap around).
extern "C" int muse_moe_trace_attach(void* buf, int launches) {
  muse::trace::g_host_buf = static_cast<unsigned long long*>(buf);
  muse::trace::g_host_slots = launches > 0 ? launches : 1;
  muse::trace::g_host_next = 0;
  unsigned long long* p = nullptr;
  return (int)cudaMemcpyToSymbol(muse::trace::g_trace_buf, &p, sizeof(p));
}
extern "C" int muse_moe_trace_stride(void) { return muse::trace::kTraceStride; }
#endif
