// Expert GEMMs on the 5th-generation tensor cores (tcgen05, sm_100a), swap-AB:
// the weight rows are the MMA's M = 128 side, the tokens of one expert its N side.
//
//   GEMM1 (mode 1): h = xs . W13^T over K = H, epilogue silu(gate) * up -> inter (bf16)
//                   (reference.py:103-104; SGLang keeps inter in bf16, baseline.py:132)
//   GEMM2 (mode 2): y = inter . W2^T over K = I, epilogue y * gs * (1 + post_norm_w) -> ypart
//                   (fp32) and the per-pair sum of squares -> ssq (reference.py:88-90, 105)
//
// One persistent CTA per SM walks a static list of (expert, 128-row tile, token tile) items.
// Warp roles (14 warps):
//   warp 0      producer: 1-D bulk copies of the prepared fp4 code and scale tiles, TMA
//               tiles of the activations (128-byte swizzle) into an S-stage ring
//   warp 1      TMEM allocator and MMA issuer: tcgen05.mma with A in tensor memory, B in
//               shared memory, fp32 accumulators in tensor memory (two buffers)
//   warps 2-5   epilogue: tcgen05.ld of the accumulators, fused activation / norm, stores
//   warps 6-13  dequantisers, two groups of four taking alternate stages: thread = weight
//               row; e2m1 x e4m3 -> exact bf16 in registers, tcgen05.st into an A buffer
// Every mbarrier wait is bounded; on timeout the CTA records an error flag and unwinds.
#include "common.cuh"
#include "kernels.cuh"
#include "layout.cuh"
#include "ptx.cuh"

namespace muse {

namespace {

constexpr int kThreads = 448;
constexpr int kProducerWarp = 0;
constexpr int kMmaWarp = 1;
constexpr int kEpiWarp0 = 2;
constexpr int kDeqWarp0 = 6;
constexpr int kNumABuf = 4;
constexpr int kACols = kChunkK / 2;              // TMEM columns per A buffer (bf16 pairs)
constexpr int kAccCol0 = kNumABuf * kACols;      // 256
constexpr int kAccCols = 128;                    // max token tile (N)
constexpr int kTmemCols = 512;
constexpr int kMaxStages = 8;
constexpr int kMaxExperts = kMaxLocalExperts;
// raw code value = e2m1 * 2^-126; scales held as sf * 2^60; product = e2m1 * sf * 2^-66.
constexpr float kUnscale = 73786976294838206464.0f;  // 2^66

struct SharedCtl {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t a_full[kNumABuf];
  uint64_t a_empty[kNumABuf];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int total_items;
  int item_prefix[kMaxExperts + 1];  // cumulative items per expert
  int ntiles[kMaxExperts];           // token tiles per expert
  uint32_t scale_lut[256];           // e4m3 byte -> bf16x2 (sf * 2^60, sf * 2^60)
};

struct Item {
  int e, m, n, row0, nvalid;
};

__device__ __forceinline__ Item decode_item(const SharedCtl& c, const int32_t* offsets, int it,
                                            int n_local, int m_tiles, int n_box) {
  int lo = 0, hi = n_local;  // find e with prefix[e] <= it < prefix[e+1]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (c.item_prefix[mid] <= it) lo = mid; else hi = mid;
  }
  Item r;
  r.e = lo;
  const int local = it - c.item_prefix[lo];
  const int nt = c.ntiles[lo];
  r.m = local / nt;
  r.n = local - r.m * nt;
  const int begin = offsets[lo], cnt = offsets[lo + 1] - begin;
  r.row0 = begin + r.n * n_box;
  r.nvalid = min(n_box, cnt - r.n * n_box);
  (void)m_tiles;
  return r;
}

// bf16x2 multiply (round to nearest); exact here: both factors have <= 4 significant bits.
__device__ __forceinline__ uint32_t hmul2_bf16(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// One permuted code word (8 elements) -> 4 bf16x2 of e2m1 * sf * 2^-66.
__device__ __forceinline__ void dequant8(uint32_t w, uint32_t scale2, uint32_t* out) {
  constexpr uint32_t kMask = 0x81C081C0u;
  const uint32_t r0 = w & kMask;
  const uint32_t r1 = ptx::rotl(w, 4) & kMask;
  const uint32_t r2 = ptx::rotl(w, 10) & kMask;
  const uint32_t r3 = ((w << 6) & 0x80C080C0u) | ((w >> 2) & 0x01000100u);
  out[0] = hmul2_bf16(r0, scale2);
  out[1] = hmul2_bf16(r1, scale2);
  out[2] = hmul2_bf16(r2, scale2);
  out[3] = hmul2_bf16(r3, scale2);
}

__device__ __forceinline__ void record_error(int* flag, int code) {
  if (flag) atomicExch(flag, code);
}

__global__ void __launch_bounds__(kThreads, 1)
expert_gemm_tc(const __grid_constant__ CUtensorMap tmap_b, const GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;
  const int n_box = a.n_box;
  const uint32_t b_bytes = 2u * n_box * 128u;
  const uint32_t stage_bytes = b_bytes + kTileCodeBytes + kTileScaleBytes;
  SharedCtl& ctl = *reinterpret_cast<SharedCtl*>(smem + (size_t)S * stage_bytes);
  auto b_smem = [&](int s) { return smem + (size_t)s * stage_bytes; };
  auto a_smem = [&](int s) { return smem + (size_t)s * stage_bytes + b_bytes; };
  auto sf_smem = [&](int s) { return smem + (size_t)s * stage_bytes + b_bytes + kTileCodeBytes; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_local = a.n_local;

  // ---- set-up: barriers, scale table, work list, tensor memory
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(&ctl.full[s], 1);
      ptx::mbar_init(&ctl.empty[s], 1 + 4);  // MMA commit + 4 dequant warps
    }
    for (int b = 0; b < kNumABuf; ++b) {
      ptx::mbar_init(&ctl.a_full[b], 4);
      ptx::mbar_init(&ctl.a_empty[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(&ctl.acc_full[b], 1);
      ptx::mbar_init(&ctl.acc_empty[b], 4);
    }
    ptx::mbar_init(&ctl.drain, 1);
    ptx::fence_barrier_init();
  }
  if (warp == kProducerWarp && lane == 0) ptx::prefetch_tensormap(&tmap_b);
  for (int i = threadIdx.x; i < 256; i += kThreads) {
    const float f = e4m3_to_float(i) * 1152921504606846976.0f;  // * 2^60
    const __nv_bfloat16 h = __float2bfloat16_rn(f);
    const uint32_t u = *reinterpret_cast<const uint16_t*>(&h);
    ctl.scale_lut[i] = u | (u << 16);
  }
  // items per expert, exclusive scan by the first 8 warps (n_local <= 256)
  if (threadIdx.x < 256) {
    const int e = threadIdx.x;
    int cnt = 0;
    if (e < n_local) cnt = a.offsets[e + 1] - a.offsets[e];
    const int nt = (cnt + n_box - 1) / n_box;
    const int v = nt * a.m_tiles;
    if (e < n_local) ctl.ntiles[e] = nt;
    int incl = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += o;
    }
    ctl.item_prefix[e + 1] = incl;  // warp-local for now
  }
  if (warp == kMmaWarp) {
    ptx::tmem_alloc(&ctl.tmem_base, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (threadIdx.x == 0) {
    ctl.item_prefix[0] = 0;
    int carry = 0;
    for (int w = 0; w < 8; ++w) {  // add the totals of earlier warps
      const int last = ctl.item_prefix[32 * w + 32];
      for (int i = 1; i <= 32; ++i) ctl.item_prefix[32 * w + i] += carry;
      carry += last;
    }
    ctl.total_items = ctl.item_prefix[n_local];
  }
  __syncthreads();

  const uint32_t tbase = ctl.tmem_base;
  const int total = ctl.total_items;
  bool ok = true;

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------------ producer
    // The whole warp walks the schedule; lane 0 waits and issues.
    int stage = 0;
    uint32_t phase = 0;
    long long issued = 0;
    for (int it = blockIdx.x; it < total && ok; it += gridDim.x) {
      const Item t = decode_item(ctl, a.offsets, it, n_local, a.m_tiles, n_box);
      const size_t tile0 = ((size_t)t.e * a.m_tiles + t.m) * a.k_chunks;
      for (int kc = 0; kc < a.k_chunks; ++kc) {
        int good = 1;
        if (lane == 0) {
          good = ptx::mbar_wait(&ctl.empty[stage], phase ^ 1);
          if (good) {
            ptx::mbar_arrive_expect_tx(&ctl.full[stage], stage_bytes);
            ptx::bulk_g2s(a_smem(stage), a.wq + (tile0 + kc) * kTileCodeBytes, kTileCodeBytes,
                          &ctl.full[stage]);
            ptx::bulk_g2s(sf_smem(stage), a.wsf + (tile0 + kc) * kTileScaleBytes, kTileScaleBytes,
                          &ctl.full[stage]);
            ptx::tma_load_2d(b_smem(stage), &tmap_b, kc * kChunkK, t.row0, &ctl.full[stage]);
            ptx::tma_load_2d(b_smem(stage) + n_box * 128, &tmap_b, kc * kChunkK + 64, t.row0,
                             &ctl.full[stage]);
          }
        }
        if (!__shfl_sync(0xffffffffu, good, 0)) { ok = false; break; }
        ++issued;
        if (++stage == S) { stage = 0; phase ^= 1; }
      }
    }
    if (!ok && lane == 0) {
      record_error(a.error_flag, 1);
      // let copies already in flight land before the CTA can exit
      for (long long i = (issued > S ? issued - S : 0); i < issued; ++i)
        ptx::mbar_wait(&ctl.full[(int)(i % S)], (uint32_t)((i / S) & 1));
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA issuer
    // The whole warp walks the schedule; lane 0 waits and issues (tcgen05.mma is issued by
    // one thread).
    const uint32_t idesc = ptx::idesc_bf16_f32(kTileM, n_box);
    long long c = 0;
    int li = 0;
    for (int it = blockIdx.x; it < total && ok; it += gridDim.x, ++li) {
      const int acc = li & 1;
      int good = 1;
      if (lane == 0) good = ptx::mbar_wait(&ctl.acc_empty[acc], ((li >> 1) & 1) ^ 1);
      if (!__shfl_sync(0xffffffffu, good, 0)) { ok = false; break; }
      ptx::tc_fence_after();
      const uint32_t d_tmem = tbase + kAccCol0 + acc * kAccCols;
      for (int kc = 0; kc < a.k_chunks; ++kc, ++c) {
        const int s = (int)(c % S);
        const int ab = (int)(c % kNumABuf);
        if (lane == 0)
          good = ptx::mbar_wait(&ctl.full[s], (uint32_t)((c / S) & 1)) &&
                 ptx::mbar_wait(&ctl.a_full[ab], (uint32_t)((c / kNumABuf) & 1));
        if (!__shfl_sync(0xffffffffu, good, 0)) { ok = false; break; }
        ptx::tc_fence_after();
        if (lane == 0) {
          const uint32_t b0 = ptx::smem_u32(b_smem(s));
#pragma unroll
          for (int kk = 0; kk < kChunkK / 16; ++kk) {
            const uint64_t bdesc =
                ptx::smem_desc_k_sw128(b0 + (kk >> 2) * n_box * 128 + (kk & 3) * 32, 1024);
            ptx::mma_bf16_ts(d_tmem, tbase + ab * kACols + kk * 8, bdesc, idesc, (kc | kk) != 0);
          }
          ptx::mma_commit(&ctl.empty[s]);
          ptx::mma_commit(&ctl.a_empty[ab]);
        }
        __syncwarp();
      }
      if (!ok) break;
      if (lane == 0) ptx::mma_commit(&ctl.acc_full[acc]);
      __syncwarp();
    }
    if (lane == 0) {
      if (!ok) record_error(a.error_flag, 2);
      // all issued MMAs complete before tensor memory is released
      ptx::mma_commit(&ctl.drain);
      ptx::mbar_wait(&ctl.drain, 0);
    }
    __syncwarp();
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + 4) {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;
    int li = 0;
    for (int it = blockIdx.x; it < total; it += gridDim.x, ++li) {
      const Item t = decode_item(ctl, a.offsets, it, n_local, a.m_tiles, n_box);
      const int acc = li & 1;
      if (!ptx::mbar_wait(&ctl.acc_full[acc], (li >> 1) & 1)) { ok = false; break; }
      ptx::tc_fence_after();
      const uint32_t taddr = tbase + ((uint32_t)(32 * q) << 16) + kAccCol0 + acc * kAccCols;
      const float gsc = a.gs[t.e] * kUnscale;
      if (a.mode == 1) {
        const int j = 64 * t.m + 16 * q + (lane & 15);  // intermediate index of this lane
        for (int cb = 0; cb * 16 < t.nvalid; ++cb) {
          uint32_t v[16];
          ptx::tmem_ld16(taddr + cb * 16, v);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int col = 0; col < 16; ++col) {
            const float mine = __uint_as_float(v[col]) * gsc;
            const float other = __shfl_xor_sync(0xffffffffu, mine, 16);
            const int n = cb * 16 + col;
            if (lane < 16 && n < t.nvalid) {
              const float g = mine, u = other;
              const float act = g / (1.0f + __expf(-g)) * u;
              const __nv_bfloat16 hb = __float2bfloat16_rn(act);
              a.inter[(size_t)(t.row0 + n) * a.ld_out + j] = *reinterpret_cast<const uint16_t*>(&hb);
            }
          }
        }
      } else {
        const int h = kTileM * t.m + 32 * q + lane;  // output row of this lane
        const float wn = gsc * (1.0f + bf16_bits_to_float(a.post_norm_w[h]));
        for (int cb = 0; cb * 16 < t.nvalid; ++cb) {
          uint32_t v[16];
          ptx::tmem_ld16(taddr + cb * 16, v);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int col = 0; col < 16; ++col) {
            const int n = cb * 16 + col;
            if (n < t.nvalid) {  // warp-uniform
              const float y = __uint_as_float(v[col]) * wn;
              a.ypart[(size_t)(t.row0 + n) * a.ld_out + h] = y;
              float s2 = y * y;
#pragma unroll
              for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
              if (lane == 0) atomicAdd(&a.ssq[t.row0 + n], s2);
            }
          }
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&ctl.acc_empty[acc]);
    }
    if (!ok && lane == 0) record_error(a.error_flag, 3);
  } else {
    // ------------------------------------------------------------------ dequantisers
    const int g = (warp - kDeqWarp0) >> 2;   // 0 or 1: even / odd chunks
    const int q = warp & 3;                  // TMEM lane quarter
    const int row = 32 * q + lane;           // weight row of this thread
    const uint32_t lane_addr = (uint32_t)(32 * q) << 16;
    long long c = 0;
    for (int it = blockIdx.x; it < total && ok; it += gridDim.x) {
      for (int kc = 0; kc < a.k_chunks; ++kc, ++c) {
        if ((c & 1) != g) continue;
        const int s = (int)(c % S);
        const int ab = (int)(c % kNumABuf);
        if (!ptx::mbar_wait(&ctl.full[s], (uint32_t)((c / S) & 1)) ||
            !ptx::mbar_wait(&ctl.a_empty[ab], (uint32_t)(((c / kNumABuf) & 1) ^ 1))) {
          ok = false;
          break;
        }
        const uint8_t* arow = a_smem(s) + row * kRowCodeBytes;
        const uint2 sfw = *reinterpret_cast<const uint2*>(sf_smem(s) + row * kRowScaleBytes);
        const uint32_t sfb[2] = {sfw.x, sfw.y};
        uint4 codes[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          codes[j] = *reinterpret_cast<const uint4*>(arow + 16 * code_slot(row, j));
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t out[32];
#pragma unroll
          for (int jj = 0; jj < 2; ++jj) {
            const int j = 2 * half + jj;  // 16-byte chunk = 32 elements = 2 scale blocks
            const uint32_t wv[4] = {codes[j].x, codes[j].y, codes[j].z, codes[j].w};
#pragma unroll
            for (int wd = 0; wd < 4; ++wd) {
              const int blk = 2 * j + (wd >> 1);
              const uint32_t sbyte = (sfb[blk >> 2] >> (8 * (blk & 3))) & 0xFF;
              dequant8(wv[wd], ctl.scale_lut[sbyte], &out[jj * 16 + wd * 4]);
            }
          }
          ptx::tmem_st32(tbase + lane_addr + ab * kACols + half * 32, out);
        }
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          ptx::mbar_arrive(&ctl.a_full[ab]);
          ptx::mbar_arrive(&ctl.empty[s]);
        }
      }
    }
    if (!ok && lane == 0) record_error(a.error_flag, 4);
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == kMmaWarp) ptx::tmem_dealloc(tbase, kTmemCols);
}

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

size_t gemm_smem_bytes(int n_box, int stages) {
  const size_t stage = 2u * n_box * 128u + kTileCodeBytes + kTileScaleBytes;
  return 1024 + stages * stage + sizeof(SharedCtl);
}

int pick_stages(int n_box) {
  const size_t stage = 2u * n_box * 128u + kTileCodeBytes + kTileScaleBytes;
  int s = (int)((200u * 1024u - sizeof(SharedCtl) - 1024) / stage);
  return s < kMaxStages ? s : kMaxStages;
}

int launch_expert_gemm(const CUtensorMap& tmap_b, const GemmArgs& args, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return MUSE_ERR_NO_DEVICE;
  if (!g_num_sms[dev]) {
    e = cudaDeviceGetAttribute(&g_num_sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
  }
  if (!g_attr_set[dev]) {
    e = cudaFuncSetAttribute(expert_gemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    g_attr_set[dev] = true;
  }
  const size_t smem = gemm_smem_bytes(args.n_box, args.stages);
  expert_gemm_tc<<<g_num_sms[dev], kThreads, smem, stream>>>(tmap_b, args);
  return last_launch_status();
}

}  // namespace muse
