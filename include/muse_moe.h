/*
 * muse_moe.h -- C ABI of the B200 (sm_100a) routed W4A16 MoE layer.
 *
 * Plain pointers, sizes and a cudaStream_t; no torch types. Every device pointer is a
 * global-memory address on the current device; every call is asynchronous on `stream`,
 * allocates nothing, never synchronises the host and can be captured in a CUDA graph
 * (after the first call on a device, which sets kernel attributes).
 *
 * Tensor conventions (the reference's Weights / Inputs, baseline.py:27-52):
 *   x            bf16  [T, H]              hidden states, row-major
 *   topk_ids     int32 [T, K]              GLOBAL expert ids
 *   topk_weights fp32  [T, K]
 *   w13          u8    [E, 2I, H/2]        E2M1 codes, element 2i in the low nibble;
 *                                          rows [0, I) gate, [I, 2I) up
 *   w13_sf       u8    [E, 2I, H/16]       fp8 e4m3fn block scales (raw bytes)
 *   w13_gs       fp32  [E]                 global scales
 *   w2 / w2_sf / w2_gs   [E, H, I/2] / [E, H, I/16] / [E]
 *   post_norm_w  bf16  [H]                 the post-expert RMSNorm weight (applied as 1 + w)
 *   out          bf16  [T, H]
 * "Prepared" weights are the output of muse_moe_prepare_weights: the same bytes in the
 * kernels' tile order, same total size (a lossless repack).
 *
 * Return value of every entry point: 0 on success, a positive cudaError_t code when a CUDA
 * call or launch failed, or one of the negative MUSE_ERR_* codes below.
 */
#ifndef MUSE_MOE_H_
#define MUSE_MOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* muse_stream_t; /* == cudaStream_t */

#define MUSE_OK                      0
#define MUSE_ERR_INVALID_ARGUMENT   (-1)  /* null pointer, negative size, inconsistent dims   */
#define MUSE_ERR_UNSUPPORTED_SHAPE  (-2)  /* H or I not a multiple of 128, K > 16, E_l > 256  */
#define MUSE_ERR_WORKSPACE_TOO_SMALL (-3) /* workspace smaller than muse_moe_workspace_size   */
#define MUSE_ERR_NO_DEVICE          (-4)  /* no sm_100 device current                          */
#define MUSE_ERR_DEVICE_TIMEOUT     (-5)  /* a bounded device-side wait expired                */
#define MUSE_ERR_SCRATCH_LIMIT      (-6)  /* muse_moe_forward_noalloc: needs > its 32 MiB      */

/* Library version, (major << 16) | minor. */
int muse_moe_version(void);

/* Human-readable text for a return code (static storage). */
const char* muse_moe_error_string(int code);

/*
 * Bytes of scratch memory muse_moe_forward needs for `tokens` tokens. Replaces the
 * per-call torch.empty caches of baseline.py:132-135 (cache1/cache2/cache3) and the
 * moe_align_block_size outputs of baseline.py:129-130.
 */
int muse_moe_workspace_size(int tokens, int top_k, int local_count, int hidden, int inter,
                            size_t* bytes);

/*
 * Byte offsets of the scratch buffers inside the workspace, for inspection by tests:
 * offsets[0..8] = expert_offsets, pair_order, pair_row, xs (bf16 [T*K, H] gathered hidden
 * states), inter (bf16 [T*K, I]), ypart (fp32 [T*K, H]), ssq (fp32 [T*K, H/32]: the sum of
 * squares of each 32-column slice of a ypart row), sync (int32 token-tile counters of the
 * single-launch path, zeroed by each call), total bytes.
 * Rows of xs / inter / ypart / ssq are in pair_order order.
 */
int muse_moe_workspace_offsets(int tokens, int top_k, int local_count, int hidden, int inter,
                               size_t* offsets);

/*
 * Sticky per-device status word of the kernels' bounded waits: 0, or the code of the last
 * failure (then a call returned garbage): 1-4 a wait of the expert GEMM's producer / MMA /
 * epilogue / dequantiser role expired, 5 the single launch's combine waited in vain for its
 * rows, 6 an expert-parallel exchange waited in vain for a peer, 7 an exchange found the
 * device's generation parity different from the caller's. Synchronous: copies from the device
 * on the current device; reset != 0 clears it. Not for use inside a captured graph.
 */
int muse_moe_device_status(int* status, int reset);

/*
 * Lossless repack of `n_experts` experts into the kernels' tile order (same byte counts).
 * Replaces prepare() (baseline.py:82-103; the reference's own repack, submission_v6.py:
 * 138-246). Inputs and outputs are device buffers; sizes as in the conventions above.
 */
int muse_moe_prepare_weights(const uint8_t* w13, const uint8_t* w13_sf,
                             const uint8_t* w2, const uint8_t* w2_sf,
                             int n_experts, int hidden, int inter,
                             uint8_t* w13_out, uint8_t* w13_sf_out,
                             uint8_t* w2_out, uint8_t* w2_sf_out, muse_stream_t stream);

/*
 * Token -> local-expert grouping. Replaces moe_align_block_size (baseline.py:121-130) and the
 * unique/nonzero loop of ref_kernel (reference.py:99-102). For the local experts
 * [local_start, local_start + local_count):
 *   expert_offsets int32[local_count + 1]  exclusive prefix of the per-expert pair counts
 *   pair_order     int32[tokens * top_k]   flat pair index t*K+s, grouped by expert, and in
 *                                          ascending flat order within an expert (stable);
 *                                          entries past expert_offsets[local_count] are -1
 *   pair_row       int32[tokens * top_k]   inverse of pair_order, -1 for non-local pairs
 * Bit-exact with a stable sort by expert.
 */
int muse_moe_route(const int32_t* topk_ids, int tokens, int top_k, int local_start,
                   int local_count, int32_t* expert_offsets, int32_t* pair_order,
                   int32_t* pair_row, muse_stream_t stream);

/*
 * Router top-k, the caller side of the layer: topk_ids / topk_weights for every token from a
 * row-major fp32 score matrix [tokens, n_experts], on the device (so a model step can stay in
 * one graph). Replaces the routing of reference.generate_input (reference.py:72-84):
 * scores.topk(K) -> ids in descending score order (equal scores: lower id first; NaN ranks
 * above every number, as torch.topk orders it), and
 *   mode 0: weights = selected scores / their sum          (the reference's renormalisation)
 *   mode 1: weights = softmax over the K selected scores   (logits -> softmax -> top-K ->
 *                                                            renormalise, the same values)
 * top_k <= 16, top_k <= n_experts <= 1024.
 */
int muse_moe_router_topk(const float* scores, int tokens, int n_experts, int top_k, int mode,
                         int32_t* topk_ids, float* topk_weights, muse_stream_t stream);

/*
 * The whole routed-expert layer call: routing, GEMM1 (w13) with SiLU(gate)*up, GEMM2 (w2),
 * post-expert RMSNorm (eps 1e-8) and the top-k-weighted combine, written as bf16 into `out`.
 * Tokens with no local pair get zeros. Replaces kernel_fn (baseline.py:106-151) and computes
 * ref_kernel's function (reference.py:93-107).
 *   w13p/w13_sfp/w2p/w2_sfp  prepared weights of the LOCAL experts (expert local_start first)
 *   w13_gs/w2_gs             fp32[local_count] global scales of the local experts
 *   workspace                >= muse_moe_workspace_size(...) bytes, 256-byte aligned
 */
int muse_moe_forward(const void* x, const int32_t* topk_ids, const float* topk_weights,
                     int tokens, int top_k, int local_start, int local_count,
                     int hidden, int inter,
                     const uint8_t* w13p, const uint8_t* w13_sfp, const float* w13_gs,
                     const uint8_t* w2p, const uint8_t* w2_sfp, const float* w2_gs,
                     const void* post_norm_w, void* out,
                     void* workspace, size_t workspace_bytes, muse_stream_t stream);

/*
 * muse_moe_forward with every option in one call:
 *   n_experts     experts in the whole model (the reference's Config n_experts, baseline.py:
 *                 37-44); local_count of them are computed here. The batch's pairs spread over
 *                 all n_experts, so a local expert expects T*K / n_experts of them: the token
 *                 tile, and with it the kernels' pipeline layout, is chosen from that (on an
 *                 expert-parallel slice T*K / local_count would overstate it R-fold). 0 means
 *                 local_count (what muse_moe_forward assumes). Results do not depend on it.
 *   out_f32       0: out is bf16 [T, H] (muse_moe_forward); 1: out is the fp32 sum before the
 *                 cast (muse_moe_forward_partial).
 *   stage_events  NULL, or five CUDA events recorded as in muse_moe_forward_profiled.
 * Replaces kernel_fn (baseline.py:106-151), like muse_moe_forward.
 */
int muse_moe_forward_ex(const void* x, const int32_t* topk_ids, const float* topk_weights,
                        int tokens, int top_k, int local_start, int local_count, int n_experts,
                        int hidden, int inter,
                        const uint8_t* w13p, const uint8_t* w13_sfp, const float* w13_gs,
                        const uint8_t* w2p, const uint8_t* w2_sfp, const float* w2_gs,
                        const void* post_norm_w, void* out, int out_f32,
                        void* workspace, size_t workspace_bytes, muse_stream_t stream,
                        void* const* stage_events);

/*
 * One expert-parallel rank's share of the layer: muse_moe_forward for the local experts
 * [local_start, local_start + local_count), but `out_f32` (fp32 [T, H]) receives the fp32 sum
 * over this rank's local slots of topk_weight * norm(y), before any bf16 rounding (zeros for
 * tokens with no local pair). Summing out_f32 over all ranks and casting to bf16
 * (muse_moe_cast_bf16) gives muse_moe_forward's output for the whole expert range. Replaces the
 * per-GPU part of the reference's ep8 layer (reference.py:18-22, TASK.md:29: each GPU computes
 * only its local experts' pairs); the cross-rank sum is the caller's collective.
 */
int muse_moe_forward_partial(const void* x, const int32_t* topk_ids, const float* topk_weights,
                             int tokens, int top_k, int local_start, int local_count,
                             int hidden, int inter,
                             const uint8_t* w13p, const uint8_t* w13_sfp, const float* w13_gs,
                             const uint8_t* w2p, const uint8_t* w2_sfp, const float* w2_gs,
                             const void* post_norm_w, float* out_f32,
                             void* workspace, size_t workspace_bytes, muse_stream_t stream);

/*
 * out[i] = bf16(in[i]) (round to nearest even) for n fp32 values; n a multiple of 8, both
 * pointers 16-byte aligned. The final cast of an expert-parallel layer's summed partials
 * (reference.py:107, the bf16 cast of the fp32 accumulator).
 */
int muse_moe_cast_bf16(const float* in, void* out, size_t n, muse_stream_t stream);

/*
 * The decode-layout exchange of an expert-parallel layer over NVLink peer memory:
 * out (bf16 [n], this rank) = sum over ranks r = 0 .. ranks-1, in that order, of rank r's share
 * (fp32 [n], its muse_moe_forward_partial output). shares0[r] / shares1[r] are rank r's two
 * share buffers and flags[r] its flag array (32 uint32, zero before the first call), all as
 * device addresses valid on this GPU (peer mappings of every rank's symmetric buffers, this
 * rank's own included). The call's generation g = 1, 2, 3, ... is counted on the device (so a
 * captured graph stays valid); call g reads the buffers of parity g & 1, so the caller writes
 * its share of the g-th call into shares{g & 1}[rank]. Waits for the peers are bounded (1 s);
 * on expiry muse_moe_device_status reports 6 (see muse_moe_peer_exchange_bf16 for what a
 * failure leaves behind). muse_moe_peer_exchange_bf16 in mode 0, without a parity check.
 * Replaces the all-reduce that sums the ep8 ranks' partial outputs (reference.py:18-22,
 * TASK.md:29 run one rank per GPU).
 */
int muse_moe_peer_allreduce_bf16(const uint64_t* shares0, const uint64_t* shares1,
                                 const uint64_t* flags, int ranks, int rank, size_t n, void* out,
                                 muse_stream_t stream);

/*
 * The expert-parallel exchange with every option (the two calls below are shorthands for it).
 * Sums the ranks' fp32 shares (shares0[r] / shares1[r], each of n elements, rank r's muse_moe_
 * forward_partial output; parity g & 1 for the g-th call) in rank order, casts to bf16, and:
 *   mode 0  all-reduce, one round: every rank reads every rank's whole share (R * n fp32 over
 *           NVLink per rank) -- fewest synchronisations, for small shares;
 *   mode 1  reduce-scatter: out (bf16 [n / ranks]) = this rank's slice of the sum (n a multiple
 *           of 8 * ranks);
 *   mode 2  all-reduce, two rounds: each rank sums only its 1/R slice (reads R * n / R fp32),
 *           writes it to out and to its bf16 staging buffer staging[r] (n bf16, symmetric like the
 *           shares), and after a second round of flags copies every other rank's slice from that
 *           rank's staging buffer (n bf16 in all): the reduce-scatter + all-gather of the decode
 *           exchange, for large shares. Launched cooperatively.
 * flags[r]: rank r's flag array, 32 uint32, zero before the first call (and again before reuse
 * after a failure). expect_parity: 0 or 1 = the parity of the buffer the caller wrote this call's
 * share into; if the device's generation disagrees the call does nothing and the device status
 * becomes 7. -1 skips the check. timeout_us bounds every wait for the peers (0 = 1 s); on expiry
 * the device status becomes 6, the output is unspecified and the generation is not advanced --
 * the ranks are then out of step and the flag arrays must be re-created (zeroed, then a barrier
 * of all ranks) before the next call. All ranks produce identical bits. Replaces the all-reduce
 * (decode) or reduce-scatter (prefill) that sums the ep ranks' partial outputs
 * (reference.py:18-22, TASK.md:29: one rank per GPU).
 */
int muse_moe_peer_exchange_bf16(const uint64_t* shares0, const uint64_t* shares1,
                                const uint64_t* flags, const uint64_t* staging, int ranks, int rank,
                                size_t n, int mode, int expect_parity, long long timeout_us,
                                void* out, muse_stream_t stream);

/*
 * One expert-parallel decode call of this rank, layer and exchange together: this rank's fp32
 * share of the layer (its local experts, as muse_moe_forward_partial; n_experts as in
 * muse_moe_forward_ex) is written into its share buffer of the call's parity,
 * (expect_parity ? shares1 : shares0)[rank], and every rank's share is then summed into bf16
 * `out` [tokens, hidden] exactly as muse_moe_peer_exchange_bf16 does in `mode` (0 or 2), with
 * the same buffers, flags, generation count, parity check and wait limit. When the layer is a
 * single cooperative launch (small batches; muse_moe_launch_plan_ex path 2), mode is 0 and at
 * most two ranks take part (measured faster there; slower from four), the exchange runs inside
 * that launch after its combine -- its last block to finish the combine
 * signals the peers, every block waits for them and sums its part -- so the call is one
 * launch; otherwise it is the layer's launches followed by the exchange kernel. The output bits
 * are the same either way. expect_parity must be 0 or 1 (it names the share buffer). Replaces
 * the ep8 rank's layer plus the all-reduce of the ranks' partial outputs (reference.py:18-22,
 * TASK.md:29).
 */
int muse_moe_forward_exchange_bf16(const void* x, const int32_t* topk_ids, const float* topk_weights,
                                   int tokens, int top_k, int local_start, int local_count,
                                   int n_experts, int hidden, int inter, const uint8_t* w13p,
                                   const uint8_t* w13_sfp, const float* w13_gs, const uint8_t* w2p,
                                   const uint8_t* w2_sfp, const float* w2_gs, const void* post_norm_w,
                                   void* workspace, size_t workspace_bytes, const uint64_t* shares0,
                                   const uint64_t* shares1, const uint64_t* flags,
                                   const uint64_t* staging, int ranks, int rank, int mode,
                                   int expect_parity, long long timeout_us, void* out,
                                   muse_stream_t stream);

/*
 * The prefill-layout exchange (tokens split over the ranks, ranks x n_per_rank elements in every
 * share): out (bf16 [n_per_rank], this rank) = sum over ranks r, in order, of elements
 * [rank * n_per_rank, (rank + 1) * n_per_rank) of rank r's share -- this rank's tokens. Same
 * buffers, flags, generation count and bounded waits as muse_moe_peer_allreduce_bf16 (the two
 * calls share one generation sequence); muse_moe_peer_exchange_bf16 in mode 1. Replaces the reduce-scatter that returns each rank the
 * sum for its own tokens (reference.py:18-22, TASK.md:29).
 */
int muse_moe_peer_reduce_scatter_bf16(const uint64_t* shares0, const uint64_t* shares1,
                                      const uint64_t* flags, int ranks, int rank, size_t n_per_rank,
                                      void* out, muse_stream_t stream);

/*
 * Prefill dispatch (tokens split over the ranks, tokens_per_rank = T_r on every rank): sends row
 * t of this rank's x (bf16 [T_r, hidden]) to slot rank * T_r + t of rank d's receive buffer
 * recv_x[d] (bf16 [ranks * T_r, hidden]) only when d owns one of the token's experts (rank d owns
 * global expert ids [expert_start[d], expert_start[d + 1])), and the token's ids and weights to
 * the same slot of every rank's recv_ids[d] / recv_weights[d] ([ranks * T_r, top_k]; the other
 * ranks route it nowhere). masks (this rank's memory, uint32 [T_r]) receives each token's
 * destination ranks as a bit mask, for muse_moe_peer_routed_reduce_scatter_bf16. The kernel
 * then signals every rank and waits, bounded by timeout_us (0 = 1 s; expiry: device status 6),
 * for all ranks' dispatch of the same generation, so this rank's receive buffers are complete
 * when it finishes; then run muse_moe_forward_partial on them (ranks * T_r rows) and the routed
 * reduce-scatter. Receive buffers and flags are peer mappings as for the exchange (flags: the
 * same 32-word arrays; the generation is the exchange's). Replaces the all-gather of every
 * token to every rank before the ep ranks' partial layers (reference.py:18-22, TASK.md:29).
 */
int muse_moe_ep_dispatch(const void* x, const int32_t* topk_ids, const float* topk_weights,
                         int tokens_per_rank, int top_k, int hidden, int ranks, int rank,
                         const int* expert_start, const uint64_t* recv_x, const uint64_t* recv_ids,
                         const uint64_t* recv_weights, const uint64_t* flags, uint32_t* masks,
                         long long timeout_us, muse_stream_t stream);

/*
 * The prefill exchange after muse_moe_ep_dispatch: out (bf16 [T_r, hidden], this rank) = for each
 * of this rank's tokens t, the sum over the ranks in masks[t], in rank order, of row
 * rank * T_r + t of their shares (fp32 [ranks * T_r, hidden], parity g & 1 as for the exchange).
 * A rank whose experts the token does not use holds zeros in that row, so the result equals the
 * full sum, but only the rows of the token's destination ranks cross NVLink.
 * muse_moe_peer_exchange_bf16's flags, generation, parity check and bounded waits. Replaces the
 * reduce-scatter of the ep ranks' partial outputs (reference.py:18-22, TASK.md:29).
 */
int muse_moe_peer_routed_reduce_scatter_bf16(const uint64_t* shares0, const uint64_t* shares1,
                                             const uint64_t* flags, int ranks, int rank,
                                             int tokens_per_rank, int hidden, const uint32_t* masks,
                                             int expect_parity, long long timeout_us, void* out,
                                             muse_stream_t stream);

/*
 * muse_moe_forward, with five caller-created CUDA events (cudaEvent_t, passed as void*)
 * recorded on `stream` around the kernels: [0] start, [1] before GEMM1, [2] after GEMM1,
 * [3] after GEMM2, [4] after the combine. For per-kernel timing; same results as
 * muse_moe_forward. No counterpart in the reference (which times whole kernel_fn calls);
 * it replaces nothing.
 */
int muse_moe_forward_profiled(const void* x, const int32_t* topk_ids, const float* topk_weights,
                              int tokens, int top_k, int local_start, int local_count,
                              int hidden, int inter,
                              const uint8_t* w13p, const uint8_t* w13_sfp, const float* w13_gs,
                              const uint8_t* w2p, const uint8_t* w2_sfp, const float* w2_gs,
                              const void* post_norm_w, void* out,
                              void* workspace, size_t workspace_bytes, muse_stream_t stream,
                              void* const* stage_events);

/*
 * The launch plan of one muse_moe_forward call for these shapes (host only, no device work):
 *   plan[0] kernels launched (1, 3 or 5, by plan[3]; 0 if T = 0)
 *   plan[1] token tile (the MMA's N), plan[2] pipeline stages,
 *   plan[3] 2: the whole layer in one cooperative launch after a memset of its counters
 *              (T*K <= 128 and token tile <= 32); 1: GEMM1 routes and gathers x in its own
 *              prologue, then GEMM2 and the combine (T*K <= 1024, token tile <= 32);
 *           0: route, gather, GEMM1, GEMM2, combine;
 *   plan[4] 1 if the expert GEMMs run pair-tile items (each dequantised weight chunk feeds two
 *           128-token tiles; prefill batches averaging >= 128 pairs per local expert), else 0.
 * plan has room for 5 ints. No counterpart in the reference; a diagnostic for benchmarks and
 * tests.
 */
int muse_moe_launch_plan(int tokens, int top_k, int local_count, int hidden, int inter,
                         int* plan);

/* muse_moe_launch_plan for a call of muse_moe_forward_ex with n_experts (0 = local_count). */
int muse_moe_launch_plan_ex(int tokens, int top_k, int local_count, int n_experts, int hidden,
                            int inter, int* plan);

/*
 * muse_moe_forward without a workspace argument: it allocates nothing and takes its scratch
 * from a fixed 32 MiB array in device global memory that the library owns. For callers that
 * cannot allocate device memory -- code running inside another runtime's execution callback
 * (an inference server's plugin or custom-op hook) whose host framework owns all device
 * allocations, or a serving loop that must not call cudaMalloc/cudaFree because they can
 * synchronise the device. No counterpart in the reference (its kernel_fn allocates through
 * torch); it replaces nothing.
 *   - Calls needing more than 32 MiB of scratch (muse_moe_workspace_size) are refused with
 *     MUSE_ERR_SCRATCH_LIMIT before any launch; decode-sized batches fit (top-8: up to 87
 *     tokens at H = 7168, I = 2048; up to 297 at H = 2048, I = 768).
 *   - A device holds the 32 MiB from the first call on it until the process exits. Every call
 *     looks the array's device address up on the current device (so a device reset, which may
 *     move it, is followed); a call made while its stream is being captured reuses the address
 *     of the last call on that device, so make one call on the device before capturing (a first
 *     call inside a capture returns MUSE_ERR_INVALID_ARGUMENT), and capture again after a reset.
 *   - All calls on a device share the array and it keeps the last call's contents. Nothing in
 *     it needs to start at zero (every value a call reads, the same call wrote first), but
 *     calls that overlap on the GPU race on it: serialise them.
 * Same results as muse_moe_forward.
 */
int muse_moe_forward_noalloc(const void* x, const int32_t* topk_ids, const float* topk_weights,
                             int tokens, int top_k, int local_start, int local_count,
                             int hidden, int inter,
                             const uint8_t* w13p, const uint8_t* w13_sfp, const float* w13_gs,
                             const uint8_t* w2p, const uint8_t* w2_sfp, const float* w2_gs,
                             const void* post_norm_w, void* out, muse_stream_t stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* MUSE_MOE_H_ */
