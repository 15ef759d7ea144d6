"""CPU oracle for the routed W4A16 MoE layer -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the reference's fp32 dequantise-then-accumulate path
(`reference.py:93-107`, with `nvfp4.py:40-47,90-97` and `checks.py:31-55`). It is the checker
for the CUDA path: only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline /
reference legs import it. The product path (the C-ABI library and its host wrapper) never
imports, calls or falls back to anything here.

Pinning: `tests/golden/make_golden.py` runs the reference's own Python modules on CPU in the
build container and stores their outputs under `tests/golden/`; `tests/test_oracle_golden.py`
checks every function below against those fixtures.

All arrays are numpy. bf16 tensors are carried as their raw uint16 bit patterns, fp8 e4m3
tensors as raw uint8 bytes, so that every byte the GPU sees is the byte the oracle sees.
"""

from __future__ import annotations

import numpy as np

# nvfp4.py:24 -- magnitudes of the 3-bit E2M1 code; bit 3 is the sign (nvfp4.py:40-47).
E2M1_GRID = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
BLOCK = 16                 # nvfp4.py:16, elements per e4m3 block scale
POST_NORM_EPS = 1e-8       # reference.py:24
REL_L2_TOL = 1.5e-2        # reference.py:25
ROW_FACTOR = 5.0           # checks.py:14
ROW_NORM_FLOOR = 0.1       # checks.py:17


def e2m1_table() -> np.ndarray:
    """float32[16]: value of each 4-bit code (sign in bit 3), as nvfp4.unpack_e2m1 decodes it."""
    mag = np.array(E2M1_GRID, dtype=np.float32)
    return np.concatenate([mag, -mag]).astype(np.float32)


def e4m3_table() -> np.ndarray:
    """float32[256]: OCP fp8 e4m3fn decoding of every byte (bias 7, no infinities,
    S.1111.111 is NaN, exponent 0 is subnormal with scale 2^-6)."""
    b = np.arange(256, dtype=np.int64)
    sign = np.where(b >> 7, -1.0, 1.0)
    exp = (b >> 3) & 0xF
    man = (b & 0x7).astype(np.float64)
    val = np.where(exp == 0, man / 8.0 * 2.0 ** -6, (1.0 + man / 8.0) * 2.0 ** (exp - 7))
    val = np.where((exp == 15) & (man == 7), np.nan, val)
    return (sign * val).astype(np.float32)


_E2M1 = e2m1_table()
_E4M3 = e4m3_table()
# float32 [256, 2]: the two values of a packed code byte (low nibble first, nvfp4.py:5-6), so a
# packed row is unpacked by one table lookup per byte
_E2M1_PAIR = np.stack([_E2M1[np.arange(256) & 0x0F], _E2M1[np.arange(256) >> 4]], axis=1)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> uint16 bf16 bits, round to nearest even (torch's `.to(torch.bfloat16)`)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def unpack_e2m1(packed: np.ndarray) -> np.ndarray:
    """uint8 [..., K/2] -> float32 [..., K]; element 2i is the low nibble (nvfp4.py:40-47)."""
    p = np.asarray(packed, dtype=np.uint8)
    return np.take(_E2M1_PAIR, p, axis=0).reshape(p.shape[:-1] + (p.shape[-1] * 2,))


def dequantize(packed: np.ndarray, sf: np.ndarray, gs: float | np.floating) -> np.ndarray:
    """Restates nvfp4.dequantize (nvfp4.py:90-97): e2m1 * (float(sf) * gs), all in float32.
    The block scale and the global scale are multiplied first, as the reference does."""
    vals = unpack_e2m1(packed)
    k = vals.shape[-1]
    scale = _E4M3[np.asarray(sf, dtype=np.uint8)] * np.float32(gs)
    out = vals.reshape(vals.shape[:-1] + (k // BLOCK, BLOCK)) * scale[..., None]
    return out.reshape(vals.shape).astype(np.float32, copy=False)


def silu(x: np.ndarray) -> np.ndarray:
    return x / (np.float32(1.0) + np.exp(-x))


def post_expert_norm(y: np.ndarray, w_bits: np.ndarray) -> np.ndarray:
    """reference.py:88-90: y * (1 + w), then RMS-normalise the row with eps 1e-8 (fp32)."""
    y = y.astype(np.float32) * (np.float32(1.0) + bf16_to_f32(w_bits))
    ms = np.mean(y * y, axis=-1, keepdims=True, dtype=np.float32)
    return y / np.sqrt(ms + np.float32(POST_NORM_EPS))


def route(topk_ids: np.ndarray, local_start: int, local_count: int):
    """Token -> local-expert grouping, the order `ref_kernel` visits pairs in
    (reference.py:99-102: ascending expert, then `(ids == e).nonzero()` row-major order).

    Returns (offsets int32[local_count + 1], pair_order int32[P], pair_row int32[T*K]):
    pair_order[r] is the flat index t*K + s of the r-th pair; pair_row is its inverse
    (-1 for a pair whose expert is not local). This is a stable sort by expert, and the
    CUDA routing kernel must reproduce it bit for bit."""
    ids = np.asarray(topk_ids, dtype=np.int64).reshape(-1)
    e = ids - local_start
    local = (e >= 0) & (e < local_count)
    flat = np.nonzero(local)[0]
    order = np.argsort(e[flat], kind="stable")
    pair_order = flat[order].astype(np.int32)
    counts = np.bincount(e[flat], minlength=local_count)
    offsets = np.zeros(local_count + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(counts)
    pair_row = np.full(ids.shape[0], -1, dtype=np.int32)
    pair_row[pair_order] = np.arange(pair_order.shape[0], dtype=np.int32)
    return offsets, pair_order, pair_row


def router_topk(scores: np.ndarray, top_k: int, mode: str = "renorm"):
    """The routing step of reference.generate_input (reference.py:72-84): for each token the
    top_k scores in descending order (equal scores: lower expert id first; NaN above every
    number, torch.topk's order), ids int32 [T, K], and weights fp32 [T, K]: the selected scores
    over their sum ("renorm", reference.py:82), or their softmax ("softmax": the synthetic
    configs' logits -> softmax -> top-K -> renormalise). Sums run in selection order."""
    s = np.asarray(scores, dtype=np.float32)
    T, E = s.shape
    ids = np.zeros((T, top_k), dtype=np.int32)
    wts = np.zeros((T, top_k), dtype=np.float32)
    for t in range(T):
        row = s[t]
        # sort key: NaN first, then descending value, then ascending id
        order = sorted(range(E), key=lambda e: (0 if np.isnan(row[e]) else 1,
                                                0.0 if np.isnan(row[e]) else -float(row[e]), e))
        sel = order[:top_k]
        ids[t] = sel
        v = row[sel].astype(np.float32)
        if mode == "renorm":
            total = np.float32(0.0)
            for x in v:
                total = np.float32(total + x)
            wts[t] = v / total
        else:
            ex = np.exp((v - v[0]).astype(np.float32)).astype(np.float32)
            total = np.float32(0.0)
            for x in ex:
                total = np.float32(total + x)
            wts[t] = ex / total
    return ids, wts


def ref_kernel(x_bits, topk_ids, topk_weights, weights: dict, local_start: int, local_count: int,
               d_expert: int, return_f32: bool = False):
    """Restates reference.ref_kernel (reference.py:93-107) for any shape.

    x_bits: uint16 [T, H] (bf16 bits). topk_ids: int32 [T, K] global ids. topk_weights:
    float32 [T, K]. weights: w13 u8 [E, 2I, H/2], w13_sf u8 [E, 2I, H/16], w13_gs f32 [E],
    w2 u8 [E, H, I/2], w2_sf u8 [E, H, I/16], w2_gs f32 [E], post_norm_w u16 [H]; indexed
    by GLOBAL expert id. Returns uint16 bf16 bits [T, H] (or the float32 sum before the cast)."""
    x = bf16_to_f32(x_bits)
    ids = np.asarray(topk_ids, dtype=np.int64)
    wts = np.asarray(topk_weights, dtype=np.float32)
    out = np.zeros(x.shape, dtype=np.float32)
    lo, hi = local_start, local_start + local_count
    for e in np.unique(ids).tolist():
        if not lo <= e < hi:
            continue
        tok, slot = np.nonzero(ids == e)
        w13 = dequantize(weights["w13"][e], weights["w13_sf"][e], weights["w13_gs"][e])
        h = x[tok] @ w13.T
        inter = silu(h[:, :d_expert]) * h[:, d_expert:]
        w2 = dequantize(weights["w2"][e], weights["w2_sf"][e], weights["w2_gs"][e])
        y = inter @ w2.T
        contrib = post_expert_norm(y, weights["post_norm_w"]) * wts[tok, slot][:, None]
        _add_rows(out, tok, contrib)
    if return_f32:
        return out
    return f32_to_bf16(out)


def ref_kernel_threads(x_bits, topk_ids, topk_weights, weights: dict, local_start: int,
                       local_count: int, d_expert: int, threads: int = 1):
    """ref_kernel with the per-expert work (dequantise, two GEMMs, norm) spread over a thread
    pool; numpy releases the GIL inside those operations. Contributions are added in ascending
    expert order afterwards, so the result equals ref_kernel's bit for bit. This is the CPU
    baseline timed by bench.py (all host cores)."""
    from concurrent.futures import ThreadPoolExecutor

    x = bf16_to_f32(x_bits)
    ids = np.asarray(topk_ids, dtype=np.int64)
    wts = np.asarray(topk_weights, dtype=np.float32)
    lo, hi = local_start, local_start + local_count
    experts = [e for e in np.unique(ids).tolist() if lo <= e < hi]

    def one(e):
        tok, slot = np.nonzero(ids == e)
        w13 = dequantize(weights["w13"][e], weights["w13_sf"][e], weights["w13_gs"][e])
        h = x[tok] @ w13.T
        inter = silu(h[:, :d_expert]) * h[:, d_expert:]
        w2 = dequantize(weights["w2"][e], weights["w2_sf"][e], weights["w2_gs"][e])
        y = inter @ w2.T
        return tok, post_expert_norm(y, weights["post_norm_w"]) * wts[tok, slot][:, None]

    out = np.zeros(x.shape, dtype=np.float32)
    with ThreadPoolExecutor(max_workers=max(1, threads)) as ex:
        for tok, contrib in ex.map(one, experts):
            _add_rows(out, tok, contrib)
    return f32_to_bf16(out)


def _add_rows(out: np.ndarray, tok: np.ndarray, contrib: np.ndarray) -> None:
    """out[tok[i]] += contrib[i] in fp32, as index_add_ does (reference.py:106). A token meets an
    expert at most once when its top-k ids are distinct, and then one indexed add is the same
    arithmetic as np.add.at; repeated ids fall back to it."""
    if tok.size and np.unique(tok).size == tok.size:
        out[tok] += contrib
    else:
        np.add.at(out, tok, contrib)


def compare(out_bits: np.ndarray, ref_bits: np.ndarray, tol: float = REL_L2_TOL):
    """Restates checks.compare (checks.py:31-55) on bf16 bit patterns.
    Returns (ok, message, rel_l2, worst_row_err)."""
    out = bf16_to_f32(out_bits).astype(np.float64)
    ref = bf16_to_f32(ref_bits).astype(np.float64)
    if out.shape != ref.shape:
        return False, f"expected {ref.shape}, got {out.shape}", np.inf, np.inf
    if not np.isfinite(out).all():
        return False, "output contains NaN or Inf", np.inf, np.inf
    diff = out - ref
    err = float(np.linalg.norm(diff) / max(np.linalg.norm(ref), 1e-12))
    rows_diff = np.linalg.norm(diff.reshape(-1, ref.shape[-1]), axis=-1)
    rows_ref = np.linalg.norm(ref.reshape(-1, ref.shape[-1]), axis=-1)
    floor = max(ROW_NORM_FLOOR * rows_ref.mean(), 1e-12) if rows_ref.size else 1e-12
    row_err = rows_diff / np.maximum(rows_ref, floor)
    worst = float(row_err.max()) if row_err.size else 0.0
    if err > tol:
        return False, f"relative L2 error {err:.3e} > {tol:g}", err, worst
    if worst > ROW_FACTOR * tol:
        return False, f"relative L2 error {err:.3e}, worst row {worst:.3e} > {ROW_FACTOR:g} x {tol:g}", err, worst
    return True, f"relative L2 error {err:.3e} (worst row {worst:.3e})", err, worst


def algorithmic_bytes(topk_ids, local_start: int, local_count: int, hidden: int, inter: int) -> int:
    """Bytes one layer call must move at minimum: the NVFP4 weights (codes + e4m3 scales) of every
    distinct local expert hit, plus x in and out in bf16 and the routing (the byte model of
    reference.py:125-136 without its 0.75 routing share)."""
    ids = np.asarray(topk_ids, dtype=np.int64)
    e = ids - local_start
    used = np.unique(e[(e >= 0) & (e < local_count)]).size
    t, k = ids.shape
    return int(used * 3 * inter * hidden * (0.5 + 1.0 / BLOCK) + 2 * t * hidden * 2 + t * k * 8)


def algorithmic_flops(topk_ids, local_start: int, local_count: int, hidden: int, inter: int) -> int:
    """2 * pairs * 3 * I * H: GEMM1 (2I x H) and GEMM2 (H x I) for every local (token, slot) pair."""
    ids = np.asarray(topk_ids, dtype=np.int64)
    e = ids - local_start
    pairs = int(((e >= 0) & (e < local_count)).sum())
    return 2 * pairs * 3 * inter * hidden
