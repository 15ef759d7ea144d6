"""Algorithmic byte and FLOP counts of one layer call and of each expert GEMM launch.

These are the minimum bytes the work has to move, not what the kernels measure: the NVFP4
weights (codes + e4m3 scales) of every distinct local expert that has at least one pair, and
the activations each stage reads or writes once. The whole-call model follows the reference's
speed-of-light byte count (reference.py:125-136) without its routing share.
"""

from __future__ import annotations

import numpy as np

BLOCK = 16  # NVFP4 block size along K (nvfp4.py)


def _pairs_and_experts(topk_ids, local_start: int, local_count: int) -> tuple[int, int]:
    e = np.asarray(topk_ids, dtype=np.int64) - local_start
    local = (e >= 0) & (e < local_count)
    return int(local.sum()), int(np.unique(e[local]).size)


def weight_bytes(rows: int, k: int) -> float:
    """Codes (half a byte per element) plus one e4m3 scale per 16 elements."""
    return rows * k * (0.5 + 1.0 / BLOCK)


def layer_bytes(topk_ids, local_start: int, local_count: int, hidden: int, inter: int) -> int:
    """Weights of the experts hit, x in and out (bf16) and the routing (ids + weights)."""
    t, k = np.asarray(topk_ids).shape
    _, used = _pairs_and_experts(topk_ids, local_start, local_count)
    return int(used * weight_bytes(3 * inter, hidden) + 2 * t * hidden * 2 + t * k * 8)


def layer_flops(topk_ids, local_start: int, local_count: int, hidden: int, inter: int) -> int:
    """2 * pairs * 3 * I * H: GEMM1 (2I x H) and GEMM2 (H x I) for every local pair."""
    pairs, _ = _pairs_and_experts(topk_ids, local_start, local_count)
    return 2 * pairs * 3 * inter * hidden


def gemm1_bytes(topk_ids, local_start: int, local_count: int, hidden: int, inter: int) -> int:
    """GEMM1 launch: w13 of the experts hit, x read once (bf16), the expert ids, and the bf16
    SiLU(gate)*up rows it writes for every local pair."""
    t, k = np.asarray(topk_ids).shape
    pairs, used = _pairs_and_experts(topk_ids, local_start, local_count)
    return int(used * weight_bytes(2 * inter, hidden) + 2 * t * hidden + 4 * t * k + 2 * pairs * inter)


def gemm2_bytes(topk_ids, local_start: int, local_count: int, hidden: int, inter: int) -> int:
    """GEMM2 launch: w2 of the experts hit, the bf16 inter rows, and the fp32 per-pair output
    rows and sums of squares it writes."""
    pairs, used = _pairs_and_experts(topk_ids, local_start, local_count)
    return int(used * weight_bytes(hidden, inter) + 2 * pairs * inter + 4 * pairs * hidden + 4 * pairs)


def gemm1_flops(topk_ids, local_start: int, local_count: int, hidden: int, inter: int) -> int:
    """GEMM1 launch: 2 * pairs * 2I * H."""
    pairs, _ = _pairs_and_experts(topk_ids, local_start, local_count)
    return 2 * pairs * 2 * inter * hidden
