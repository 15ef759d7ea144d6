"""Helpers shared by the GPU parity tests: move seeded CPU inputs to the device and run the
oracle on the very same bytes."""

from __future__ import annotations

import numpy as np
import torch

from oracle import moe_oracle as orc


def to_numpy_weights(w: dict) -> dict:
    out = {}
    for k, v in w.items():
        v = v.detach().cpu()
        if v.dtype == torch.float8_e4m3fn:
            v = v.view(torch.uint8)
        elif v.dtype == torch.bfloat16:
            v = v.view(torch.uint16)
        out[k] = v.numpy()
    return out


def to_device(d: dict, dev) -> dict:
    return {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in d.items()}


def oracle_out(data: dict, w_np: dict, rows=None) -> np.ndarray:
    """Oracle output (bf16 bits) for the given CPU inputs; `rows` restricts it to some tokens."""
    cfg = data["config"]
    x = data["hidden_states"].cpu().view(torch.uint16).numpy()
    ids = data["topk_ids"].cpu().numpy()
    wts = data["topk_weights"].cpu().numpy()
    if rows is not None:
        x, ids, wts = x[rows], ids[rows], wts[rows]
    return orc.ref_kernel(x, ids, wts, w_np, cfg["local_start"], cfg["local_count"], cfg["d_expert"])


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.uint16).numpy()


def coverage_rows(topk_ids, local_start: int, local_count: int, n_box: int, n_rows: int = 64,
                  seed: int = 0) -> list[int]:
    """Tokens to check against the oracle at sizes where every row would take too long: for
    every token-tile index n (0 .. the most tiles any local expert has), a token whose pair sits
    in tile n of the expert with the most tiles; a token of the hottest and of the coldest
    local expert hit; the first and last tokens; then seeded random tokens up to n_rows."""
    ids = np.asarray(topk_ids)
    T = ids.shape[0]
    offsets, order, _ = orc.route(ids, local_start, local_count)
    counts = np.diff(offsets)
    hit = np.nonzero(counts)[0]
    rows = {0, T - 1}
    if hit.size:
        hot = int(hit[np.argmax(counts[hit])])
        cold = int(hit[np.argmin(counts[hit])])
        for e in (hot, cold):
            rows.add(int(order[offsets[e]]) // ids.shape[1])
        for n in range(-(-int(counts[hot]) // n_box)):
            rows.add(int(order[offsets[hot] + n * n_box]) // ids.shape[1])
        # the last pair of every expert (its partly filled last tile)
        rng = np.random.default_rng(seed)
        for e in rng.permutation(hit)[:8]:
            rows.add(int(order[offsets[e + 1] - 1]) // ids.shape[1])
    rng = np.random.default_rng(seed + 1)
    while len(rows) < min(n_rows, T):
        rows.add(int(rng.integers(T)))
    return sorted(rows)
