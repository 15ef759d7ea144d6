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
