"""A plain PyTorch fp32 restatement of the layer, for full-output checks at BASELINE.json's
largest sizes -- TEST INFRASTRUCTURE ONLY.

The CPU oracle (oracle/moe_oracle.py) is the pinned restatement of ref_kernel; at cfg5 sizes
(T = 8192, E = 256, H = 7168, I = 2048: ~5.8 TFLOP) it would take minutes on the host, so the
GPU tests run this torch version on the device for every row and the CPU oracle on sampled
rows. It follows reference.py:93-107 step by step -- per local expert: the (token, slot) pairs,
fp32 dequantisation e2m1 * (e4m3 * gs) (nvfp4.py:90-97), x @ W13^T, silu(gate) * up,
@ W2^T, post_expert_norm (reference.py:88-90), times the top-k weight, index_add_ into an fp32
output, one bf16 cast -- in fp32 with TF32 off. tests/test_torch_ref.py pins it to the oracle.
"""

from __future__ import annotations

import torch

_GRID = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
POST_NORM_EPS = 1e-8   # reference.py:24


def dequantize(packed: torch.Tensor, sf: torch.Tensor, gs: torch.Tensor) -> torch.Tensor:
    """uint8 [R, K/2] codes (element 2i in the low nibble), e4m3 [R, K/16] scales, fp32 gs ->
    fp32 [R, K] = e2m1 * (float(sf) * gs)."""
    grid = torch.tensor(_GRID, dtype=torch.float32, device=packed.device)
    p = packed.view(torch.uint8)
    codes = torch.stack((p & 0xF, p >> 4), dim=-1).flatten(-2).long()
    vals = torch.where((codes & 8) != 0, -grid[codes & 7], grid[codes & 7])
    scale = sf.view(torch.float8_e4m3fn).float() * gs.float()
    r, k = vals.shape
    return (vals.view(r, k // 16, 16) * scale.unsqueeze(-1)).view(r, k)


@torch.no_grad()
def layer(x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor, w: dict,
          local_start: int, local_count: int, inter: int, return_f32: bool = False) -> torch.Tensor:
    """bf16 [T, H] (or the fp32 sum) for weights `w` indexed by GLOBAL expert id."""
    prev_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        xf = x.float()
        ids = topk_ids.long()
        wts = topk_weights.float()
        out = torch.zeros(xf.shape, dtype=torch.float32, device=x.device)
        pnw = 1.0 + w["post_norm_w"].float()
        for e in torch.unique(ids).tolist():
            if not local_start <= e < local_start + local_count:
                continue
            tok, slot = (ids == e).nonzero(as_tuple=True)
            w13 = dequantize(w["w13"][e], w["w13_sf"][e], w["w13_gs"][e])
            h = xf[tok] @ w13.T
            act = torch.nn.functional.silu(h[:, :inter]) * h[:, inter:]
            w2 = dequantize(w["w2"][e], w["w2_sf"][e], w["w2_gs"][e])
            y = (act @ w2.T) * pnw
            y = y * torch.rsqrt((y * y).mean(dim=-1, keepdim=True) + POST_NORM_EPS)
            out.index_add_(0, tok, y * wts[tok, slot].unsqueeze(-1))
        return out if return_f32 else out.to(torch.bfloat16)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev_tf32
