"""Seeded synthetic inputs for the routed W4A16 MoE layer (host-side, torch).

Two families of generators live here:

* the benchmark configurations: fp32 N(0, 0.02) weights passed through NVFP4 quantisation
  (`quantize_nvfp4`, the algorithm of nvfp4.py:50-87), bf16 N(0, 1) activations and a
  softmax/top-k router whose logits are normal, uniform or Zipf-biased;
* the reference problem's own generators (`reference_weights` / `reference_input`,
  restating reference.py:33-85 and nvfp4.py:105-141) at any shape.

Everything is generated on a `torch.Generator` of the chosen device. On the CPU the byte
streams are reproducible across machines with the same torch build, which is what the
golden fixtures under tests/golden rely on. None of this is on the timed path.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

BLOCK = 16
E2M1_MAX = 6.0
E4M3_MAX = 448.0
_E2M1_MIDS = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)   # round-to-nearest thresholds, nvfp4.py:26


# ----------------------------------------------------------------------------- NVFP4 codec

def quantize_nvfp4(x: torch.Tensor, global_scale: torch.Tensor | float | None = None):
    """Quantise the last dim of x to NVFP4 (nvfp4.py:66-87).

    Returns (packed uint8 [..., K/2] with element 2i in the low nibble, block scales
    float8_e4m3fn [..., K/16], global scale float32 []). With global_scale None the scale is
    amax / (6 * 448) (nvfp4.py:60-63), so the largest block scale lands at the top of e4m3."""
    k = x.shape[-1]
    if k % BLOCK:
        raise ValueError(f"last dim {k} is not a multiple of {BLOCK}")
    xf = x.float()
    if global_scale is None:
        amax = xf.abs().amax()
        gs = torch.where(amax > 0, amax / (E2M1_MAX * E4M3_MAX), torch.ones_like(amax))
    else:
        gs = torch.as_tensor(global_scale, dtype=torch.float32, device=x.device)
    blocks = xf.reshape(*xf.shape[:-1], k // BLOCK, BLOCK)
    sf = (blocks.abs().amax(dim=-1) / E2M1_MAX / gs).clamp(max=E4M3_MAX).to(torch.float8_e4m3fn)
    scale = (sf.float() * gs).unsqueeze(-1)
    q = torch.where(scale > 0, blocks / scale, torch.zeros_like(blocks)).reshape(xf.shape)
    # Code = number of midpoints strictly below |q| (ties round toward the smaller magnitude,
    # as torch.bucketize(right=False) does in nvfp4.py:55).
    mids = torch.tensor(_E2M1_MIDS, dtype=torch.float32, device=x.device)
    mag = torch.bucketize(q.abs().clamp(max=E2M1_MAX), mids).to(torch.uint8)
    sign = ((q < 0) & (mag > 0)).to(torch.uint8) << 3
    codes = (sign | mag).reshape(*q.shape[:-1], k // 2, 2)
    packed = codes[..., 0] | (codes[..., 1] << 4)
    return packed, sf, gs


def dequantize_nvfp4(packed: torch.Tensor, sf: torch.Tensor, gs) -> torch.Tensor:
    """e2m1 * (float(sf) * gs) in fp32 (nvfp4.py:90-97); used by tests and the EP demo only."""
    grid = torch.tensor((0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0), device=packed.device)
    p = packed.view(torch.uint8)
    codes = torch.stack((p & 0xF, p >> 4), dim=-1).flatten(-2)
    mag = grid[(codes & 0x7).long()]
    vals = torch.where((codes & 0x8) != 0, -mag, mag)
    k = vals.shape[-1]
    g = torch.as_tensor(gs, dtype=torch.float32, device=packed.device)
    out = vals.reshape(*vals.shape[:-1], k // BLOCK, BLOCK) * (sf.float() * g).unsqueeze(-1)
    return out.reshape(vals.shape)


# ----------------------------------------------------------------------------- configurations

@dataclass(frozen=True)
class MoEShape:
    """One layer shape: E experts (global), top-K, hidden H, intermediate I, and the local
    expert range [local_start, local_start + local_count) this GPU computes."""
    n_experts: int
    top_k: int
    hidden: int
    inter: int
    local_start: int = 0
    local_count: int | None = None
    router: str = "uniform"          # "normal" | "uniform" | "zipf" | "reference-normal" | ...
    zipf_s: float = 1.1

    @property
    def n_local(self) -> int:
        return self.n_experts if self.local_count is None else self.local_count


# The five configurations the benchmark is quoted on (and cfg0, the reference problem).
CONFIGS: dict[str, MoEShape] = {
    "cfg1": MoEShape(8, 2, 1024, 512, router="normal"),
    "cfg2": MoEShape(128, 8, 2048, 768, router="uniform"),
    "cfg3": MoEShape(128, 8, 2048, 768, router="zipf"),
    "cfg4": MoEShape(256, 8, 7168, 2048, router="uniform"),
    "cfg5": MoEShape(256, 8, 7168, 2048, router="zipf"),
    "cfg0": MoEShape(256, 8, 4096, 4096, local_start=0, local_count=32, router="reference-normal"),
}
TOKENS: dict[str, tuple[int, ...]] = {
    "cfg1": (16,), "cfg2": (1, 4, 16, 32), "cfg3": (128, 256, 512), "cfg4": (1, 32, 256),
    "cfg5": (4096, 8192), "cfg0": (1, 16, 32, 8, 128, 256),
}
WEIGHTS_SEED = 5252   # reference.py:26


def baseline_weights(shape: MoEShape, seed: int = WEIGHTS_SEED, device="cpu", std: float = 0.02,
                     experts: range | None = None):
    """Per-expert NVFP4 weights from fp32 N(0, std), each matrix with its own dynamic global
    scale. Returns the reference's Weights dict (baseline.py:27-34) for ALL experts (or the
    given subset, indexed from 0). Generated expert by expert in the order w13, w2."""
    e_range = range(shape.n_experts) if experts is None else experts
    g = torch.Generator(device=device).manual_seed(seed)
    H, I = shape.hidden, shape.inter
    n = len(e_range)
    w13 = torch.empty((n, 2 * I, H // 2), dtype=torch.uint8, device=device)
    w13_sf = torch.empty((n, 2 * I, H // BLOCK), dtype=torch.float8_e4m3fn, device=device)
    w2 = torch.empty((n, H, I // 2), dtype=torch.uint8, device=device)
    w2_sf = torch.empty((n, H, I // BLOCK), dtype=torch.float8_e4m3fn, device=device)
    gs13 = torch.empty((n,), dtype=torch.float32, device=device)
    gs2 = torch.empty((n,), dtype=torch.float32, device=device)
    for j, _ in enumerate(e_range):
        a = torch.randn((2 * I, H), generator=g, device=device) * std
        w13[j], w13_sf[j], gs13[j] = quantize_nvfp4(a)
        b = torch.randn((H, I), generator=g, device=device) * std
        w2[j], w2_sf[j], gs2[j] = quantize_nvfp4(b)
    post = (0.1 * torch.randn((H,), generator=g, device=device)).to(torch.bfloat16)
    return {"w13": w13, "w13_sf": w13_sf, "w13_gs": gs13, "w2": w2, "w2_sf": w2_sf, "w2_gs": gs2,
            "post_norm_w": post}


def _router_logits(shape: MoEShape, tokens: int, g: torch.Generator, device) -> torch.Tensor:
    E = shape.n_experts
    if shape.router == "normal":
        return torch.randn((tokens, E), generator=g, device=device)
    if shape.router == "uniform":
        return torch.rand((tokens, E), generator=g, device=device)
    if shape.router == "zipf":
        # p_e proportional to rank_e^-s over a seeded permutation of the experts; adding log p_e
        # to N(0,1) logits makes top-k sampling follow the Zipf popularity (Gumbel-style skew).
        rank = torch.randperm(E, generator=g, device=device).float() + 1.0
        logp = -shape.zipf_s * torch.log(rank)
        return torch.randn((tokens, E), generator=g, device=device) + logp
    raise ValueError(f"unknown router {shape.router!r}")


def baseline_input(shape: MoEShape, tokens: int, seed: int, device="cpu"):
    """The reference's Inputs dict (baseline.py:48-52): bf16 N(0,1) hidden states, top-K of a
    softmax router (weights renormalised to sum 1), global expert ids."""
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn((tokens, shape.hidden), generator=g, device=device).to(torch.bfloat16)
    probs = torch.softmax(_router_logits(shape, tokens, g, device), dim=-1)
    top = probs.topk(shape.top_k, dim=-1)
    return {
        "hidden_states": x,
        "topk_ids": top.indices.to(torch.int32),
        "topk_weights": (top.values / top.values.sum(-1, keepdim=True)).float(),
        "config": make_config(shape, tokens),
    }


def make_config(shape: MoEShape, tokens: int) -> dict:
    """The Config TypedDict of baseline.py:37-45."""
    return {"bs": tokens, "d_hidden": shape.hidden, "d_expert": shape.inter,
            "n_experts": shape.n_experts, "local_start": shape.local_start,
            "local_count": shape.n_local, "top_k": shape.top_k,
            "sharding": "full" if shape.n_local == shape.n_experts else f"ep{shape.n_experts // shape.n_local}"}


# ----------------------------------------------------------- the reference problem's generators

SCALE_LOG2_MEAN = 7.0    # nvfp4.py:20
SCALE_LOG2_STD = 0.4     # nvfp4.py:21
POPULARITY = 0.03        # reference.py:28


def random_nvfp4(rows: int, k: int, *, generator, device, leading=()):
    """Restates nvfp4.random_weights (nvfp4.py:105-128, default scales): uniform code bytes,
    log-normal e4m3 block scales clamped to [8, 448], global scale 1/sqrt(8.6 E[s^2] k)."""
    packed = torch.randint(0, 256, (*leading, rows, k // 2), dtype=torch.uint8, generator=generator,
                           device=device)
    z = torch.randn((*leading, rows, k // BLOCK), generator=generator, device=device)
    sf = torch.exp2(SCALE_LOG2_MEAN + SCALE_LOG2_STD * z).clamp(8.0, E4M3_MAX).to(torch.float8_e4m3fn)
    mean_sq = 4.0 ** SCALE_LOG2_MEAN * math.exp(2 * (math.log(2) * SCALE_LOG2_STD) ** 2)
    gs = torch.tensor(1.0 / (8.6 * mean_sq * k) ** 0.5, dtype=torch.float32, device=device)
    return packed, sf, gs


def reference_weights(shape: MoEShape, seed: int = WEIGHTS_SEED, device="cpu"):
    """Restates reference.generate_weights (reference.py:33-50) at any shape."""
    g = torch.Generator(device=device).manual_seed(seed)
    E, H, I = shape.n_experts, shape.hidden, shape.inter
    w13, w13_sf, gs13 = random_nvfp4(2 * I, H, generator=g, device=device, leading=(E,))
    w2, w2_sf, gs2 = random_nvfp4(H, I, generator=g, device=device, leading=(E,))
    return {"w13": w13, "w13_sf": w13_sf, "w13_gs": gs13.expand(E).contiguous(),
            "w2": w2, "w2_sf": w2_sf, "w2_gs": gs2.expand(E).contiguous(),
            "post_norm_w": (0.1 * torch.randn((H,), generator=g, device=device)).to(torch.bfloat16)}


def _outlier_channels(x, *, generator, frac=0.01, scale=30.0):
    """nvfp4.outlier_channels (nvfp4.py:131-141)."""
    k = x.shape[-1]
    n = max(1, int(k * frac))
    idx = torch.randperm(k, generator=generator, device=x.device)[:n]
    out = x.clone()
    out[..., idx] = (out[..., idx].float() * scale).to(x.dtype)
    return out


def reference_scores(shape: MoEShape, tokens: int, seed: int, dist: str = "normal", device="cpu"):
    """(x bf16 [T, H], router scores fp32 [T, E]) as reference.generate_input draws them
    (reference.py:62-71): uniform scores plus a Student-t popularity ("normal") or a pow-6
    heat and outlier channels ("skewed")."""
    g = torch.Generator(device=device).manual_seed(seed)
    E = shape.n_experts
    x = torch.randn((tokens, shape.hidden), generator=g, device=device).to(torch.bfloat16)
    scores = torch.rand((tokens, E), generator=g, device=device)
    if dist == "normal":
        z = torch.randn((E,), generator=g, device=device)
        u = torch.rand((E,), generator=g, device=device).clamp(min=1e-12)
        scores = scores + POPULARITY * z / (-u.log()).sqrt()
    if dist == "skewed":
        heat = torch.rand((E,), generator=g, device=device).pow(6) * 4
        scores = scores + heat
        x = _outlier_channels(x, generator=g)
    return x, scores


def reference_input(shape: MoEShape, tokens: int, seed: int, dist: str = "normal",
                    rank: str = "busiest", device="cpu"):
    """Restates reference.generate_input (reference.py:53-85) at any shape: uniform scores plus
    a Student-t popularity ("normal") or a pow-6 heat and outlier channels ("skewed"), top-K,
    and the "busiest" rotation that makes the local experts the busiest rank's."""
    x, scores = reference_scores(shape, tokens, seed, dist, device)
    E, K = shape.n_experts, shape.top_k
    routed = scores.topk(K, dim=-1)
    count = shape.n_local
    ids = routed.indices
    if rank == "busiest" and count < E:
        pairs = torch.bincount((ids // count).flatten(), minlength=E // count)
        ids = (ids - count * pairs.argmax()) % E
    return {
        "hidden_states": x,
        "topk_ids": ids.to(torch.int32),
        "topk_weights": (routed.values / routed.values.sum(-1, keepdim=True)).float(),
        "config": make_config(shape, tokens) | {"sharding": "ep8" if count * 8 == E else make_config(shape, tokens)["sharding"]},
    }
