"""The reference-facing interface: prepare(weights) / kernel_fn(data, state) / moe_forward.

Mirrors baseline.py:27-52 (the TypedDicts), baseline.py:82-151 (prepare / kernel_fn) and
reference.py:93 (ref_kernel's signature, here moe_forward). Tensors must already be on a CUDA
device; torch supplies device memory and the current stream, the work runs in libmusemoe.so.

Graph rules (TASK.md:72-78): kernel_fn makes no host sync, branches only on shapes and
`config`, and allocates only through torch's caching allocator (its output and one scratch
workspace), so it can be captured in a CUDA graph after one eager call.
"""

from __future__ import annotations

import ctypes
import weakref
from typing import TypedDict

import torch

from . import _lib


class Weights(TypedDict):
    w13: torch.Tensor          # uint8 [E, 2I, H/2], gate rows [0, I) then up rows [I, 2I), packed E2M1
    w13_sf: torch.Tensor       # float8_e4m3fn [E, 2I, H/16]
    w13_gs: torch.Tensor       # float32 [E]
    w2: torch.Tensor           # uint8 [E, H, I/2]
    w2_sf: torch.Tensor        # float8_e4m3fn [E, H, I/16]
    w2_gs: torch.Tensor        # float32 [E]
    post_norm_w: torch.Tensor  # bfloat16 [H], the post-expert RMSNorm's weight (applied as 1 + w)


class Config(TypedDict):
    bs: int           # tokens, M
    d_hidden: int     # H
    d_expert: int     # I
    n_experts: int    # experts in the model
    local_start: int  # this GPU computes experts [local_start, local_start + local_count)
    local_count: int
    top_k: int
    sharding: str


class Inputs(TypedDict):
    hidden_states: torch.Tensor  # bfloat16 [M, H]
    topk_ids: torch.Tensor       # int32 [M, K], global expert ids
    topk_weights: torch.Tensor   # float32 [M, K]
    config: Config


def _ptr(t: torch.Tensor, byte_offset: int = 0) -> int:
    return t.data_ptr() + byte_offset


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise _lib.MuseError(_lib.MUSE_ERR_NO_DEVICE, f"{name} must be a CUDA tensor (no CPU path)")


def prepare(weights: Weights, experts: range | None = None) -> dict:
    """Repack the NVFP4 weights into the kernels' tile order (lossless, same bytes;
    baseline.py:82-103). Untimed. The returned state serves any local expert range inside the
    repacked experts: all of them, or only `experts` (a contiguous global range, e.g. one
    expert-parallel rank's block) when given."""
    w13, w2 = weights["w13"], weights["w2"]
    _require_cuda(w13, "w13")
    E, two_i, h_half = w13.shape
    H, I = 2 * h_half, two_i // 2
    if tuple(w2.shape) != (E, H, I // 2):
        raise _lib.MuseError(_lib.MUSE_ERR_INVALID_ARGUMENT, f"w2 shape {tuple(w2.shape)} != {(E, H, I // 2)}")
    sel = range(E) if experts is None else experts
    if sel.step != 1 or not (0 <= sel.start < sel.stop <= E):
        raise _lib.MuseError(_lib.MUSE_ERR_INVALID_ARGUMENT, f"experts {sel} is not a contiguous range of [0, {E})")
    lo, n = sel.start, len(sel)
    dev = w13.device
    srcs = [weights["w13"], weights["w13_sf"], weights["w2"], weights["w2_sf"]]
    srcs = [s[lo:lo + n].contiguous().view(torch.uint8) for s in srcs]
    outs = [torch.empty_like(s) for s in srcs]
    with torch.cuda.device(dev):
        _lib.call("muse_moe_prepare_weights", *[_ptr(s) for s in srcs], n, H, I,
                  *[_ptr(o) for o in outs], _stream(dev))
    return {
        "w13": outs[0], "w13_sf": outs[1], "w2": outs[2], "w2_sf": outs[3],
        "w13_gs": weights["w13_gs"][lo:lo + n].to(device=dev, dtype=torch.float32).contiguous(),
        "w2_gs": weights["w2_gs"][lo:lo + n].to(device=dev, dtype=torch.float32).contiguous(),
        "post_norm_w": weights["post_norm_w"].to(device=dev, dtype=torch.bfloat16).contiguous(),
        "n_experts": n, "expert_base": lo, "hidden": H, "inter": I,
    }


def _call_args(data: Inputs, state: dict, out: torch.Tensor | None, workspace: torch.Tensor | None,
               out_dtype: torch.dtype, stage_events: list | None = None):
    """Validated argument list of muse_moe_forward_ex for one layer call, plus the output tensor.
    config["n_experts"] (the model's expert count, baseline.py:37-44) sizes the token tile; a
    missing or inconsistent value falls back to the local count."""
    cfg = data["config"]
    x = data["hidden_states"]
    _require_cuda(x, "hidden_states")
    if x.dtype != torch.bfloat16:
        raise _lib.MuseError(_lib.MUSE_ERR_INVALID_ARGUMENT, "hidden_states must be bfloat16")
    x = x.contiguous()
    ids = data["topk_ids"].to(torch.int32).contiguous()
    wts = data["topk_weights"].to(torch.float32).contiguous()
    T, H = x.shape
    K = ids.shape[1]
    I = state["inter"]
    lo, cnt = int(cfg["local_start"]), int(cfg["local_count"])
    base = int(state.get("expert_base", 0))   # global id of the state's first expert
    if H != state["hidden"] or lo < base or lo + cnt > base + state["n_experts"] \
            or tuple(ids.shape) != (T, K) or tuple(wts.shape) != (T, K):
        raise _lib.MuseError(_lib.MUSE_ERR_INVALID_ARGUMENT,
                             f"inconsistent shapes: x {tuple(x.shape)}, ids {tuple(ids.shape)}, "
                             f"weights {tuple(wts.shape)}, local [{lo}, {lo + cnt}) of "
                             f"[{base}, {base + state['n_experts']})")
    dev = x.device
    if out is None:
        out = torch.empty((T, H), dtype=out_dtype, device=dev)
    elif out.dtype != out_dtype or tuple(out.shape) != (T, H) or not out.is_contiguous():
        raise _lib.MuseError(_lib.MUSE_ERR_INVALID_ARGUMENT, f"out must be a contiguous {out_dtype} [{T}, {H}]")
    ws_bytes = _lib.workspace_size(T, K, cnt, H, I)
    if workspace is None:
        ws = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=dev)
    else:
        ws, ws_bytes = workspace, workspace.numel() * workspace.element_size()
    e0 = lo - base
    w13_e, w13sf_e = 2 * I * H // 2, 2 * I * H // 16     # bytes per expert
    w2_e, w2sf_e = H * I // 2, H * I // 16
    n_experts = int(cfg.get("n_experts", 0) or 0)
    if n_experts < lo + cnt:
        n_experts = 0
    ev = None
    if stage_events is not None:
        if len(stage_events) != 5:
            raise _lib.MuseError(_lib.MUSE_ERR_INVALID_ARGUMENT, "stage_events needs five CUDA events")
        for e in stage_events:   # torch creates the CUDA event on its first record
            if not e.cuda_event:
                e.record()
        ev = (ctypes.c_void_p * 5)(*(e.cuda_event for e in stage_events))
    args = (_ptr(x), _ptr(ids), _ptr(wts), T, K, lo, cnt, n_experts, H, I,
            _ptr(state["w13"], e0 * w13_e), _ptr(state["w13_sf"], e0 * w13sf_e),
            _ptr(state["w13_gs"], e0 * 4),
            _ptr(state["w2"], e0 * w2_e), _ptr(state["w2_sf"], e0 * w2sf_e),
            _ptr(state["w2_gs"], e0 * 4),
            _ptr(state["post_norm_w"]), _ptr(out), 1 if out_dtype == torch.float32 else 0,
            _ptr(ws), ws_bytes, _stream(dev), ev)
    return args, out


def kernel_fn(data: Inputs, state: dict, out: torch.Tensor | None = None,
              workspace: torch.Tensor | None = None,
              stage_events: list | None = None) -> torch.Tensor:
    """One routed-expert layer call (baseline.py:106-151): returns bf16 [T, H] on the GPU.
    `out` and `workspace` (uint8, >= workspace_size bytes) may be supplied by the caller.
    `stage_events` (five torch.cuda.Event(enable_timing=True)) are recorded around the kernels:
    start, before GEMM1, after GEMM1, after GEMM2, after the combine."""
    args, out = _call_args(data, state, out, workspace, torch.bfloat16, stage_events)
    _lib.call("muse_moe_forward_ex", *args)
    return out


def kernel_fn_partial(data: Inputs, state: dict, out: torch.Tensor | None = None,
                      workspace: torch.Tensor | None = None) -> torch.Tensor:
    """This rank's fp32 share of the layer (the local experts of data["config"]): fp32 [T, H],
    the sum over local slots before the bf16 cast; zeros for tokens with no local pair. The sum
    of every rank's share, cast to bf16, is kernel_fn's output over all experts."""
    args, out = _call_args(data, state, out, workspace, torch.float32)
    _lib.call("muse_moe_forward_ex", *args)
    return out


def kernel_fn_exchange(data: Inputs, state: dict, share: torch.Tensor, exchange: dict,
                       out: torch.Tensor | None = None,
                       workspace: torch.Tensor | None = None) -> torch.Tensor:
    """One expert-parallel decode call of this rank (muse_moe_forward_exchange_bf16): this
    rank's fp32 share of the layer (kernel_fn_partial's value) is written into `share` -- the
    rank's share buffer of the call's parity, fp32 [T, H] -- and every rank's share is summed
    into bf16 [T, H]. `exchange` holds the exchange's arguments: shares0, shares1, flags,
    staging (ctypes uint64 arrays of the ranks' buffer addresses), ranks, rank, mode (0 or 2),
    parity (of `share`) and timeout_us. Small batches run it as one launch."""
    args, share = _call_args(data, state, share, workspace, torch.float32)
    T, H = share.shape
    if out is None:
        out = torch.empty((T, H), dtype=torch.bfloat16, device=share.device)
    elif out.dtype != torch.bfloat16 or tuple(out.shape) != (T, H) or not out.is_contiguous():
        raise _lib.MuseError(_lib.MUSE_ERR_INVALID_ARGUMENT, f"out must be a contiguous bfloat16 [{T}, {H}]")
    # args: x, ids, wts, T, K, lo, cnt, n_experts, H, I, 6 weight pointers, post_norm_w, out,
    # out_f32, workspace, workspace bytes, stream, events
    ex = exchange
    _lib.call("muse_moe_forward_exchange_bf16", *args[:17], args[19], args[20],
              ex["shares0"], ex["shares1"], ex["flags"], ex["staging"], ex["ranks"], ex["rank"],
              ex["mode"], ex["parity"], int(ex.get("timeout_us", 0)), _ptr(out), args[21])
    return out


def cast_bf16(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 copy of a contiguous fp32 CUDA tensor (numel a multiple of 8), on the current stream."""
    _require_cuda(x, "x")
    if x.dtype != torch.float32 or not x.is_contiguous() or x.numel() % 8:
        raise _lib.MuseError(_lib.MUSE_ERR_INVALID_ARGUMENT, "cast_bf16 needs contiguous fp32, numel % 8 == 0")
    if out is None:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    _lib.call("muse_moe_cast_bf16", _ptr(x), _ptr(out), x.numel(), _stream(x.device))
    return out


def route_topk(scores: torch.Tensor, top_k: int, mode: str = "renorm",
               out: tuple[torch.Tensor, torch.Tensor] | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """(topk_ids int32 [T, K], topk_weights fp32 [T, K]) from router scores fp32 [T, E], on the
    device: the routing step of reference.generate_input (reference.py:72-84), scores.topk(K)
    then weights = values / values.sum(-1) ("renorm"), or the softmax router's weights, the
    softmax over the K selected scores ("softmax"). Ids are in descending score order; equal
    scores keep the lower expert id first."""
    _require_cuda(scores, "scores")
    if scores.dtype != torch.float32 or scores.dim() != 2 or not scores.is_contiguous():
        raise _lib.MuseError(_lib.MUSE_ERR_INVALID_ARGUMENT, "scores must be contiguous fp32 [T, E]")
    if mode not in ("renorm", "softmax"):
        raise _lib.MuseError(_lib.MUSE_ERR_INVALID_ARGUMENT, f"unknown router mode {mode!r}")
    T, E = scores.shape
    if out is None:
        out = (torch.empty((T, top_k), dtype=torch.int32, device=scores.device),
               torch.empty((T, top_k), dtype=torch.float32, device=scores.device))
    ids, wts = out
    _lib.call("muse_moe_router_topk", _ptr(scores), T, E, top_k, 0 if mode == "renorm" else 1,
              _ptr(ids), _ptr(wts), _stream(scores.device))
    return ids, wts


# prepare() results cached per weights dict (never on `data`, TASK.md:75).
_STATE_CACHE: dict[int, tuple[weakref.ref, dict]] = {}


def moe_forward(data: Inputs, weights: Weights) -> torch.Tensor:
    """ref_kernel's signature (reference.py:93): prepare once per weights, then kernel_fn."""
    key = id(weights["w13"])
    hit = _STATE_CACHE.get(key)
    if hit is None or hit[0]() is not weights["w13"]:
        _STATE_CACHE[key] = (weakref.ref(weights["w13"]), prepare(weights))
        hit = _STATE_CACHE[key]
    return kernel_fn(data, hit[1])
