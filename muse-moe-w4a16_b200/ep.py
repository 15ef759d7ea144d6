"""Expert parallelism across the GPUs of one node: one process per GPU, experts split into
contiguous blocks; the decode and prefill exchanges run over NVLink peer memory in this
library's kernels (collectives only for CPU tensors).

The reference's problem is always expert-parallel: GPU r holds experts
[32r, 32r + 32) and computes only their (token, slot) pairs (reference.py:18-22, TASK.md:29).
Here a rank computes the fp32 sum of its local slots for the tokens it sees
(`kernel_fn_partial`, one CUDA launch sequence), the ranks' partials are summed in fp32 and
cast to bf16 once, so the output is the single-GPU layer's output up to the order of one fp32
addition per rank.

Two layouts of the tokens:
  replicated (decode): every rank holds the same T tokens. Each rank writes its fp32 share
      [T, H] straight into its own symmetric buffer (mapped into every rank's address space),
      and one kernel of this library (`muse_moe_peer_exchange_bf16`) sums the R shares over
      NVLink in rank order and casts to bf16 -- every rank returns the same bits. Small shares
      are summed whole by every rank (one round of flags); larger ones are reduce-scattered
      (each rank sums its 1/R slice) and then all-gathered in bf16 from the ranks' staging
      buffers (two rounds), so a rank reads ~1.5 x T x H x 4 bytes over NVLink instead of
      R x T x H x 4. (With CPU tensors, as in the gloo tests of the exchange logic, the shares
      are summed by an all-reduce collective instead.)
  sharded (prefill): rank r holds its own T_r tokens (T_r equal on every rank). This library's
      dispatch kernel sends each token's row over NVLink only to the ranks that own one of its
      experts (and its ids and weights to every rank), into fixed-capacity receive buffers of
      R * T_r rows; every rank writes its experts' share of those R * T_r rows into its
      symmetric buffer, and the routed reduce-scatter returns each rank, for each of its own
      tokens, the rank-ordered sum over the token's destination ranks only (the other ranks'
      rows are zero and never cross NVLink). (CPU tensors: an all-gather and a reduce-scatter
      collective, as in the gloo tests.)

Every exchange tells the kernel which share buffer (generation parity) the host wrote into; a
disagreement with the device's count, or a peer that never signals within `timeout_us`, sets
the library's device status (7 / 6) instead of summing the wrong buffers. `check_status()`
reads it (synchronising) and raises; after such a failure call `reset_exchange()` on every rank.

Collectives use fixed shapes (no counts sent to the host), so a call issues no host
synchronisation.
"""

from __future__ import annotations

import ctypes
from typing import Callable

import torch
import torch.distributed as dist

from . import _lib
from .layer import Inputs, Weights, cast_bf16, kernel_fn_exchange, kernel_fn_partial, prepare


def expert_block(n_experts: int, rank: int, world: int) -> range:
    """Contiguous experts of `rank`: the first n_experts % world ranks hold one extra."""
    if world <= 0 or not 0 <= rank < world or n_experts < world:
        raise _lib.MuseError(_lib.MUSE_ERR_INVALID_ARGUMENT,
                             f"cannot split {n_experts} experts over {world} ranks (rank {rank})")
    base, extra = divmod(n_experts, world)
    lo = rank * base + min(rank, extra)
    return range(lo, lo + base + (1 if rank < extra else 0))


def _with_local_range(data: Inputs, experts: range) -> Inputs:
    cfg = dict(data["config"])
    cfg["local_start"], cfg["local_count"] = experts.start, len(experts)
    return {**data, "config": cfg}


class ExpertParallelMoE:
    """One rank of an expert-parallel layer.

    `weights` may hold every expert (each rank repacks only its own block) or only this rank's
    block, in which case pass `n_experts` (the model's expert count) and set `weights_are_local`.
    `local_fn(data) -> fp32 [T, H]` and `cast_fn(fp32) -> bf16` default to the CUDA kernels;
    tests replace them to check the exchange logic on CPU ranks.
    """

    def __init__(self, weights: Weights | None, group=None, *, n_experts: int | None = None,
                 weights_are_local: bool = False,
                 local_fn: Callable[[Inputs], torch.Tensor] | None = None,
                 cast_fn: Callable[[torch.Tensor], torch.Tensor] | None = None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if n_experts is None:
            n_experts = weights["w13"].shape[0]
        self.n_experts = n_experts
        self.experts = expert_block(n_experts, self.rank, self.world)
        self.state = None
        if local_fn is None:
            if weights_are_local:
                state = prepare(weights)
                state["expert_base"] = self.experts.start
            else:
                state = prepare(weights, self.experts)
            self.state = state
            local_fn = lambda d: kernel_fn_partial(d, self.state)  # noqa: E731
        self._local = local_fn
        self._cast = cast_fn or cast_bf16
        self._peer = None   # symmetric buffers of the exchange, set up on first use
        self._recv = None   # symmetric receive buffers of the prefill dispatch, set up on first use
        self._gen = 0       # exchanges completed (the device keeps its own count; they agree)
        self.timeout_us = 0  # bound of the exchange's waits for the peers (0: the library's 1 s)
        # shares of at most this many bytes are summed whole by every rank (one flag round);
        # larger ones are reduce-scattered and all-gathered (two rounds, ~R/1.5 x fewer bytes)
        self.one_round_bytes = 1 << 20

    def forward_replicated(self, data: Inputs, stage_events: list | None = None) -> torch.Tensor:
        """Decode layout: the same T tokens on every rank -> bf16 [T, H] on every rank.
        `stage_events` (three torch.cuda.Event(enable_timing=True)), if given, are recorded before
        this rank's layer kernels, between them and the exchange, and after the exchange."""
        x = data["hidden_states"]
        local = _with_local_range(data, self.experts)
        if x.shape[0] == 0:
            # every rank has the same (empty) batch: nothing to exchange, generation unchanged
            return torch.empty((0, x.shape[1]), dtype=torch.bfloat16, device=x.device)
        if not x.is_cuda or self.state is None:
            part = self._local(local)
            dist.all_reduce(part, op=dist.ReduceOp.SUM, group=self.group)
            return self._cast(part)
        self._peer_buffers(x.shape[0] * x.shape[1], x.device)
        out = self._decode(local, (self._gen + 1) & 1, stage_events)
        self._gen += 1      # only once both launches were accepted
        return out

    def exchange_mode(self, numel: int) -> int:
        """Mode of muse_moe_peer_exchange_bf16 for a decode share of `numel` fp32 values."""
        if self.world == 1 or numel * 4 * (self.world - 1) <= self.one_round_bytes:
            return 0
        return 2

    def _decode(self, local: Inputs, parity: int, stage_events: list | None = None) -> torch.Tensor:
        """The rank's share written into its share buffer `parity`, then the peer exchange (the
        kernel takes the generation from the device and checks it has this parity). One library
        call -- for small batches one launch, the exchange inside the layer's single launch --
        unless stage events are asked for, which need the layer and the exchange apart."""
        x = local["hidden_states"]
        T, H = x.shape
        peer = self._peer
        share = peer["buf"][parity * peer["cap"]:parity * peer["cap"] + T * H].view(T, H)
        mode = self.exchange_mode(T * H)
        if not stage_events:
            return kernel_fn_exchange(local, self.state, share, {
                "shares0": peer["shares"][0], "shares1": peer["shares"][1], "flags": peer["flags"],
                "staging": peer["staging"], "ranks": self.world, "rank": self.rank,
                "mode": mode, "parity": parity, "timeout_us": self.timeout_us})
        stage_events[0].record()
        kernel_fn_partial(local, self.state, out=share)
        stage_events[1].record()
        out = torch.empty((T, H), dtype=torch.bfloat16, device=x.device)
        self._exchange(T * H, mode, parity, out)
        stage_events[2].record()
        return out

    def _exchange(self, n: int, mode: int, parity: int, out: torch.Tensor) -> None:
        peer = self._peer
        _lib.call("muse_moe_peer_exchange_bf16", peer["shares"][0], peer["shares"][1], peer["flags"],
                  peer["staging"], self.world, self.rank, n, mode, parity, int(self.timeout_us),
                  out.data_ptr(), torch.cuda.current_stream(out.device).cuda_stream)

    def check_status(self) -> None:
        """Raise MuseError if an exchange (or a layer kernel) on this device has failed since the
        last check: 6 = a peer never signalled in time, 7 = generation parity mismatch. Reading
        the status synchronises the device; it clears the status."""
        st = _lib.device_status(reset=True)
        if st:
            raise _lib.MuseError(_lib.MUSE_ERR_DEVICE_TIMEOUT,
                                 f"device status {st} on rank {self.rank}: the exchange is out of step; "
                                 "call reset_exchange() on every rank")

    def reset_exchange(self) -> None:
        """Zero this rank's flags and generation count and wait for every rank to do the same
        (collective): the exchange restarts from generation 1 on all ranks."""
        if self._peer is None:
            return
        dev = self._peer["buf"].device
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)
        self._peer["buf"][self._peer["flags_at"]:].zero_()
        torch.cuda.synchronize(dev)
        self._gen = 0
        dist.barrier(group=self.group)

    def decode_graphs(self, data: Inputs) -> "DecodeGraphs":
        """CUDA graphs of the decode call for these (device) inputs; see DecodeGraphs."""
        return DecodeGraphs(self, data)

    def reserve_decode(self, tokens: int, hidden: int, device) -> None:
        """Size the decode exchange buffers for batches of up to `tokens` (collective). Graphs
        captured before a batch grows the buffers would point at released memory, so reserve
        the largest batch before capturing any."""
        self._peer_buffers(tokens * hidden, device)

    def _peer_buffers(self, numel: int, device) -> dict:
        """Symmetric buffer [2 shares of cap floats | flags] of every rank, mapped into this one
        (collective: every rank calls it with the same numel on its first decode call, and again
        when a call needs more room)."""
        if self._peer is not None and numel <= self._peer["cap"]:
            return self._peer
        import torch.distributed._symmetric_memory as symm
        if self._peer is not None:   # growing: no rank may still be reading the old buffers
            torch.cuda.synchronize(device)
            dist.barrier(group=self.group)
        cap = (max(numel, 1 << 16) + 63) // 64 * 64        # floats; keeps the shares 256-byte aligned
        # [share 0: cap fp32 | share 1: cap fp32 | bf16 staging: cap bf16 | flags: 64 words]
        flags_at = 2 * cap + cap // 2
        buf = symm.empty(flags_at + 64, dtype=torch.float32, device=device)
        buf[flags_at:].zero_()                               # flags and the generation counter start at 0
        torch.cuda.synchronize(device)
        handle = symm.rendezvous(buf, self.group if self.group is not None else dist.group.WORLD)
        bases = [int(p) for p in handle.buffer_ptrs]
        u64 = ctypes.c_uint64 * self.world
        self._peer = {
            "buf": buf, "handle": handle, "cap": cap, "flags_at": flags_at,
            "shares": [u64(*[b + k * cap * 4 for b in bases]) for k in (0, 1)],
            "staging": u64(*[b + 2 * cap * 4 for b in bases]),
            "flags": u64(*[b + flags_at * 4 for b in bases]),
        }
        self._gen = 0
        dist.barrier(group=self.group)                       # every rank's flags are zero before use
        return self._peer

    def forward_sharded(self, data: Inputs) -> torch.Tensor:
        """Prefill layout: this rank's T_r tokens (T_r equal on every rank) -> bf16 [T_r, H],
        the layer's output for those tokens over all experts."""
        x, ids, wts = data["hidden_states"], data["topk_ids"], data["topk_weights"]
        t_r = x.shape[0]
        R = self.world
        if t_r == 0:   # T_r is the same on every rank: no rank exchanges anything
            return torch.empty((0, x.shape[1]), dtype=torch.bfloat16, device=x.device)
        if not x.is_cuda or self.state is None:
            full = {}
            for name, t in (("hidden_states", x), ("topk_ids", ids.to(torch.int32)),
                            ("topk_weights", wts.to(torch.float32))):
                t = t.contiguous()
                g = torch.empty((R * t_r,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
                dist.all_gather_into_tensor(g, t, group=self.group)
                full[name] = g
            gathered = _with_local_range({**data, **full}, self.experts)
            part = self._local(gathered)
            mine = torch.empty((t_r, part.shape[1]), dtype=part.dtype, device=part.device)
            dist.reduce_scatter_tensor(mine, part, op=dist.ReduceOp.SUM, group=self.group)
            return self._cast(mine)
        if x.dtype != torch.bfloat16 or x.dim() != 2 or tuple(ids.shape) != tuple(wts.shape) or ids.shape[0] != t_r:
            # checked before the dispatch signals the peers: a call that fails later leaves the
            # ranks out of step (see check_status)
            raise _lib.MuseError(_lib.MUSE_ERR_INVALID_ARGUMENT,
                                 "hidden_states must be bf16 [T_r, H] with topk_ids / topk_weights [T_r, K]")
        H, K = x.shape[1], ids.shape[1]
        self._peer_buffers(R * t_r * H, x.device)
        recv = self._recv_buffers(R * t_r, H, K, x.device)
        peer = self._peer
        parity = (self._gen + 1) & 1
        masks = torch.empty(t_r, dtype=torch.int32, device=x.device)
        ids32, wts32 = ids.to(torch.int32).contiguous(), wts.to(torch.float32).contiguous()
        starts = (ctypes.c_int * (R + 1))(*[expert_block(self.n_experts, r, R).start for r in range(R)],
                                          self.n_experts)
        stream = torch.cuda.current_stream(x.device).cuda_stream
        _lib.call("muse_moe_ep_dispatch", x.contiguous().data_ptr(), ids32.data_ptr(), wts32.data_ptr(),
                  t_r, K, H, R, self.rank, starts, recv["x"], recv["ids"], recv["wts"], peer["flags"],
                  masks.data_ptr(), int(self.timeout_us), stream)
        n = R * t_r
        received = _with_local_range({**data, "hidden_states": recv["x_local"][:n * H].view(n, H),
                                      "topk_ids": recv["ids_local"][:n * K].view(n, K),
                                      "topk_weights": recv["wts_local"][:n * K].view(n, K)}, self.experts)
        base = parity * peer["cap"]
        share = peer["buf"][base:base + n * H].view(n, H)
        kernel_fn_partial(received, self.state, out=share)
        out = torch.empty((t_r, H), dtype=torch.bfloat16, device=x.device)
        _lib.call("muse_moe_peer_routed_reduce_scatter_bf16", peer["shares"][0], peer["shares"][1],
                  peer["flags"], R, self.rank, t_r, H, masks.data_ptr(), parity, int(self.timeout_us),
                  out.data_ptr(), stream)
        self._gen += 1
        return out

    def _recv_buffers(self, rows: int, hidden: int, top_k: int, device) -> dict:
        """Symmetric receive buffers of the prefill dispatch -- x rows (bf16 [rows, hidden]), ids
        and weights ([rows, top_k]) -- of every rank, mapped into this one (collective: every
        rank calls it with the same sizes; grown when a call needs more room)."""
        need_x, need_k = rows * hidden, rows * top_k
        if self._recv is not None and need_x <= self._recv["cap_x"] and need_k <= self._recv["cap_k"]:
            return self._recv
        import torch.distributed._symmetric_memory as symm
        if self._recv is not None:   # growing: no rank may still be writing into the old buffers
            torch.cuda.synchronize(device)
            dist.barrier(group=self.group)
        cap_x = (max(need_x, 1 << 16) + 127) // 128 * 128          # bf16 elements
        cap_k = (max(need_k, 1 << 10) + 63) // 64 * 64              # int32 / fp32 elements
        # [x: cap_x bf16 | ids: cap_k int32 | weights: cap_k fp32], in 4-byte words
        words = cap_x // 2 + 2 * cap_k
        buf = symm.empty(words, dtype=torch.int32, device=device)
        handle = symm.rendezvous(buf, self.group if self.group is not None else dist.group.WORLD)
        bases = [int(p) for p in handle.buffer_ptrs]
        u64 = ctypes.c_uint64 * self.world
        ids_at, wts_at = cap_x * 2, cap_x * 2 + cap_k * 4          # byte offsets
        self._recv = {
            "buf": buf, "handle": handle, "cap_x": cap_x, "cap_k": cap_k,
            "x": u64(*bases), "ids": u64(*[b + ids_at for b in bases]), "wts": u64(*[b + wts_at for b in bases]),
            "x_local": buf[:cap_x // 2].view(torch.bfloat16),
            "ids_local": buf[cap_x // 2:cap_x // 2 + cap_k],
            "wts_local": buf[cap_x // 2 + cap_k:].view(torch.float32),
        }
        dist.barrier(group=self.group)
        return self._recv


class DecodeGraphs:
    """Two CUDA graphs of one rank's decode call (share buffer parity 0 and 1) for fixed input
    tensors; replay() runs the one the next generation needs and returns its output tensor.
    The generation itself is counted on the device, so every rank must replay (or call
    forward_replicated) in the same sequence. Holds no collective library call."""

    def __init__(self, moe: ExpertParallelMoE, data: Inputs):
        x = data["hidden_states"]
        moe._peer_buffers(x.shape[0] * x.shape[1], x.device)
        self.moe = moe
        self.buf = moe._peer["buf"]
        local = _with_local_range(data, moe.experts)
        self.graphs, self.outs = [], []
        for parity in (0, 1):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.outs.append(moe._decode(local, parity))
            self.graphs.append(g)

    def replay(self) -> torch.Tensor:
        if self.moe._peer is None or self.moe._peer["buf"] is not self.buf:
            raise _lib.MuseError(_lib.MUSE_ERR_INVALID_ARGUMENT,
                                 "the decode buffers were reallocated after this capture (reserve_decode first)")
        k = (self.moe._gen + 1) & 1
        self.graphs[k].replay()
        self.moe._gen += 1
        return self.outs[k]
