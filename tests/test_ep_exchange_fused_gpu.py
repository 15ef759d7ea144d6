"""The expert-parallel decode call that runs the layer and the exchange together
(muse_moe_forward_exchange_bf16), on one GPU with the second rank simulated in local memory:
its share buffers and flag array are ordinary device buffers, its share and its round-1 signal
are written by the test.

Rank 0 owns experts [0, 8) of 16. Small batches run as one cooperative launch, the exchange
after the combine; larger ones as the layer's launches then the exchange kernel. Either way the
output must be, bit for bit, bf16 of (this rank's fp32 share + the peer's share) -- the share
being kernel_fn_partial's value, written into the share buffer of the call's parity -- and the
flag words must move as the exchange protocol says. A peer that never signals ends the call with
device status 6 instead of a hang; a parity that does not match the device's generation does
nothing and sets 7."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
R, E, K, H, I = 2, 16, 8, 1024, 512
GEN = 16                                   # flag-array word: generation counter


def _u64(*ptrs):
    return (ctypes.c_uint64 * len(ptrs))(*ptrs)


@pytest.fixture(scope="module")
def setup(pkg):
    from muse_moe_w4a16_b200 import ep, layer, synth
    shape = synth.MoEShape(E, K, H, I, router="uniform")
    w = synth.baseline_weights(shape, seed=71, device=DEV)
    return shape, w, layer.prepare(w, ep.expert_block(E, 0, R)), layer.prepare(w)


class Ranks:
    def __init__(self, T):
        g = torch.Generator(device="cpu").manual_seed(T)
        self.shares = [[torch.zeros(T, H, device=DEV) for _ in range(R)] for _ in range(2)]
        self.shares[1][1].copy_(torch.randn(T, H, generator=g))     # the peer's share of call 1
        self.flags = [torch.zeros(32, dtype=torch.int32, device=DEV) for _ in range(R)]

    def exchange(self, ranks=R, parity=1, timeout_us=1_000_000):
        return {"shares0": _u64(*[s.data_ptr() for s in self.shares[0][:ranks]]),
                "shares1": _u64(*[s.data_ptr() for s in self.shares[1][:ranks]]),
                "flags": _u64(*[f.data_ptr() for f in self.flags[:ranks]]),
                "staging": _u64(*([0] * ranks)), "ranks": ranks, "rank": 0, "mode": 0,
                "parity": parity, "timeout_us": timeout_us}


@pytest.mark.parametrize("T,fused", [(2, True), (16, True), (40, False)])
def test_layer_and_exchange_give_the_two_step_bits(pkg, setup, T, fused):
    from muse_moe_w4a16_b200 import _lib, ep, layer, synth
    shape, _, state0, _ = setup
    assert _lib.launch_plan(T, K, E // R, H, I, E)["fused"] == fused
    d = {k: (v.to(DEV) if isinstance(v, torch.Tensor) else v)
         for k, v in synth.baseline_input(shape, T, seed=T).items()}
    local = ep._with_local_range(d, ep.expert_block(E, 0, R))
    local["config"]["n_experts"] = E
    part0 = layer.kernel_fn_partial(local, state0)
    _lib.device_status(reset=True)
    r = Ranks(T)
    r.flags[0][1] = 1                      # rank 1's round-1 signal of generation 1
    out = layer.kernel_fn_exchange(local, state0, r.shares[1][0], r.exchange())
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) == 0
    # this rank's share, written into the buffer of parity 1
    np.testing.assert_array_equal(r.shares[1][0].cpu().numpy().view(np.uint32),
                                  part0.cpu().numpy().view(np.uint32))
    want = orc.f32_to_bf16(part0.cpu().numpy() + r.shares[1][1].cpu().numpy())
    np.testing.assert_array_equal(out.view(torch.int16).cpu().numpy().view(np.uint16), want)
    assert r.flags[1].cpu().numpy()[0] == 1      # rank 0 signalled round 1 to its peer
    assert r.flags[0].cpu().numpy()[GEN] == 1    # and completed generation 1


def test_single_rank_call_equals_the_layer(pkg, setup):
    """ranks = 1: the exchange is the bf16 cast of the only share, i.e. kernel_fn's output."""
    from muse_moe_w4a16_b200 import _lib, layer, synth
    shape, _, _, state = setup
    d = {k: (v.to(DEV) if isinstance(v, torch.Tensor) else v)
         for k, v in synth.baseline_input(shape, 3, seed=9).items()}
    want = layer.kernel_fn(d, state)
    r = Ranks(3)
    out = layer.kernel_fn_exchange(d, state, r.shares[1][0], r.exchange(ranks=1))
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) == 0
    assert torch.equal(out.view(torch.int16), want.view(torch.int16))


def test_peer_that_never_signals_ends_with_status_6(pkg, setup):
    from muse_moe_w4a16_b200 import _lib, ep, layer, synth
    shape, _, state0, _ = setup
    d = {k: (v.to(DEV) if isinstance(v, torch.Tensor) else v)
         for k, v in synth.baseline_input(shape, 2, seed=4).items()}
    local = ep._with_local_range(d, ep.expert_block(E, 0, R))
    _lib.device_status(reset=True)
    r = Ranks(2)                           # rank 1 never signals: the 2 ms limit runs out
    layer.kernel_fn_exchange(local, state0, r.shares[1][0], r.exchange(timeout_us=2000))
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) == 6
    assert r.flags[1].cpu().numpy()[0] == 1      # this rank did signal
    assert r.flags[0].cpu().numpy()[GEN] == 0    # but did not complete the generation


def test_parity_mismatch_does_nothing_and_sets_7(pkg, setup):
    from muse_moe_w4a16_b200 import _lib, ep, layer, synth
    shape, _, state0, _ = setup
    d = {k: (v.to(DEV) if isinstance(v, torch.Tensor) else v)
         for k, v in synth.baseline_input(shape, 2, seed=5).items()}
    local = ep._with_local_range(d, ep.expert_block(E, 0, R))
    _lib.device_status(reset=True)
    r = Ranks(2)
    r.flags[0][1] = 1
    layer.kernel_fn_exchange(local, state0, r.shares[0][0], r.exchange(parity=0))  # device expects 1
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) == 7
    assert r.flags[1].cpu().numpy()[0] == 0      # no signal sent
    assert r.flags[0].cpu().numpy()[GEN] == 0
