"""The expert-parallel exchange's failure path on one GPU, with the second rank simulated in
local memory: its flags and staging buffer are ordinary device buffers that the host fills.

A wait that runs out must end the kernel with device status 6, leave the generation where it
was and the output untouched; after the flags are re-created the same call succeeds. A call
whose expected buffer parity disagrees with the device's generation does nothing and reports 7.
Nothing here faults, traps or hangs: every wait is bounded by the call's own 1 ms limit."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
N = 4096                     # fp32 elements in a share
GEN, FAIL = 16, 19           # flag-array words: generation counter, failure mark


def _u64(*ts):
    return (ctypes.c_uint64 * len(ts))(*[t.data_ptr() for t in ts])


class TwoRanks:
    def __init__(self):
        g = torch.Generator(device="cpu").manual_seed(7)
        self.share = [[torch.randn(N, generator=g).to(DEV) for _ in range(2)] for _ in range(2)]  # [parity][rank]
        self.staging = [torch.zeros(N, dtype=torch.bfloat16, device=DEV) for _ in range(2)]
        self.flags = [torch.zeros(32, dtype=torch.int32, device=DEV) for _ in range(2)]

    def call(self, out, mode, parity, timeout_us):
        from muse_moe_w4a16_b200 import _lib
        return _lib.load_library().muse_moe_peer_exchange_bf16(
            _u64(*self.share[0]), _u64(*self.share[1]), _u64(*self.flags), _u64(*self.staging), 2, 0, N,
            mode, parity, timeout_us, out.data_ptr(), torch.cuda.current_stream().cuda_stream)


def test_wait_runs_out_then_the_exchange_recovers(pkg):
    from muse_moe_w4a16_b200 import _lib
    _lib.device_status(reset=True)
    r = TwoRanks()
    sentinel = torch.full((N,), 7, dtype=torch.int16, device=DEV)
    out = sentinel.clone().view(torch.bfloat16)
    # rank 1 never signals: the 1 ms limit runs out
    assert r.call(out, 2, 1, 1000) == 0
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) == 6
    assert torch.equal(out.view(torch.int16), sentinel)
    f0 = r.flags[0].cpu().numpy()
    assert f0[GEN] == 0 and f0[FAIL] == 0           # generation not advanced, failure mark cleared
    assert r.flags[1].cpu().numpy()[0] == 1         # rank 0 did signal its peer

    # re-create the flags; rank 1's two signals of generation 1 and its staged slice are supplied
    r.flags[0].zero_()
    r.flags[0][1] = 1          # round 1 from rank 1
    r.flags[0][8 + 1] = 1      # round 2 from rank 1
    half = N // 2
    peer_slice = torch.randn(half, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).to(DEV)
    r.staging[1][half:] = peer_slice
    assert r.call(out, 2, 1, 1_000_000) == 0
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) == 0
    got = out.view(torch.int16).cpu().numpy().view(np.uint16)
    mine = (r.share[1][0][:half] + r.share[1][1][:half]).cpu().numpy()   # parity 1: generation 1
    np.testing.assert_array_equal(got[:half], orc.f32_to_bf16(mine))
    np.testing.assert_array_equal(got[half:], peer_slice.view(torch.int16).cpu().numpy().view(np.uint16))
    np.testing.assert_array_equal(r.staging[0][:half].view(torch.int16).cpu().numpy(), got[:half].view(np.int16))
    assert r.flags[0].cpu().numpy()[GEN] == 1

    # generation 2 has parity 0: a caller that wrote into buffer 1 is refused, nothing moves
    before = out.clone()
    assert r.call(out, 2, 1, 1000) == 0
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) == 7
    assert torch.equal(out.view(torch.int16), before.view(torch.int16))
    assert r.flags[0].cpu().numpy()[GEN] == 1


def test_one_round_and_reduce_scatter_modes(pkg):
    from muse_moe_w4a16_b200 import _lib
    _lib.device_status(reset=True)
    r = TwoRanks()
    r.flags[0][1] = 1            # rank 1's round-1 signal of generation 1
    out = torch.empty(N, dtype=torch.bfloat16, device=DEV)
    assert r.call(out, 0, 1, 1_000_000) == 0
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) == 0
    want = orc.f32_to_bf16((r.share[1][0] + r.share[1][1]).cpu().numpy())
    np.testing.assert_array_equal(out.view(torch.int16).cpu().numpy().view(np.uint16), want)
    # generation 2 (parity 0), reduce-scatter: rank 0 gets the first half
    r.flags[0][1] = 2
    half = torch.empty(N // 2, dtype=torch.bfloat16, device=DEV)
    assert r.call(half, 1, 0, 1_000_000) == 0
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) == 0
    want = orc.f32_to_bf16((r.share[0][0][:N // 2] + r.share[0][1][:N // 2]).cpu().numpy())
    np.testing.assert_array_equal(half.view(torch.int16).cpu().numpy().view(np.uint16), want)
    assert r.flags[0].cpu().numpy()[GEN] == 2
