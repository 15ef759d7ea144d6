"""The prefill dispatch and the routed reduce-scatter on one GPU, with the second rank simulated
in local memory: its receive buffers, share buffers and flag array are ordinary device buffers,
and its signals are written by the test.

Rank 0 owns experts [0, 8) and rank 1 experts [8, 16). A token's row must reach exactly the
ranks that own one of its experts, its ids and weights every rank; the routed reduce-scatter
must sum, for each of rank 0's tokens, only the shares of the token's destination ranks, in rank
order. A dispatch whose peer never signals ends with device status 6 instead of hanging: every
wait is bounded by the call's own limit."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
R, T, K, H = 2, 6, 4, 256
STARTS = [0, 8, 16]
GEN, DISPATCH = 16, 20               # flag-array words: generation counter, dispatch slots
IDS = np.array([[0, 1, 2, 3],        # rank 0 only
                [8, 9, 10, 11],      # rank 1 only
                [0, 9, 3, 12],       # both
                [7, 6, 5, 4],        # rank 0 only
                [15, 8, 14, 9],      # rank 1 only
                [1, 15, 2, 14]], dtype=np.int32)
MASKS = np.array([1, 2, 3, 1, 2, 3], dtype=np.uint32)


def _u64(*ts):
    return (ctypes.c_uint64 * len(ts))(*[t.data_ptr() for t in ts])


class Ranks:
    def __init__(self):
        g = torch.Generator(device="cpu").manual_seed(11)
        self.x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
        self.ids = torch.from_numpy(IDS).to(DEV)
        self.wts = torch.rand(T, K, generator=g).to(DEV)
        self.recv_x = [torch.full((R * T, H), 7, dtype=torch.int16, device=DEV) for _ in range(R)]
        self.recv_ids = [torch.full((R * T, K), -5, dtype=torch.int32, device=DEV) for _ in range(R)]
        self.recv_w = [torch.zeros(R * T, K, device=DEV) for _ in range(R)]
        self.flags = [torch.zeros(32, dtype=torch.int32, device=DEV) for _ in range(R)]
        self.masks = torch.zeros(T, dtype=torch.int32, device=DEV)

    def dispatch(self, timeout_us):
        from muse_moe_w4a16_b200 import _lib
        starts = (ctypes.c_int * (R + 1))(*STARTS)
        return _lib.load_library().muse_moe_ep_dispatch(
            self.x.data_ptr(), self.ids.data_ptr(), self.wts.data_ptr(), T, K, H, R, 0, starts,
            _u64(*self.recv_x), _u64(*self.recv_ids), _u64(*self.recv_w), _u64(*self.flags),
            self.masks.data_ptr(), timeout_us, torch.cuda.current_stream().cuda_stream)


def test_dispatch_sends_rows_to_the_owning_ranks_only(pkg):
    from muse_moe_w4a16_b200 import _lib
    _lib.device_status(reset=True)
    r = Ranks()
    r.flags[0][DISPATCH + 1] = 1          # rank 1's dispatch of generation 1
    assert r.dispatch(1_000_000) == 0
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) == 0
    np.testing.assert_array_equal(r.masks.cpu().numpy().view(np.uint32), MASKS)
    x16 = r.x.view(torch.int16).cpu().numpy()
    for d in range(R):
        rows = r.recv_x[d].cpu().numpy()
        for t in range(T):
            slot = 0 * T + t                              # rank 0's tokens
            if (MASKS[t] >> d) & 1:
                np.testing.assert_array_equal(rows[slot], x16[t])
            else:
                assert (rows[slot] == 7).all()            # never written
        assert (rows[T:] == 7).all()                      # rank 1's slots: not this rank's to write
        np.testing.assert_array_equal(r.recv_ids[d].cpu().numpy()[:T], IDS)
        np.testing.assert_array_equal(r.recv_w[d].cpu().numpy()[:T], r.wts.cpu().numpy())
    assert r.flags[1].cpu().numpy()[DISPATCH + 0] == 1    # rank 0 signalled its peer
    assert r.flags[0].cpu().numpy()[GEN] == 0             # the dispatch does not advance the count


def test_dispatch_wait_runs_out(pkg):
    from muse_moe_w4a16_b200 import _lib
    _lib.device_status(reset=True)
    r = Ranks()                            # rank 1 never signals: the 1 ms limit runs out
    assert r.dispatch(1000) == 0
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) == 6


def test_routed_reduce_scatter_sums_the_destination_ranks(pkg):
    from muse_moe_w4a16_b200 import _lib
    _lib.device_status(reset=True)
    g = torch.Generator(device="cpu").manual_seed(5)
    # shares of parity 1 (generation 1): rank r's [R * T, H] rows; rows of tokens a rank does not
    # serve are zero in a real call -- here they hold values that must not be read
    shares = [[torch.randn(R * T, H, generator=g).to(DEV) for _ in range(R)] for _ in range(2)]
    flags = [torch.zeros(32, dtype=torch.int32, device=DEV) for _ in range(R)]
    flags[0][1] = 1                        # rank 1's round-1 signal of generation 1
    masks = torch.from_numpy(MASKS.view(np.int32)).to(DEV)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
    rc = _lib.load_library().muse_moe_peer_routed_reduce_scatter_bf16(
        _u64(*shares[0]), _u64(*shares[1]), _u64(*flags), R, 0, T, H, masks.data_ptr(), 1, 1_000_000,
        out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) == 0
    sh = [s.cpu().numpy() for s in shares[1]]
    want = np.zeros((T, H), dtype=np.float32)
    for t in range(T):
        for rr in range(R):
            if (MASKS[t] >> rr) & 1:
                want[t] += sh[rr][0 * T + t]
    np.testing.assert_array_equal(out.view(torch.int16).cpu().numpy().view(np.uint16), orc.f32_to_bf16(want))
    assert flags[0].cpu().numpy()[GEN] == 1
    assert flags[1].cpu().numpy()[0] == 1  # rank 0 signalled round 1 to its peer
