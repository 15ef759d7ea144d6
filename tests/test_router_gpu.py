"""Parity of the device router top-k (muse_moe_router_topk) with the CPU oracle.

Bar: ids bit-exact (including the tie and NaN order); weights within 2e-6 relative of the
oracle (fp32 division of the same selection-order sum; the softmax mode uses the device exp).
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
DEV = torch.device("cuda:0")


def run(pkg, scores: np.ndarray, K: int, mode: str):
    ids, wts = pkg.route_topk(torch.from_numpy(np.ascontiguousarray(scores, np.float32)).to(DEV), K, mode)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), wts.cpu().numpy()


def check(pkg, scores, K, mode, rtol):
    ids, wts = run(pkg, scores, K, mode)
    rids, rwts = orc.router_topk(scores, K, mode)
    np.testing.assert_array_equal(ids, rids)
    np.testing.assert_allclose(wts, rwts, rtol=rtol, atol=0)


@pytest.mark.parametrize("name", ["router_normal_bs7", "router_skewed_bs5", "router_softmax_bs9"])
def test_router_matches_reference_fixtures(pkg, name):
    z = np.load(GOLDEN / f"{name}.npz")
    meta = json.loads(str(z["meta"]))
    ids, wts = run(pkg, z["scores"], meta["K"], meta["mode"])
    np.testing.assert_array_equal(ids, z["topk_ids"])
    np.testing.assert_allclose(wts, z["topk_weights"], rtol=2e-6, atol=0)


@pytest.mark.parametrize("T,E,K", [(1, 256, 8), (33, 256, 8), (257, 256, 8), (64, 128, 8), (9, 8, 2),
                                   (17, 40, 5), (5, 1000, 16), (3, 16, 16), (300, 64, 4)])
@pytest.mark.parametrize("mode", ["renorm", "softmax"])
def test_router_matches_oracle(pkg, T, E, K, mode):
    rng = np.random.default_rng(T * 7919 + E * 31 + K)
    scores = rng.random((T, E), dtype=np.float32) if mode == "renorm" else \
        rng.standard_normal((T, E)).astype(np.float32)
    check(pkg, scores, K, mode, 2e-6 if mode == "renorm" else 1e-5)


def test_router_ties_and_nan(pkg):
    scores = np.array([[1.0, 3.0, 3.0, np.nan, 2.0, 3.0, 0.0, 3.0],
                       [0.5] * 8,
                       [-1.0, -2.0, -1.0, -3.0, -1.0, -4.0, -1.0, -5.0]], dtype=np.float32)
    ids, wts = run(pkg, scores, 4, "renorm")
    rids, rwts = orc.router_topk(scores, 4, "renorm")
    np.testing.assert_array_equal(ids, rids)
    assert np.isnan(wts[0]).all()
    np.testing.assert_allclose(wts[1:], rwts[1:], rtol=2e-6)


def test_router_empty_batch(pkg):
    ids, wts = run(pkg, np.zeros((0, 256), np.float32), 8, "renorm")
    assert ids.shape == (0, 8) and wts.shape == (0, 8)


def test_router_feeds_the_layer_in_one_graph(pkg):
    """Router and layer captured together: the graph's output equals the eager pair's."""
    from muse_moe_w4a16_b200 import synth
    shape = synth.MoEShape(256, 8, 256, 256, local_start=0, local_count=32, router="reference-normal")
    w = synth.reference_weights(shape, device="cpu")
    st = pkg.prepare({k: v.to(DEV) for k, v in w.items()})
    x, scores = synth.reference_scores(shape, 12, seed=77)
    x, scores = x.to(DEV), scores.to(DEV)
    cfg = synth.make_config(shape, 12)

    def step():
        ids, wts = pkg.route_topk(scores, 8)
        return pkg.kernel_fn({"hidden_states": x, "topk_ids": ids, "topk_weights": wts, "config": cfg}, st)

    eager = step().clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = step()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    ids, _ = orc.router_topk(scores.cpu().numpy(), 8)
    want = scores.cpu().topk(8, dim=-1).indices.numpy()
    np.testing.assert_array_equal(ids, want)
