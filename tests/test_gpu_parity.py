"""Parity of the CUDA layer (through the C ABI) with the CPU oracle, on seeded inputs.

Bar: routing indices bit-exact; layer output within checks.py's rule at tol 1.5e-2
(reference.py:25): relative L2 <= 1.5e-2 overall and <= 7.5e-2 per row, finite. The
observed error is far smaller (the kernels accumulate in fp32; inter is bf16 like SGLang's).
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from tests.gpu_util import bits, oracle_out, to_device, to_numpy_weights

pytestmark = pytest.mark.gpu
TOL = 1.5e-2
GOLDEN = Path(__file__).resolve().parent / "golden"
DEV = torch.device("cuda:0")


@pytest.fixture(scope="module")
def synth(pkg):
    from muse_moe_w4a16_b200 import synth as s
    return s


def run_route(pkg, ids: torch.Tensor, lo: int, cnt: int):
    from muse_moe_w4a16_b200 import _lib
    T, K = ids.shape
    ids = ids.to(DEV).contiguous()
    offsets = torch.full((cnt + 1,), -7, dtype=torch.int32, device=DEV)
    order = torch.full((max(T * K, 1),), -7, dtype=torch.int32, device=DEV)
    row = torch.full((max(T * K, 1),), -7, dtype=torch.int32, device=DEV)
    _lib.call("muse_moe_route", ids.data_ptr(), T, K, lo, cnt, offsets.data_ptr(), order.data_ptr(),
              row.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return offsets.cpu().numpy(), order.cpu().numpy()[:T * K], row.cpu().numpy()[:T * K]


@pytest.mark.parametrize("T,K,E,lo,cnt", [
    (1, 8, 128, 0, 128), (4, 8, 128, 0, 128), (33, 8, 256, 0, 32), (257, 8, 256, 32, 32),
    (5, 2, 8, 0, 8), (128, 8, 256, 0, 256), (3, 4, 16, 12, 4), (4096, 8, 256, 0, 256),
    (8192, 8, 256, 64, 64), (1000, 3, 64, 0, 1)])
def test_route_bit_exact(pkg, T, K, E, lo, cnt):
    rng = np.random.default_rng(T * 7 + E + lo)
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    offsets, order, row = run_route(pkg, torch.from_numpy(ids), lo, cnt)
    o_ref, order_ref, row_ref = orc.route(ids, lo, cnt)
    np.testing.assert_array_equal(offsets, o_ref)
    P = order_ref.size
    np.testing.assert_array_equal(order[:P], order_ref)
    assert (order[P:] == -1).all()
    np.testing.assert_array_equal(row, row_ref)


def test_route_ids_outside_every_range(pkg):
    ids = torch.tensor([[-5, 300], [7, 1 << 30]], dtype=torch.int32)
    offsets, order, row = run_route(pkg, ids, 0, 8)
    assert (offsets == np.array([0] * 8 + [1])).all()
    assert order[0] == 2 and (order[1:] == -1).all()
    assert list(row) == [-1, -1, 0, -1]


def _check_layer(pkg, w, data, rows=None, w_np=None):
    w_np = to_numpy_weights(w) if w_np is None else w_np
    out = pkg.moe_forward(to_device(data, DEV), to_device(w, DEV))
    torch.cuda.synchronize()
    got = bits(out)
    ref = oracle_out(data, w_np, rows=rows)
    if rows is not None:
        got = got[rows]
    ok, msg, err, worst = orc.compare(got, ref, TOL)
    assert ok, msg
    return err, worst


@pytest.mark.parametrize("name", ["small_e4_k2", "small_ep_e8_k3", "small_zipf_e16_k4"])
def test_layer_matches_golden_small(pkg, name):
    import json
    z = np.load(GOLDEN / f"{name}.npz")
    meta = json.loads(str(z["meta"]))
    w = {"w13": torch.from_numpy(z["w13"]), "w13_sf": torch.from_numpy(z["w13_sf"]).view(torch.float8_e4m3fn),
         "w13_gs": torch.from_numpy(z["w13_gs"]), "w2": torch.from_numpy(z["w2"]),
         "w2_sf": torch.from_numpy(z["w2_sf"]).view(torch.float8_e4m3fn), "w2_gs": torch.from_numpy(z["w2_gs"]),
         "post_norm_w": torch.from_numpy(z["post_norm_w"]).view(torch.bfloat16)}
    data = {"hidden_states": torch.from_numpy(z["x"]).view(torch.bfloat16),
            "topk_ids": torch.from_numpy(z["topk_ids"]), "topk_weights": torch.from_numpy(z["topk_weights"]),
            "config": {"local_start": meta["local_start"], "local_count": meta["local_count"],
                       "d_expert": meta["I"], "d_hidden": meta["H"]}}
    out = pkg.moe_forward(to_device(data, DEV), to_device(w, DEV))
    ok, msg, err, _ = orc.compare(bits(out), z["out"], TOL)   # against the REFERENCE's output
    assert ok and err < 5e-3, msg


def test_layer_cfg1(pkg, synth):
    shape = synth.CONFIGS["cfg1"]
    w = synth.baseline_weights(shape, seed=5252)
    err, _ = _check_layer(pkg, w, synth.baseline_input(shape, 16, seed=1016))
    assert err < 5e-3


@pytest.fixture(scope="module")
def cfg2_weights(synth):
    shape = synth.CONFIGS["cfg2"]
    return shape, synth.baseline_weights(shape, seed=5252, device="cuda")


@pytest.mark.parametrize("T", [1, 4, 16, 32])
def test_layer_cfg2_decode(pkg, synth, cfg2_weights, T):
    shape, w = cfg2_weights
    err, _ = _check_layer(pkg, w, synth.baseline_input(shape, T, seed=2000 + T))
    assert err < 5e-3


@pytest.mark.parametrize("T", [128, 256, 257, 512])
def test_layer_cfg3_zipf(pkg, synth, cfg2_weights, T):
    _, w = cfg2_weights
    shape = synth.CONFIGS["cfg3"]
    err, _ = _check_layer(pkg, w, synth.baseline_input(shape, T, seed=3000 + T))
    assert err < 5e-3


@pytest.mark.parametrize("bs,dist", [(4, "normal"), (33, "normal"), (1, "normal"), (128, "skewed")])
def test_layer_reference_problem_reduced(pkg, synth, bs, dist):
    """The reference's own generators and gating shapes (TASK.md:46-54) at H = I = 512, E = 64,
    ep8 (8 local experts), busiest rotation."""
    shape = synth.MoEShape(64, 8, 512, 512, local_start=0, local_count=8, router="reference")
    w = synth.reference_weights(shape, seed=5252)
    err, _ = _check_layer(pkg, w, synth.reference_input(shape, bs, seed=100 + bs, dist=dist))
    assert err < 5e-3


@pytest.fixture(scope="module")
def slice_weights(synth):
    shape = synth.MoEShape(16, 8, 2048, 1024, local_start=4, local_count=4, router="uniform")
    w = synth.baseline_weights(shape, seed=404)
    return shape, to_device(w, DEV), to_numpy_weights(w)


@pytest.mark.parametrize("ids", [
    [[4, 0, 1, 2, 3, 8, 9, 10]],                              # one local expert, one pair
    [[5, 6, 0, 1, 2, 3, 8, 9]],                               # two experts
    [[4, 6, 7, 0, 1, 2, 3, 8]],                               # three experts
    [[7, 0, 1, 2, 3, 8, 9, 10], [7, 4, 0, 1, 2, 3, 8, 9]],    # two tokens in one expert's tile
])
def test_layer_decode_on_a_sparse_expert_slice(pkg, synth, slice_weights, ids):
    """Decode on an expert-parallel slice that receives only 1-3 experts' pairs (most of the
    single launch's CTAs get no item; each item's chunks are split over the pipelines of one
    CTA). Output within the oracle's tolerance, and bit-identical from call to call."""
    from muse_moe_w4a16_b200 import _lib
    shape, w, w_np = slice_weights
    T = len(ids)
    assert _lib.launch_plan(T, 8, 4, 2048, 1024, 16)["fused"]
    d = synth.baseline_input(shape, T, seed=40 + T)
    d["topk_ids"] = torch.tensor(ids, dtype=torch.int32)
    st = pkg.prepare(w)
    dd = to_device(d, DEV)
    first = bits(pkg.kernel_fn(dd, st))
    second = bits(pkg.kernel_fn(dd, st))
    assert _lib.device_status() == 0
    np.testing.assert_array_equal(first, second)
    ok, msg, err, _ = orc.compare(first, oracle_out(d, w_np), TOL)
    assert ok and err < 5e-3, msg


@pytest.mark.parametrize("T,K,E,lo,cnt", [(1024, 2, 6, 0, 4), (700, 4, 8, 2, 5), (1500, 3, 3, 0, 3)])
def test_layer_pair_tile_items(pkg, synth, T, K, E, lo, cnt):
    """Prefill-sized batches (>= 128 pairs per local expert on average) run items of two
    128-token tiles that share each dequantised weight chunk; experts with an odd number of
    tiles end with a one-tile item. Every row against the oracle."""
    from muse_moe_w4a16_b200 import _lib
    H, I = 256, 384
    assert _lib.launch_plan(T, K, cnt, H, I, E)["pair_tiles"]
    shape = synth.MoEShape(E, K, H, I, local_start=lo, local_count=cnt, router="zipf")
    w = synth.baseline_weights(shape, seed=T + E)
    err, _ = _check_layer(pkg, w, synth.baseline_input(shape, T, seed=T))
    assert err < 5e-3


def test_layer_tokens_without_local_pairs_are_zero(pkg, synth):
    shape = synth.MoEShape(16, 2, 256, 128, local_start=8, local_count=4, router="uniform")
    w = synth.baseline_weights(shape, seed=1)
    data = synth.baseline_input(shape, 9, seed=3)
    data["topk_ids"][0] = torch.tensor([0, 1], dtype=torch.int32)   # token 0: nothing local
    out = pkg.moe_forward(to_device(data, DEV), to_device(w, DEV))
    assert (bits(out)[0] == 0).all()
    _check_layer(pkg, w, data)


def test_layer_empty_batch(pkg, synth):
    shape = synth.MoEShape(8, 2, 128, 128)
    w = synth.baseline_weights(shape, seed=1)
    data = synth.baseline_input(shape, 0, seed=3)
    out = pkg.moe_forward(to_device(data, DEV), to_device(w, DEV))
    assert out.shape == (0, 128)


def test_layer_cuda_graph_replay(pkg, synth, cfg2_weights):
    """kernel_fn captured in a CUDA graph, replayed on fresh inputs copied into its buffers."""
    shape, w = cfg2_weights
    state = pkg.prepare(w)
    d0 = to_device(synth.baseline_input(shape, 16, seed=1), DEV)
    pkg.kernel_fn(d0, state)  # eager call first: sets kernel attributes
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = pkg.kernel_fn(d0, state)
    w_np = to_numpy_weights(w)
    for seed in (5, 6):
        d = synth.baseline_input(shape, 16, seed=seed)
        for k in ("hidden_states", "topk_ids", "topk_weights"):
            d0[k].copy_(d[k])
        g.replay()
        torch.cuda.synchronize()
        ok, msg, *_ = orc.compare(bits(out), oracle_out(d, w_np), TOL)
        assert ok, msg


# ----------------------------------------------------------------------------- stage checks

_POS = [(6, 7, 8, 15), (22, 23, 24, 31), (2, 3, 4, 11), (18, 19, 20, 27),
        (28, 29, 30, 5), (12, 13, 14, 21), (0, 1, 10, 9), (16, 17, 26, 25)]


def _unpermute_words(w: np.ndarray) -> np.ndarray:
    w = w.astype(np.uint64)
    out = np.zeros_like(w)
    for k, pos in enumerate(_POS):
        for b, p in enumerate(pos):
            out |= ((w >> np.uint64(p)) & np.uint64(1)) << np.uint64(4 * k + b)
    return out.astype(np.uint32)


def _untile(codes: np.ndarray, scales: np.ndarray, E: int, rows: int, k: int, gate_up_inter: int):
    """Invert the prepared layout (csrc/layout.cuh) back to [E, rows, k/2] / [E, rows, k/16]."""
    mt, kc = rows // 128, k // 128
    c = codes.reshape(E, mt, kc, 128, 4, 16)          # [.., row, slot, 16 bytes]
    s = scales.reshape(E, mt, kc, 128, 8)
    r = np.arange(128)
    slot_of_chunk = np.stack([np.arange(4) ^ ((ri >> 1) & 3) for ri in r])   # [128, 4]
    c = np.take_along_axis(c, slot_of_chunk[None, None, None, :, :, None], axis=4)
    words = _unpermute_words(c.reshape(-1).view(np.uint32)).view(np.uint8).reshape(c.shape)
    words = words.reshape(E, mt, kc, 128, 64).transpose(0, 1, 3, 2, 4).reshape(E, mt, 128, k // 2)
    s = s.transpose(0, 1, 3, 2, 4).reshape(E, mt, 128, k // 16)
    out_c = np.zeros((E, rows, k // 2), np.uint8)
    out_s = np.zeros((E, rows, k // 16), np.uint8)
    for m in range(mt):
        for ri in range(128):
            if gate_up_inter:
                q, i = ri >> 5, ri & 31
                j = 64 * m + 16 * q + (i & 15)
                src = j if i < 16 else gate_up_inter + j
            else:
                src = 128 * m + ri
            out_c[:, src] = words[:, m, ri]
            out_s[:, src] = s[:, m, ri]
    return out_c, out_s


def test_prepare_repack_is_lossless(pkg, synth):
    shape = synth.MoEShape(3, 2, 256, 384)
    w = synth.baseline_weights(shape, seed=9)
    st = pkg.prepare(to_device(w, DEV))
    torch.cuda.synchronize()
    H, I = 256, 384
    c13, s13 = _untile(st["w13"].cpu().numpy(), st["w13_sf"].cpu().numpy(), 3, 2 * I, H, I)
    np.testing.assert_array_equal(c13, w["w13"].numpy())
    np.testing.assert_array_equal(s13, w["w13_sf"].view(torch.uint8).numpy())
    c2, s2 = _untile(st["w2"].cpu().numpy(), st["w2_sf"].cpu().numpy(), 3, H, I, 0)
    np.testing.assert_array_equal(c2, w["w2"].numpy())
    np.testing.assert_array_equal(s2, w["w2_sf"].view(torch.uint8).numpy())


def test_stage_outputs_match_oracle(pkg, synth):
    """GEMM1's inter and GEMM2's ypart/ssq, read from the workspace, against fp32 restatements
    of reference.py:103-106 per pair (inter is stored in bf16)."""
    from muse_moe_w4a16_b200 import _lib
    shape = synth.MoEShape(8, 2, 256, 256, router="normal")
    T, K, H, I = 16, 2, 256, 256
    w = synth.baseline_weights(shape, seed=5252)
    d = synth.baseline_input(shape, T, seed=77)
    st = pkg.prepare(to_device(w, DEV))
    nbytes = _lib.workspace_size(T, K, 8, H, I)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=DEV)
    pkg.kernel_fn(to_device(d, DEV), st, workspace=ws)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    off = _lib.workspace_offsets(T, K, 8, H, I)
    wsc = ws.cpu()
    P = T * K
    order = wsc[off["pair_order"]:off["pair_order"] + 4 * P].view(torch.int32).numpy()
    inter = wsc[off["inter"]:off["inter"] + 2 * P * I].view(torch.bfloat16).float().numpy().reshape(P, I)
    ypart = wsc[off["ypart"]:off["ypart"] + 4 * P * H].view(torch.float32).numpy().reshape(P, H)
    ssq = wsc[off["ssq"]:off["ssq"] + 4 * P * (H // 32)].view(torch.float32).numpy().reshape(P, H // 32)
    wn = to_numpy_weights(w)
    x = orc.bf16_to_f32(d["hidden_states"].view(torch.uint16).numpy())
    ids = d["topk_ids"].numpy()
    pnw = orc.bf16_to_f32(wn["post_norm_w"])
    for r, p in enumerate(order):
        t, s = divmod(int(p), K)
        e = int(ids[t, s])
        h = x[t] @ orc.dequantize(wn["w13"][e], wn["w13_sf"][e], wn["w13_gs"][e]).T
        ref_i = orc.silu(h[:I]) * h[I:]
        err_i = np.linalg.norm(inter[r] - ref_i) / np.linalg.norm(ref_i)
        assert err_i < 8e-3, f"inter row {r} (pair {p}, expert {e}): rel err {err_i:.3e}"
        y = inter[r] @ orc.dequantize(wn["w2"][e], wn["w2_sf"][e], wn["w2_gs"][e]).T * (1 + pnw)
        err_y = np.linalg.norm(ypart[r] - y) / np.linalg.norm(y)
        assert err_y < 1e-4, f"ypart row {r}: rel err {err_y:.3e}"
        sl = (y * y).reshape(H // 32, 32).sum(1)
        np.testing.assert_allclose(ssq[r], sl, rtol=1e-3, atol=1e-6 * float(sl.sum()))


@pytest.mark.parametrize("T,E,K,lo,cnt", [(16, 8, 2, 0, 8), (128, 256, 8, 0, 256), (33, 256, 8, 32, 32),
                                          (300, 256, 8, 0, 256), (1100, 256, 8, 0, 256),
                                          (4000, 64, 4, 16, 32)])
def test_published_routing_and_dirty_workspace(pkg, synth, T, E, K, lo, cnt):
    """Batches of <= 1024 pairs with small token tiles are routed inside the first GEMM, larger
    ones by the route kernels (one CTA, or several CTAs of 4096 pairs each from 4097 pairs on);
    either way the workspace ends up holding the oracle's routing, bit-exact, and the output is
    right even when the workspace starts full of garbage (nothing in it is read before the same
    call has written it)."""
    from muse_moe_w4a16_b200 import _lib
    H, I = 256, 256
    shape = synth.MoEShape(E, K, H, I, local_start=lo, local_count=cnt, router="uniform")
    w = synth.baseline_weights(shape, seed=21)
    d = synth.baseline_input(shape, T, seed=T + E)
    st = pkg.prepare(to_device(w, DEV))
    nbytes = _lib.workspace_size(T, K, cnt, H, I)
    ws = torch.full((nbytes,), 0x7F, dtype=torch.uint8, device=DEV)   # fp32 0x7F7F7F7F ~ 3.4e38
    dd = to_device(d, DEV)
    ref = oracle_out(d, to_numpy_weights(w))
    for _ in range(2):
        out = pkg.kernel_fn(dd, st, workspace=ws)
        torch.cuda.synchronize()
        assert _lib.device_status() == 0
        ok, msg, _, _ = orc.compare(bits(out), ref, TOL)
        assert ok, msg
    off = _lib.workspace_offsets(T, K, cnt, H, I)
    wsc = ws.cpu()
    P = T * K
    o_ref, order_ref, row_ref = orc.route(d["topk_ids"].numpy(), lo, cnt)
    offsets = wsc[off["offsets"]:off["offsets"] + 4 * (cnt + 1)].view(torch.int32).numpy()
    order = wsc[off["pair_order"]:off["pair_order"] + 4 * P].view(torch.int32).numpy()
    row = wsc[off["pair_row"]:off["pair_row"] + 4 * P].view(torch.int32).numpy()
    np.testing.assert_array_equal(offsets, o_ref)
    n = order_ref.size
    np.testing.assert_array_equal(order[:n], order_ref)
    assert (order[n:] == -1).all()
    np.testing.assert_array_equal(row, row_ref)


@pytest.mark.parametrize("T", [4, 300, 1100])
def test_profiled_forward_matches_and_times(pkg, synth, cfg2_weights, T):
    """The event-recording variant gives the same bits as the plain call (the layer is
    bit-reproducible: no floating-point atomics), and its five events bracket the kernels."""
    shape, w = cfg2_weights
    st = pkg.prepare(w)
    d = to_device(synth.baseline_input(shape, T, seed=T), DEV)
    ref = pkg.kernel_fn(d, st).clone()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    got = pkg.kernel_fn(d, st, stage_events=ev)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
    gaps = [ev[i].elapsed_time(ev[i + 1]) for i in range(4)]
    from muse_moe_w4a16_b200 import _lib
    fused = _lib.launch_plan(T, shape.top_k, shape.n_local, shape.hidden, shape.inter)["fused"]
    assert all(g >= 0 for g in gaps) and gaps[1] > 0, gaps
    if not fused:   # separate GEMM2 and combine launches
        assert gaps[2] > 0 and gaps[3] > 0, gaps


@pytest.mark.parametrize("T", [3, 40, 300])
def test_partial_shares_sum_to_the_layer(pkg, synth, T):
    """Expert-parallel building blocks on one GPU: the fp32 shares of three disjoint expert
    blocks (each repacked on its own, as an expert-parallel rank would), summed and cast to bf16
    by the library, give the single-call layer's output and the oracle's."""
    from muse_moe_w4a16_b200 import ep, layer
    shape = synth.MoEShape(24, 4, 256, 384, router="normal")
    w = synth.baseline_weights(shape, seed=77, device=DEV)
    d = to_device(synth.baseline_input(shape, T, seed=T), DEV)
    total = None
    for r in range(3):
        block = ep.expert_block(24, r, 3)
        st = layer.prepare(w, block)
        part = layer.kernel_fn_partial(ep._with_local_range(d, block), st)
        total = part if total is None else total + part
    got = layer.cast_bf16(total)
    torch.cuda.synchronize()
    whole = pkg.kernel_fn(d, pkg.prepare(w))
    ok, msg, err, _ = orc.compare(bits(got), bits(whole), TOL)
    assert ok and err < 1e-3, msg
    ok, msg, _, _ = orc.compare(bits(got), oracle_out(synth.baseline_input(shape, T, seed=T), to_numpy_weights(w)), TOL)
    assert ok, msg


def test_cast_bf16_rounds_to_nearest_even(pkg):
    from muse_moe_w4a16_b200 import layer
    x = torch.randn(4096, device=DEV) * torch.logspace(-30, 30, 4096, device=DEV)
    x[:4] = torch.tensor([1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -0.0, float("inf")], device=DEV)
    got = layer.cast_bf16(x)
    torch.cuda.synchronize()
    ref = orc.f32_to_bf16(x.cpu().numpy())
    np.testing.assert_array_equal(bits(got), ref)
