"""Pin the CPU oracle and the synthetic-input generators to the reference's own outputs.

The fixtures in tests/golden were produced by tests/golden/make_golden.py running the
reference's reference.py / nvfp4.py / checks.py on the CPU. Nothing here needs a GPU.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    z = np.load(GOLDEN / f"{name}.npz")
    return json.loads(str(z["meta"])), z


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def assert_bf16_close(out, ref, max_ulp=1, exact_frac=0.99):
    """bf16 outputs: at most `max_ulp` units apart (fp32 sums in another order may round to the
    neighbouring bf16) and almost all bit-identical."""
    a = out.astype(np.int32)
    b = ref.astype(np.int32)
    # compare in sign-magnitude order so -0/+0 and neighbours across zero are 1 apart
    def ordered(v):
        return np.where(v & 0x8000, -(v & 0x7FFF), v & 0x7FFF)
    diff = np.abs(ordered(a) - ordered(b))
    assert diff.max() <= max_ulp, f"max bf16 ulp diff {diff.max()}"
    assert (diff == 0).mean() >= exact_frac, f"only {(diff == 0).mean():.4f} bit-exact"


# ----------------------------------------------------------------------------- codec

def test_e4m3_table_matches_reference():
    _, z = load("codec_kat")
    np.testing.assert_array_equal(orc.e4m3_table(), z["e4m3"])


def test_e2m1_unpack_matches_reference():
    _, z = load("codec_kat")
    got = orc.unpack_e2m1(np.arange(256, dtype=np.uint8))
    np.testing.assert_array_equal(got, z["e2m1_unpack"])


def test_dequantize_every_code_and_scale_byte():
    meta, z = load("codec_kat")
    codes = np.tile(np.arange(256, dtype=np.uint8), (256, 1))
    scales = np.repeat(np.arange(256, dtype=np.uint8)[:, None], 32, axis=1)
    got = orc.dequantize(codes, scales, np.float32(meta["gs"]))
    np.testing.assert_array_equal(got, z["dequant_all"])  # NaN scale rows compare equal too


def test_quantize_matches_reference(pkg):
    from muse_moe_w4a16_b200 import synth
    _, z = load("quantize_kat")
    packed, sf, gs = synth.quantize_nvfp4(torch.from_numpy(z["x"]))
    np.testing.assert_array_equal(packed.numpy(), z["packed"])
    np.testing.assert_array_equal(sf.view(torch.uint8).numpy(), z["sf"])
    assert float(gs) == float(z["gs"])
    np.testing.assert_array_equal(orc.dequantize(z["packed"], z["sf"], z["gs"]), z["dequant"])
    # the edge blocks: all-zero block -> zero scale and zero codes
    assert z["sf"][0, 0, 0] == 0 and not z["packed"][0, 0, :8].any()


def test_bf16_round_trip():
    x = np.array([1.0, -2.5, 3.14159, 1e-30, 65504.0, -0.0], dtype=np.float32)
    bits = orc.f32_to_bf16(x)
    ref = torch.from_numpy(x).to(torch.bfloat16).view(torch.uint16).numpy()
    np.testing.assert_array_equal(bits, ref)
    np.testing.assert_array_equal(orc.bf16_to_f32(bits),
                                  torch.from_numpy(x).to(torch.bfloat16).float().numpy())


# ----------------------------------------------------------------------------- ref_kernel

def _weights_from(z):
    return {k: z[k] for k in ("w13", "w13_sf", "w13_gs", "w2", "w2_sf", "w2_gs", "post_norm_w")}


@pytest.mark.parametrize("name", ["small_e4_k2", "small_ep_e8_k3", "small_zipf_e16_k4"])
def test_oracle_matches_reference_small(name):
    meta, z = load(name)
    out = orc.ref_kernel(z["x"], z["topk_ids"], z["topk_weights"], _weights_from(z),
                         meta["local_start"], meta["local_count"], meta["I"])
    assert_bf16_close(out, z["out"])
    ok, msg, err, _ = orc.compare(out, z["out"])
    assert ok and err < 1e-3, msg


@pytest.mark.parametrize("name", ["small_e4_k2", "small_ep_e8_k3", "small_zipf_e16_k4"])
def test_synth_regenerates_small_fixtures(name, pkg):
    from muse_moe_w4a16_b200 import synth
    meta, z = load(name)
    shape = synth.MoEShape(meta["E"], meta["K"], meta["H"], meta["I"], local_start=meta["local_start"],
                           local_count=meta["local_count"], router=meta["router"])
    w = synth.baseline_weights(shape, seed=meta["weights_seed"])
    d = synth.baseline_input(shape, meta["T"], seed=meta["input_seed"])
    np.testing.assert_array_equal(w["w13"].numpy(), z["w13"])
    np.testing.assert_array_equal(w["w2_sf"].view(torch.uint8).numpy(), z["w2_sf"])
    np.testing.assert_array_equal(d["hidden_states"].view(torch.uint16).numpy(), z["x"])
    np.testing.assert_array_equal(d["topk_ids"].numpy(), z["topk_ids"])
    np.testing.assert_array_equal(d["topk_weights"].numpy(), z["topk_weights"])


def test_cfg1_weights_digest_and_oracle(pkg):
    from muse_moe_w4a16_b200 import synth
    meta, z = load("cfg1_t16")
    shape = synth.CONFIGS["cfg1"]
    w = synth.baseline_weights(shape, seed=meta["weights_seed"])
    for k, digest in meta["sha256"].items():
        assert sha(w[k]) == digest, f"{k} regenerated differently"
    d = synth.baseline_input(shape, 16, seed=meta["input_seed"])
    np.testing.assert_array_equal(d["hidden_states"].view(torch.uint16).numpy(), z["x"])
    np.testing.assert_array_equal(d["topk_ids"].numpy(), z["topk_ids"])
    npw = {k: (v.view(torch.uint8) if v.dtype == torch.float8_e4m3fn else
               v.view(torch.uint16) if v.dtype == torch.bfloat16 else v).numpy() for k, v in w.items()}
    out = orc.ref_kernel(z["x"], z["topk_ids"], z["topk_weights"], npw, 0, 8, 512)
    assert_bf16_close(out, z["out"])


@pytest.mark.parametrize("case", ["refgen_normal_bs9", "refgen_skewed_bs6", "refgen_normal_bs1"])
def test_reference_generators_and_oracle(case, pkg):
    from muse_moe_w4a16_b200 import synth
    wmeta, wz = load("refgen_weights")
    meta, z = load(case)
    shape = synth.MoEShape(16, 4, 128, 128, local_start=0, local_count=4, router="reference")
    w = synth.reference_weights(shape, seed=meta["weights_seed"])
    for k, digest in wmeta["sha256"].items():
        assert sha(w[k]) == digest, f"synth.reference_weights {k} differs from reference.generate_weights"
    d = synth.reference_input(shape, meta["T"], meta["input_seed"], dist=meta["dist"])
    np.testing.assert_array_equal(d["hidden_states"].view(torch.uint16).numpy(), z["x"])
    np.testing.assert_array_equal(d["topk_ids"].numpy(), z["topk_ids"])
    np.testing.assert_array_equal(d["topk_weights"].numpy(), z["topk_weights"])
    out = orc.ref_kernel(z["x"], z["topk_ids"], z["topk_weights"], _weights_from(wz), 0, 4, 128)
    assert_bf16_close(out, z["out"])


def test_compare_matches_checks():
    meta, z = load("compare_kat")
    for k, expected in meta["results"].items():
        ok, *_ = orc.compare(z[k], z["ref"])
        assert ok == expected, k


# ----------------------------------------------------------------------------- routing

def _route_by_reference_loop(ids, lo, cnt):
    """The pair order of reference.py:99-102 written out literally."""
    order = []
    for e in sorted(set(ids.reshape(-1).tolist())):
        if not lo <= e < lo + cnt:
            continue
        tok, slot = np.nonzero(ids == e)
        order += (tok * ids.shape[1] + slot).tolist()
    return np.array(order, dtype=np.int32)


@pytest.mark.parametrize("T,K,E,lo,cnt", [(1, 8, 128, 0, 128), (33, 8, 256, 32, 32), (257, 8, 256, 0, 32),
                                          (5, 2, 8, 0, 8), (64, 4, 16, 12, 4), (0, 8, 32, 0, 32)])
def test_route_oracle_is_reference_order(T, K, E, lo, cnt):
    rng = np.random.default_rng(T * 1000 + E)
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32) if T else \
        np.zeros((0, K), np.int32)
    offsets, order, row = orc.route(ids, lo, cnt)
    np.testing.assert_array_equal(order, _route_by_reference_loop(ids, lo, cnt))
    assert offsets[-1] == order.size
    assert (row[order] == np.arange(order.size)).all()
    assert (row >= 0).sum() == order.size


def test_package_byte_model_matches_oracle(pkg):
    """The benchmark's byte/FLOP model (package side) equals the oracle's statement of it."""
    from muse_moe_w4a16_b200 import traffic
    rng = np.random.default_rng(3)
    for T, K, E, lo, cnt in [(1, 8, 128, 0, 128), (33, 8, 256, 32, 32), (300, 2, 8, 0, 8)]:
        ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
        for H, I in [(2048, 768), (256, 128)]:
            assert traffic.layer_bytes(ids, lo, cnt, H, I) == orc.algorithmic_bytes(ids, lo, cnt, H, I)
            assert traffic.layer_flops(ids, lo, cnt, H, I) == orc.algorithmic_flops(ids, lo, cnt, H, I)
            g1 = traffic.gemm1_bytes(ids, lo, cnt, H, I)
            g2 = traffic.gemm2_bytes(ids, lo, cnt, H, I)
            assert g1 > 0 and g2 > 0


@pytest.mark.parametrize("name", ["router_normal_bs7", "router_skewed_bs5", "router_softmax_bs9"])
def test_router_oracle_matches_reference(name):
    """The router restatement reproduces the reference's own routing step (generate_input's
    topk + renormalisation) and the softmax router, on the fixtures' scores."""
    meta, z = load(name)
    ids, wts = orc.router_topk(z["scores"], meta["K"], meta["mode"])
    np.testing.assert_array_equal(ids, z["topk_ids"])
    np.testing.assert_allclose(wts, z["topk_weights"], rtol=2e-6, atol=0)


def test_router_oracle_tie_and_nan_order():
    scores = np.array([[1.0, 3.0, 3.0, np.nan, 2.0, 3.0],
                       [0.5, 0.5, 0.5, 0.5, 0.5, 0.5]], dtype=np.float32)
    ids, wts = orc.router_topk(scores, 4, "renorm")
    np.testing.assert_array_equal(ids[0], [3, 1, 2, 5])   # NaN first, then equal 3.0s by id
    np.testing.assert_array_equal(ids[1], [0, 1, 2, 3])
    assert np.isnan(wts[0]).all()                           # a NaN score poisons the sum
    np.testing.assert_allclose(wts[1], 0.25)
