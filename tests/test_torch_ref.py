"""Pin the torch fp32 restatement (tests/torch_ref.py, used for full-output GPU checks at the
largest sizes) to the reference's own outputs and to the CPU oracle. CPU only."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from tests import torch_ref

GOLDEN = Path(__file__).resolve().parent / "golden"


def _problem(name):
    z = np.load(GOLDEN / f"{name}.npz")
    meta = json.loads(str(z["meta"]))
    w = {"w13": torch.from_numpy(z["w13"]), "w13_sf": torch.from_numpy(z["w13_sf"]).view(torch.float8_e4m3fn),
         "w13_gs": torch.from_numpy(z["w13_gs"]), "w2": torch.from_numpy(z["w2"]),
         "w2_sf": torch.from_numpy(z["w2_sf"]).view(torch.float8_e4m3fn), "w2_gs": torch.from_numpy(z["w2_gs"]),
         "post_norm_w": torch.from_numpy(z["post_norm_w"]).view(torch.bfloat16)}
    x = torch.from_numpy(z["x"]).view(torch.bfloat16)
    return meta, z, w, x


@pytest.mark.parametrize("name", ["small_e4_k2", "small_ep_e8_k3", "small_zipf_e16_k4"])
def test_torch_ref_matches_reference_output(name):
    meta, z, w, x = _problem(name)
    out = torch_ref.layer(x, torch.from_numpy(z["topk_ids"]), torch.from_numpy(z["topk_weights"]), w,
                          meta["local_start"], meta["local_count"], meta["I"])
    got = out.view(torch.uint16).numpy()
    ok, msg, err, _ = orc.compare(got, z["out"], 1e-5)
    assert ok, msg
    assert (got == z["out"]).mean() > 0.99


def test_torch_ref_dequantize_matches_oracle_on_every_byte():
    codes = np.tile(np.arange(256, dtype=np.uint8), (256, 1))
    scales = np.repeat(np.arange(256, dtype=np.uint8)[:, None], 32, axis=1)
    gs = np.float32(0.0123)
    ref = orc.dequantize(codes, scales, gs)
    got = torch_ref.dequantize(torch.from_numpy(codes), torch.from_numpy(scales),
                               torch.tensor(gs)).numpy()
    np.testing.assert_array_equal(got, ref)


def test_torch_ref_matches_oracle_f32(pkg):
    from muse_moe_w4a16_b200 import synth
    shape = synth.MoEShape(12, 4, 256, 384, local_start=2, local_count=7, router="zipf")
    w = synth.baseline_weights(shape, seed=3)
    d = synth.baseline_input(shape, 23, seed=4)
    w_np = {k: (v.view(torch.uint8) if v.dtype == torch.float8_e4m3fn else
                v.view(torch.uint16) if v.dtype == torch.bfloat16 else v).numpy() for k, v in w.items()}
    ref = orc.ref_kernel(d["hidden_states"].view(torch.uint16).numpy(), d["topk_ids"].numpy(),
                         d["topk_weights"].numpy(), w_np, 2, 7, 384, return_f32=True)
    got = torch_ref.layer(d["hidden_states"], d["topk_ids"], d["topk_weights"], w, 2, 7, 384,
                          return_f32=True).numpy()
    np.testing.assert_allclose(got, ref, rtol=2e-5, atol=2e-5 * float(np.abs(ref).max()))
