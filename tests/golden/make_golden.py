"""Generate the golden fixtures in this directory by running the REFERENCE's own Python code
(reference.py, nvfp4.py, checks.py) on the CPU.

    python tests/golden/make_golden.py [--reference DIR]

Needs the reference checkout (its directory via --reference or $MUSE_REFERENCE_DIR); it is only run in the build
container, never on the GPU box, and never by the tests. The tests read the .npz files it
writes. Every input is generated on a CPU torch.Generator, so the same bytes can be rebuilt
by the package's synth module; the fixtures store the reference's outputs plus SHA-256
digests of inputs too large to commit.
"""

from __future__ import annotations

import argparse
import os
import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def u8(t):  # fp8 / uint8 tensors as raw bytes
    return t.contiguous().view(torch.uint8).numpy()


def u16(t):  # bf16 as raw bits
    return t.contiguous().view(torch.uint16).numpy()


def save(name: str, meta: dict, **arrays):
    path = HERE / f"{name}.npz"
    np.savez_compressed(path, meta=np.array(json.dumps(meta, sort_keys=True)), **arrays)
    print(f"wrote {path.relative_to(REPO)} ({path.stat().st_size} bytes)")


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MUSE_REFERENCE_DIR"),
                    help="directory holding the reference's reference.py / nvfp4.py / checks.py "
                         "(or set MUSE_REFERENCE_DIR)")
    a = ap.parse_args()
    if not a.reference:
        ap.error("give --reference DIR or set MUSE_REFERENCE_DIR")
    sys.path.insert(0, a.reference)
    sys.path.insert(0, str(REPO))
    import checks  # noqa: F401  (reference)
    import nvfp4  # reference
    import reference  # reference

    import __graft_entry__
    __graft_entry__.load_package()
    from muse_moe_w4a16_b200 import synth

    torch.set_num_threads(8)

    # ---- 1. codec known answers: e4m3 decoding of every byte, e2m1 unpack of every byte.
    all_bytes = torch.arange(256, dtype=torch.uint8)
    e4m3 = all_bytes.view(torch.float8_e4m3fn).float().numpy()
    e2m1 = nvfp4.unpack_e2m1(all_bytes).numpy()      # [512] = 256 bytes x (lo, hi)
    # dequantize with every (code byte, scale byte) pair for one global scale
    codes = all_bytes.repeat(256, 1)                  # [256 scale rows, 256 code bytes] -> K = 512
    scales = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).unsqueeze(1).repeat(1, 32)
    deq = nvfp4.dequantize(codes, scales, torch.tensor(0.0123, dtype=torch.float32)).numpy()
    save("codec_kat", {"gs": 0.0123}, e4m3=e4m3, e2m1_unpack=e2m1,
         dequant_all=deq.astype(np.float32))

    # ---- 2. quantize known answers (nvfp4.quantize), with edge blocks.
    g = torch.Generator().manual_seed(77)
    xq = torch.randn((3, 4, 64), generator=g) * 0.02
    xq[0, 0, :16] = 0.0                        # an all-zero block -> zero scale and codes
    xq[0, 1, 16:32] = 1e-9                     # a tiny block -> e4m3 subnormal / zero scale
    xq[1, 2, :] *= 40.0                        # a row with the tensor amax
    xq[2, 3, 5] = 0.25 * float(xq.abs().max())  # mid-grid values
    packed, sf, gs = nvfp4.quantize(xq)
    p2, sf2, gs2 = synth.quantize_nvfp4(xq)
    assert torch.equal(packed, p2) and torch.equal(u8t(sf), u8t(sf2)) and torch.equal(gs, gs2), \
        "synth.quantize_nvfp4 differs from nvfp4.quantize"
    save("quantize_kat", {}, x=xq.numpy(), packed=packed.numpy(), sf=u8(sf), gs=gs.numpy(),
         dequant=nvfp4.dequantize(packed, sf, gs).numpy())

    # ---- 3. ref_kernel on small BASELINE-style shapes, full inputs stored.
    def run_ref(weights, data, inter):
        reference.D_EXPERT = inter
        return reference.ref_kernel(data, weights)

    small_cases = {
        # name: (E, K, H, I, T, local_start, local_count, router, input seed)
        "small_e4_k2": (4, 2, 128, 128, 5, 0, 4, "normal", 11),
        "small_ep_e8_k3": (8, 3, 256, 128, 7, 2, 4, "uniform", 12),
        "small_zipf_e16_k4": (16, 4, 128, 128, 33, 0, 16, "zipf", 13),
    }
    for name, (E, K, H, I, T, lo, cnt, router, seed) in small_cases.items():
        shape = synth.MoEShape(E, K, H, I, local_start=lo, local_count=cnt, router=router)
        w = synth.baseline_weights(shape, seed=5252)
        _check_against_reference_quantize(nvfp4, synth, shape, w, seed=5252)
        d = synth.baseline_input(shape, T, seed=seed)
        out = run_ref(w, d, I)
        meta = {"E": E, "K": K, "H": H, "I": I, "T": T, "local_start": lo, "local_count": cnt,
                "router": router, "input_seed": seed, "weights_seed": 5252}
        save(name, meta, x=u16(d["hidden_states"]), topk_ids=d["topk_ids"].numpy(),
             topk_weights=d["topk_weights"].numpy(), w13=w["w13"].numpy(), w13_sf=u8(w["w13_sf"]),
             w13_gs=w["w13_gs"].numpy(), w2=w["w2"].numpy(), w2_sf=u8(w["w2_sf"]),
             w2_gs=w["w2_gs"].numpy(), post_norm_w=u16(w["post_norm_w"]), out=u16(out))

    # ---- 4. BASELINE config 1 at full size: weights by digest, inputs and output stored.
    shape = synth.CONFIGS["cfg1"]
    w = synth.baseline_weights(shape, seed=5252)
    _check_against_reference_quantize(nvfp4, synth, shape, w, seed=5252)
    d = synth.baseline_input(shape, 16, seed=1016)
    out = run_ref(w, d, shape.inter)
    meta = {"E": 8, "K": 2, "H": 1024, "I": 512, "T": 16, "local_start": 0, "local_count": 8,
            "router": "normal", "input_seed": 1016, "weights_seed": 5252,
            "sha256": {k: sha(v) for k, v in w.items()}}
    save("cfg1_t16", meta, x=u16(d["hidden_states"]), topk_ids=d["topk_ids"].numpy(),
         topk_weights=d["topk_weights"].numpy(), out=u16(out))

    # ---- 5. the reference problem's own generators at a reduced shape (ep: 4 of 16 local).
    reference.N_EXPERTS, reference.D_HIDDEN, reference.D_EXPERT = 16, 128, 128
    reference.ROUTED_PER_TOKEN = 4
    reference.LOCAL = {"ep8": (0, 4), "full": (0, 16)}
    wref = reference.generate_weights(5252, device="cpu")
    shape = synth.MoEShape(16, 4, 128, 128, local_start=0, local_count=4, router="reference")
    wsyn = synth.reference_weights(shape, seed=5252)
    for k in wref:
        assert torch.equal(u8t(wref[k]), u8t(wsyn[k])), f"synth.reference_weights differs: {k}"
    for bs, dist, seed in ((9, "normal", 21), (6, "skewed", 22), (1, "normal", 23)):
        dref = reference.generate_input(bs, "ep8", seed, dist=dist, device="cpu")
        dsyn = synth.reference_input(shape, bs, seed, dist=dist)
        for k in ("hidden_states", "topk_ids", "topk_weights"):
            assert torch.equal(u8t(dref[k]), u8t(dsyn[k])), f"synth.reference_input differs: {k}"
        out = reference.ref_kernel(dref, wref)
        ok, msg = reference.check_implementation(dref, out, wref)
        assert ok, msg
        lo, cnt = 0, 4
        meta = {"E": 16, "K": 4, "H": 128, "I": 128, "T": bs, "local_start": lo, "local_count": cnt,
                "dist": dist, "input_seed": seed, "weights_seed": 5252, "generator": "reference"}
        save(f"refgen_{dist}_bs{bs}", meta, x=u16(dref["hidden_states"]),
             topk_ids=dref["topk_ids"].numpy(), topk_weights=dref["topk_weights"].numpy(),
             out=u16(out))
    # ref_kernel only reads the local experts [0, 4): store those, with the digest of all 16.
    sl = slice(0, 4)
    save("refgen_weights", {"experts_stored": [0, 4], "E": 16,
                            "sha256": {k: sha(v) for k, v in wref.items()}},
         w13=wref["w13"][sl].numpy(), w13_sf=u8(wref["w13_sf"][sl]), w13_gs=wref["w13_gs"][sl].numpy(),
         w2=wref["w2"][sl].numpy(), w2_sf=u8(wref["w2_sf"][sl]), w2_gs=wref["w2_gs"][sl].numpy(),
         post_norm_w=u16(wref["post_norm_w"]))

    # ---- 6. checks.compare known answers (pass, overall fail, row fail, NaN).
    import checks as ck
    g = torch.Generator().manual_seed(5)
    ref_t = torch.randn((6, 64), generator=g).to(torch.bfloat16)
    noise = torch.randn((6, 64), generator=g)
    variants = {
        "pass": (ref_t.float() + 0.005 * noise).to(torch.bfloat16),
        "overall": (ref_t.float() + 0.05 * noise).to(torch.bfloat16),
        "row": ref_t.clone(),
        "nan": ref_t.clone(),
    }
    variants["row"][3] = (ref_t[3].float() * 1.2).to(torch.bfloat16)
    variants["nan"][1, 2] = float("nan")
    res = {k: bool(ck.compare(v, ref_t, 1.5e-2)[0]) for k, v in variants.items()}
    save("compare_kat", {"results": res}, ref=u16(ref_t), **{k: u16(v) for k, v in variants.items()})

    # ---- 7. router top-k: the reference's own routing step (generate_input, reference.py:72-84,
    # with a rank other than "busiest" so the ids stay unrotated) on scores drawn as it draws
    # them (synth.reference_scores, checked against the reference's hidden states), at the
    # reference problem's E=256, K=8; plus the softmax router of the synthetic configs
    # (torch softmax -> topk -> renormalise) at E=128, K=8.
    reference.N_EXPERTS, reference.D_HIDDEN, reference.ROUTED_PER_TOKEN = 256, 128, 8
    reference.LOCAL = {"ep8": (0, 32)}
    rshape = synth.MoEShape(256, 8, 128, 128, local_start=0, local_count=32, router="reference")
    for bs, dist, seed in ((7, "normal", 31), (5, "skewed", 32)):
        dref = reference.generate_input(bs, "ep8", seed, dist=dist, rank="plain", device="cpu")
        x, scores = synth.reference_scores(rshape, bs, seed, dist)
        assert torch.equal(u8t(x), u8t(dref["hidden_states"])), "synth.reference_scores differs"
        save(f"router_{dist}_bs{bs}", {"E": 256, "K": 8, "mode": "renorm", "seed": seed, "dist": dist},
             scores=scores.numpy(), topk_ids=dref["topk_ids"].numpy(), topk_weights=dref["topk_weights"].numpy())
    g = torch.Generator().manual_seed(33)
    logits = torch.randn((9, 128), generator=g)
    top = torch.softmax(logits, dim=-1).topk(8, dim=-1)
    save("router_softmax_bs9", {"E": 128, "K": 8, "mode": "softmax", "seed": 33},
         scores=logits.numpy(), topk_ids=top.indices.to(torch.int32).numpy(),
         topk_weights=(top.values / top.values.sum(-1, keepdim=True)).float().numpy())
    return 0


def u8t(t: torch.Tensor) -> torch.Tensor:
    return t.contiguous().view(torch.uint8)


def _check_against_reference_quantize(nvfp4, synth, shape, w, seed):
    """Re-draw the fp32 weights exactly as synth.baseline_weights does and quantise them with the
    reference's nvfp4.quantize: the bytes must be identical."""
    g = torch.Generator().manual_seed(seed)
    H, I = shape.hidden, shape.inter
    for j in range(shape.n_experts):
        a = torch.randn((2 * I, H), generator=g) * 0.02
        p, sf, gs = nvfp4.quantize(a)
        assert torch.equal(p, w["w13"][j]) and torch.equal(u8t(sf), u8t(w["w13_sf"][j])) \
            and float(gs) == float(w["w13_gs"][j]), f"w13 expert {j} differs from nvfp4.quantize"
        b = torch.randn((H, I), generator=g) * 0.02
        p, sf, gs = nvfp4.quantize(b)
        assert torch.equal(p, w["w2"][j]) and torch.equal(u8t(sf), u8t(w["w2_sf"][j])) \
            and float(gs) == float(w["w2_gs"][j]), f"w2 expert {j} differs from nvfp4.quantize"


if __name__ == "__main__":
    sys.exit(main())
