"""CPU check of the in-register dequantisation plan of the tcgen05 kernel (csrc/layout.cuh
permute_codes, csrc/gemm_tc.cu dequant8), restated here in numpy: for every code value in
every one of the 8 element positions of a word, the extracted bf16 must be the E2M1 value
times 2^-126 exactly, and times the scale table entry (e4m3 * 2^60) exactly e2m1 * sf * 2^-66.
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import moe_oracle as orc

POS = [(6, 7, 8, 15), (22, 23, 24, 31), (2, 3, 4, 11), (18, 19, 20, 27),
       (28, 29, 30, 5), (12, 13, 14, 21), (0, 1, 10, 9), (16, 17, 26, 25)]
MASK = 0x81C081C0


def permute_codes(w: int) -> int:
    out = 0
    for k in range(8):
        nib = (w >> (4 * k)) & 0xF
        for b in range(4):
            out |= ((nib >> b) & 1) << POS[k][b]
    return out


def rotl(x, n):
    return ((x << n) | (x >> (32 - n))) & 0xFFFFFFFF


def extract(w: int):
    r0 = w & MASK
    r1 = rotl(w, 4) & MASK
    r2 = rotl(w, 10) & MASK
    r3 = ((w << 6) & 0x80C080C0) | ((w >> 2) & 0x01000100)
    return [r0, r1, r2, r3]


def bf16_pair_values(r: int):
    lo = np.array([r & 0xFFFF], dtype=np.uint16)
    hi = np.array([r >> 16], dtype=np.uint16)
    return float(orc.bf16_to_f32(lo)[0]), float(orc.bf16_to_f32(hi)[0])


def test_permutation_is_a_bijection_of_bits():
    used = sorted(p for k in POS for p in k)
    assert used == list(range(32))


def test_every_code_in_every_position_decodes_exactly():
    e2m1 = orc.e2m1_table()
    rng = np.random.default_rng(0)
    for k in range(8):
        for code in range(16):
            for _ in range(4):
                others = int(rng.integers(0, 1 << 32))
                w = (others & ~(0xF << (4 * k))) | (code << (4 * k))
                regs = extract(permute_codes(w))
                vals = [v for r in regs for v in bf16_pair_values(r)]   # elements 0..7
                expect = [float(e2m1[(w >> (4 * j)) & 0xF]) * 2.0 ** -126 for j in range(8)]
                assert vals == expect, (k, code, hex(w))


def test_scaled_product_is_exact_in_bf16():
    """raw (e2m1 * 2^-126) x (sf * 2^60) rounded to bf16 == e2m1 * sf * 2^-66 for every finite
    e4m3 scale and every code: the product has at most 6 significant bits."""
    e2m1 = orc.e2m1_table().astype(np.float64)
    sf = orc.e4m3_table().astype(np.float64)
    finite = np.isfinite(sf)
    prod = (e2m1[:, None] * 2.0 ** -126) * (sf[None, finite] * 2.0 ** 60)
    t = torch.from_numpy(prod.astype(np.float32)).to(torch.bfloat16).double().numpy()
    np.testing.assert_array_equal(t, e2m1[:, None] * sf[None, finite] * 2.0 ** -66)
    # the raw code values themselves (including the 2^-127 subnormal of code 1) are exact bf16
    raw = torch.from_numpy((e2m1 * 2.0 ** -126).astype(np.float32)).to(torch.bfloat16).double().numpy()
    np.testing.assert_array_equal(raw, e2m1 * 2.0 ** -126)
