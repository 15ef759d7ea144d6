"""muse_moe_forward_noalloc: the layer call for callers that cannot allocate device memory.

Such callers (code inside another runtime's execution callback whose host framework owns all
device allocations, or a serving loop that must not call cudaMalloc / cudaFree because they
can synchronise the device) get an entry point whose scratch is a fixed 32 MiB array owned by
the library. These tests call it through the C ABI and check it against muse_moe_forward, with
the same tolerance as the other layer tests, on two calls in a row (the second call finds the
first one's leftovers in the shared array). This file is named so pytest collects it last.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from tests.gpu_util import bits, to_device

pytestmark = pytest.mark.gpu
TOL = 1.5e-2
DEV = torch.device("cuda:0")


def _noalloc_args(pkg, d, st):
    """Argument tuple of muse_moe_forward_noalloc for the device inputs d and prepared state st,
    with the local experts' weights offset as layer.kernel_fn offsets them."""
    cfg = d["config"]
    x = d["hidden_states"].contiguous()
    ids = d["topk_ids"].to(torch.int32).contiguous()
    wts = d["topk_weights"].to(torch.float32).contiguous()
    T, H = x.shape
    K = ids.shape[1]
    I = st["inter"]
    lo, cnt = int(cfg["local_start"]), int(cfg["local_count"])
    out = torch.full((T, H), float("nan"), dtype=torch.bfloat16, device=DEV)
    w13_e, w13sf_e, w2_e, w2sf_e = I * H, I * H // 8, H * I // 2, H * I // 16
    args = (x.data_ptr(), ids.data_ptr(), wts.data_ptr(), T, K, lo, cnt, H, I,
            st["w13"].data_ptr() + lo * w13_e, st["w13_sf"].data_ptr() + lo * w13sf_e,
            st["w13_gs"].data_ptr() + lo * 4,
            st["w2"].data_ptr() + lo * w2_e, st["w2_sf"].data_ptr() + lo * w2sf_e,
            st["w2_gs"].data_ptr() + lo * 4,
            st["post_norm_w"].data_ptr(), out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    return args, out, (x, ids, wts)


@pytest.mark.parametrize("workload,T", [("cfg2", 32), ("cfg3", 200), ("ep", 5)])
def test_noalloc_matches_forward_on_two_calls(pkg, workload, T):
    from muse_moe_w4a16_b200 import _lib, synth
    shape = synth.CONFIGS.get(workload) or synth.MoEShape(64, 8, 1024, 512, local_start=16,
                                                          local_count=16, router="uniform")
    w = synth.baseline_weights(shape, seed=31, device=DEV)
    st = pkg.prepare(w)
    dd = to_device(synth.baseline_input(shape, T, seed=T + 5), DEV)
    ref = bits(pkg.kernel_fn(dd, st))
    lib = _lib.load_library()
    for call in range(2):
        args, out, _keep = _noalloc_args(pkg, dd, st)
        rc = lib.muse_moe_forward_noalloc(*args)
        assert rc == 0, _lib.load_library().muse_moe_error_string(rc)
        torch.cuda.synchronize()
        assert _lib.device_status() == 0
        ok, msg, err, _ = orc.compare(bits(out), ref, TOL)
        assert ok, f"call {call}: {msg}"


def test_noalloc_refuses_batches_beyond_its_scratch(pkg):
    """A batch whose workspace exceeds the 32 MiB array is refused before any launch, with its
    own error code and message; the output is left untouched."""
    from muse_moe_w4a16_b200 import _lib, synth
    shape = synth.CONFIGS["cfg4"]
    T = 88
    assert _lib.workspace_size(T, shape.top_k, shape.n_local, shape.hidden, shape.inter) > 32 << 20
    lib = _lib.load_library()
    x = torch.zeros((T, shape.hidden), dtype=torch.bfloat16, device=DEV)
    ids = torch.zeros((T, shape.top_k), dtype=torch.int32, device=DEV)
    wts = torch.zeros((T, shape.top_k), dtype=torch.float32, device=DEV)
    out = torch.full((T, shape.hidden), 7.0, dtype=torch.bfloat16, device=DEV)
    dummy = torch.zeros(16, dtype=torch.uint8, device=DEV)
    p = dummy.data_ptr()
    rc = lib.muse_moe_forward_noalloc(x.data_ptr(), ids.data_ptr(), wts.data_ptr(), T, shape.top_k, 0,
                                      shape.n_local, shape.hidden, shape.inter, p, p, p, p, p, p, p,
                                      out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.MUSE_ERR_SCRATCH_LIMIT
    assert b"32 MiB" in lib.muse_moe_error_string(rc)
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())
