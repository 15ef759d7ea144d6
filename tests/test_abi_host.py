"""CPU-side checks of the C ABI and the host wrapper: the library loads, exports exactly what
include/muse_moe.h declares, validates arguments before touching the GPU, and the host path
refuses CPU tensors (there is no fallback). No kernel is launched here."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def lib(pkg):
    import __graft_entry__
    if not pkg.library_path().exists():
        __graft_entry__.build()
    return pkg.load_library()


def declared_symbols() -> set[str]:
    text = (REPO / "include" / "muse_moe.h").read_text()
    return set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\**(muse_moe_\w+)\s*\(", text, flags=re.M))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert {"muse_moe_forward", "muse_moe_route", "muse_moe_prepare_weights",
            "muse_moe_workspace_size", "muse_moe_version", "muse_moe_error_string"} <= syms


def test_library_exports_every_declared_symbol(lib, pkg):
    from muse_moe_w4a16_b200 import _lib
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version_and_errors(lib):
    assert lib.muse_moe_version() >= 1
    assert b"success" in lib.muse_moe_error_string(0)
    assert b"workspace" in lib.muse_moe_error_string(-3)


def test_workspace_size_grows_with_tokens(pkg):
    from muse_moe_w4a16_b200 import _lib
    a = _lib.workspace_size(1, 8, 128, 2048, 768)
    b = _lib.workspace_size(32, 8, 128, 2048, 768)
    assert 0 < a < b
    assert b % 256 == 0


@pytest.mark.parametrize("args,code", [
    ((1, 8, 128, 2000, 768), -2),   # hidden not a multiple of 128
    ((1, 32, 128, 2048, 768), -2),  # top_k > 16
    ((1, 8, 512, 2048, 768), -2),   # too many local experts
    ((-1, 8, 128, 2048, 768), -1),
])
def test_workspace_size_rejects_bad_shapes(lib, args, code):
    n = ctypes.c_size_t()
    assert lib.muse_moe_workspace_size(*args, ctypes.byref(n)) == code


def test_forward_rejects_null_pointers_before_any_launch(lib):
    rc = lib.muse_moe_forward(None, None, None, 4, 8, 0, 32, 2048, 768, None, None, None, None,
                              None, None, None, None, None, 0, None)
    assert rc == -1
    # zero tokens is a valid empty call and launches nothing
    rc = lib.muse_moe_forward(None, None, None, 0, 8, 0, 32, 2048, 768, None, None, None, None,
                              None, None, None, None, None, 0, None)
    assert rc == 0


def test_route_rejects_bad_arguments(lib):
    assert lib.muse_moe_route(None, 4, 8, 0, 32, None, None, None, None) == -1
    assert lib.muse_moe_route(None, 4, 8, 0, 1000, None, None, None, None) == -2


def test_router_rejects_bad_arguments(lib):
    f = lib.muse_moe_router_topk
    assert f(None, 4, 256, 8, 2, None, None, None) == -1      # unknown mode
    assert f(None, -1, 256, 8, 0, None, None, None) == -1     # negative tokens
    assert f(None, 4, 256, 17, 0, None, None, None) == -2     # K > 16
    assert f(None, 4, 4, 8, 0, None, None, None) == -2        # K > E
    assert f(None, 4, 2048, 8, 0, None, None, None) == -2     # E > 1024
    assert f(None, 0, 256, 8, 0, None, None, None) == 0       # empty batch: nothing to do
    assert f(None, 4, 256, 8, 0, None, None, None) == -1      # null pointers


def test_host_path_refuses_cpu_tensors(pkg):
    from muse_moe_w4a16_b200 import synth
    shape = synth.MoEShape(4, 2, 128, 128)
    w = synth.baseline_weights(shape)
    with pytest.raises(pkg.MuseError):
        pkg.prepare(w)
    d = synth.baseline_input(shape, 3, seed=0)
    with pytest.raises(pkg.MuseError):
        pkg.kernel_fn(d, {"inter": 128, "hidden": 128, "n_experts": 4})
    from muse_moe_w4a16_b200 import layer
    with pytest.raises(pkg.MuseError):   # the layer-plus-exchange call checks the same way
        layer.kernel_fn_exchange(d, {"inter": 128, "hidden": 128, "n_experts": 4},
                                 torch.zeros(3, 128), {})


def test_product_path_does_not_import_oracle():
    pkg_dir = REPO / "muse-moe-w4a16_b200"
    for f in pkg_dir.rglob("*.py"):
        for line in f.read_text().splitlines():
            assert not re.match(r"\s*(from|import)\s+oracle\b", line), f"{f.name}: {line}"


@pytest.mark.parametrize("T,K,E,H,I,launches,path", [
    (1, 8, 128, 2048, 768, 1, 2), (16, 8, 128, 2048, 768, 1, 2), (32, 8, 128, 2048, 768, 3, 1),
    (128, 8, 256, 7168, 2048, 3, 1), (129, 8, 256, 7168, 2048, 5, 0),
    (128, 8, 32, 4096, 4096, 5, 0), (4, 8, 32, 4096, 4096, 1, 2), (0, 8, 32, 4096, 4096, 0, 2),
])
def test_launch_plan(pkg, T, K, E, H, I, launches, path):
    """<= 128 pairs with a token tile <= 32: the whole layer in one cooperative launch;
    <= 1024 pairs: GEMM1 routes and gathers x itself, then GEMM2 and the combine; larger
    batches: route, gather, GEMM1, GEMM2, combine."""
    from muse_moe_w4a16_b200 import _lib
    plan = _lib.launch_plan(T, K, E, H, I)
    assert plan["launches"] == launches and plan["path"] == path
    assert plan["n_box"] in (16, 32, 64, 128) and plan["stages"] >= 2


def test_profiled_forward_rejects_missing_events(lib):
    from muse_moe_w4a16_b200 import _lib
    ev = (ctypes.c_void_p * 5)(1, 2, 3, 4, None)
    args = [None] * 3 + [1, 2, 0, 8, 256, 256] + [None] * 9 + [0, None]
    assert lib.muse_moe_forward_profiled(*args, None) == _lib.MUSE_ERR_INVALID_ARGUMENT
    assert lib.muse_moe_forward_profiled(*args, ev) == _lib.MUSE_ERR_INVALID_ARGUMENT


def test_peer_allreduce_rejects_bad_arguments(lib):
    """Argument checks of the expert-parallel exchange run before any device work."""
    from muse_moe_w4a16_b200 import _lib
    u64 = ctypes.c_uint64 * 2
    s0, s1, flags = u64(0x1000, 0x2000), u64(0x1100, 0x2100), u64(0x3000, 0x4000)
    f = lib.muse_moe_peer_allreduce_bf16
    bad = _lib.MUSE_ERR_INVALID_ARGUMENT
    out = ctypes.c_void_p(0x5000)
    assert f(s0, s1, flags, 2, 2, 64, out, None) == bad                 # rank out of range
    assert f(s0, s1, flags, 9, 0, 64, out, None) == bad                 # more than 8 ranks
    assert f(s0, s1, flags, 2, 0, 60, out, None) == bad                 # n not a multiple of 8
    assert f(s0, s1, flags, 2, 0, 64, None, None) == bad                # no output
    assert f(u64(0x1000, 0), s1, flags, 2, 0, 64, out, None) == bad     # null peer share
    assert f(u64(0x1004, 0x2000), s1, flags, 2, 0, 64, out, None) == bad  # misaligned share


def test_forward_exchange_rejects_bad_arguments(lib):
    """The layer-plus-exchange call checks its exchange arguments before any device work: the
    share buffer it writes is named by expect_parity, so the parity must be 0 or 1; the exchange
    modes of the decode layout are 0 and 2."""
    from muse_moe_w4a16_b200 import _lib
    u64 = ctypes.c_uint64 * 2
    s0, s1, flags = u64(0x1000, 0x2000), u64(0x1100, 0x2100), u64(0x3000, 0x4000)
    f = lib.muse_moe_forward_exchange_bf16
    bad = _lib.MUSE_ERR_INVALID_ARGUMENT
    layer = [None] * 3 + [1, 8, 0, 8, 16, 256, 256] + [None] * 7 + [None, 0]

    def call(shares0=s0, ranks=2, rank=0, mode=0, parity=1, out=0x5000):
        return f(*layer, shares0, s1, flags, None, ranks, rank, mode, parity, 0, out, None)

    assert call(rank=2) == bad                    # rank out of range
    assert call(ranks=9) == bad                   # more than 8 ranks
    assert call(parity=-1) == bad                 # the share buffer must be named
    assert call(mode=1) == bad                    # not a decode-layout mode
    assert call(out=None) == bad                  # no output
    assert call(out=0x5004) == bad                # misaligned output
    assert call(shares0=u64(0x1000, 0)) == bad    # null peer share
    assert call(shares0=u64(0x1008, 0x2000)) == bad   # misaligned share


def test_launch_plan_counts_only_local_pairs_per_expert(pkg):
    """On an expert-parallel slice the token tile follows the pairs a local expert can expect
    (T*K / model experts), not T*K / local experts: the reference problem's ep8 slice at bs 256
    keeps the 16-token decode tile; an unsharded call of the same size per expert does not."""
    from muse_moe_w4a16_b200 import _lib
    ep = _lib.launch_plan(256, 8, 32, 4096, 4096, 256)
    whole = _lib.launch_plan(256, 8, 32, 4096, 4096)
    assert ep["n_box"] == 16 and whole["n_box"] == 128
    assert _lib.launch_plan(256, 8, 32, 4096, 4096, 0) == whole
    with pytest.raises(Exception):
        _lib.launch_plan(256, 8, 32, 4096, 4096, 16)   # fewer model experts than local ones
