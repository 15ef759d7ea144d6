"""ctypes binding of the C ABI in include/muse_moe.h (libmusemoe.so, built in-tree).

This is the only place the Python side touches native code. There is deliberately no
fallback: if the library is missing or fails to load, every entry point raises MuseError.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_NAME = "libmusemoe.so"

# Every symbol include/muse_moe.h declares, with (restype, argtypes).
_P = ctypes.c_void_p
_I = ctypes.c_int
_SIZE_P = ctypes.POINTER(ctypes.c_size_t)
SIGNATURES: dict[str, tuple] = {
    "muse_moe_version": (_I, []),
    "muse_moe_error_string": (ctypes.c_char_p, [_I]),
    "muse_moe_workspace_size": (_I, [_I, _I, _I, _I, _I, _SIZE_P]),
    "muse_moe_workspace_offsets": (_I, [_I, _I, _I, _I, _I, _SIZE_P]),
    "muse_moe_device_status": (_I, [ctypes.POINTER(ctypes.c_int), _I]),
    "muse_moe_prepare_weights": (_I, [_P, _P, _P, _P, _I, _I, _I, _P, _P, _P, _P, _P]),
    "muse_moe_route": (_I, [_P, _I, _I, _I, _I, _P, _P, _P, _P]),
    "muse_moe_router_topk": (_I, [_P, _I, _I, _I, _I, _P, _P, _P]),
    "muse_moe_forward": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _I,
                              _P, _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P]),
    "muse_moe_forward_profiled": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _I,
                                       _P, _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P,
                                       ctypes.POINTER(_P)]),
    "muse_moe_launch_plan": (_I, [_I, _I, _I, _I, _I, ctypes.POINTER(_I)]),
    "muse_moe_launch_plan_ex": (_I, [_I, _I, _I, _I, _I, _I, ctypes.POINTER(_I)]),
    "muse_moe_forward_ex": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _I, _I,
                                 _P, _P, _P, _P, _P, _P, _P, _P, _I, _P, ctypes.c_size_t, _P,
                                 ctypes.POINTER(_P)]),
    "muse_moe_forward_partial": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _I,
                                      _P, _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P]),
    "muse_moe_cast_bf16": (_I, [_P, _P, ctypes.c_size_t, _P]),
    "muse_moe_peer_allreduce_bf16": (_I, [ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64),
                                          ctypes.POINTER(ctypes.c_uint64), _I, _I, ctypes.c_size_t, _P, _P]),
    "muse_moe_peer_reduce_scatter_bf16": (_I, [ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64),
                                               ctypes.POINTER(ctypes.c_uint64), _I, _I, ctypes.c_size_t, _P, _P]),
    "muse_moe_peer_exchange_bf16": (_I, [ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64),
                                         ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64),
                                         _I, _I, ctypes.c_size_t, _I, _I, ctypes.c_longlong, _P, _P]),
    "muse_moe_forward_exchange_bf16": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _I, _I,
                                            _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_size_t,
                                            ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64),
                                            ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64),
                                            _I, _I, _I, _I, ctypes.c_longlong, _P, _P]),
    "muse_moe_ep_dispatch": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, ctypes.POINTER(_I),
                                  ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64),
                                  ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64),
                                  _P, ctypes.c_longlong, _P]),
    "muse_moe_peer_routed_reduce_scatter_bf16": (_I, [ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64),
                                                      ctypes.POINTER(ctypes.c_uint64), _I, _I, _I, _I, _P, _I,
                                                      ctypes.c_longlong, _P, _P]),
    "muse_moe_forward_noalloc": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _I,
                                      _P, _P, _P, _P, _P, _P, _P, _P, _P]),
}

# Return codes (include/muse_moe.h).
MUSE_OK = 0
MUSE_ERR_INVALID_ARGUMENT = -1
MUSE_ERR_UNSUPPORTED_SHAPE = -2
MUSE_ERR_WORKSPACE_TOO_SMALL = -3
MUSE_ERR_NO_DEVICE = -4
MUSE_ERR_DEVICE_TIMEOUT = -5
MUSE_ERR_SCRATCH_LIMIT = -6


class MuseError(RuntimeError):
    """A non-zero return code from the native library (or the library is unavailable)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"muse_moe error {code}: {message}")
        self.code = code


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def library_path() -> Path:
    return Path(__file__).resolve().parent / LIB_NAME


def load_library() -> ctypes.CDLL:
    """Open libmusemoe.so (once) and attach the C signatures. Raises MuseError if absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = library_path()
            if not path.exists():
                raise MuseError(MUSE_ERR_NO_DEVICE,
                                f"{path} is not built; run `python muse-moe-w4a16_b200/build.py` "
                                "(or __graft_entry__.build()) -- there is no CPU fallback")
            lib = ctypes.CDLL(str(path))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(rc: int) -> None:
    """Raise MuseError for a non-zero return code."""
    if rc != MUSE_OK:
        msg = load_library().muse_moe_error_string(rc)
        raise MuseError(rc, msg.decode() if msg else "unknown")


def call(name: str, *args) -> None:
    """Call an int-returning entry point and raise on failure."""
    check(getattr(load_library(), name)(*args))


def workspace_offsets(tokens: int, top_k: int, local_count: int, hidden: int, inter: int) -> dict:
    """Byte offsets of the scratch buffers inside the workspace (include/muse_moe.h)."""
    arr = (ctypes.c_size_t * 9)()
    call("muse_moe_workspace_offsets", tokens, top_k, local_count, hidden, inter, arr)
    names = ("offsets", "pair_order", "pair_row", "xs", "inter", "ypart", "ssq", "sync", "total")
    return dict(zip(names, (int(v) for v in arr)))


def device_status(reset: bool = True) -> int:
    """The kernels' sticky timeout status on the current device (synchronises)."""
    st = ctypes.c_int(0)
    call("muse_moe_device_status", ctypes.byref(st), int(reset))
    return int(st.value)


def workspace_size(tokens: int, top_k: int, local_count: int, hidden: int, inter: int) -> int:
    n = ctypes.c_size_t(0)
    call("muse_moe_workspace_size", tokens, top_k, local_count, hidden, inter, ctypes.byref(n))
    return int(n.value)


def launch_plan(tokens: int, top_k: int, local_count: int, hidden: int, inter: int,
                n_experts: int = 0) -> dict:
    """Kernels, token tile, stages and routing mode of one forward call (include/muse_moe.h);
    n_experts: experts in the whole model (0: local_count)."""
    arr = (ctypes.c_int * 5)()
    call("muse_moe_launch_plan_ex", tokens, top_k, local_count, n_experts, hidden, inter, arr)
    return {"launches": arr[0], "n_box": arr[1], "stages": arr[2], "path": int(arr[3]),
            "fused": arr[3] == 2, "route_inline": arr[3] >= 1, "pair_tiles": bool(arr[4])}
