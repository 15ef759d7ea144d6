"""muse-moe-w4a16 for B200: a routed W4A16 (NVFP4-weight, bf16-activation) MoE layer.

The public surface mirrors the reference's plugin interface (baseline.py:27-52, 82-151 and
reference.py:93):

* ``prepare(weights) -> state``         untimed weight repack into the kernels' tile layout
* ``kernel_fn(data, state) -> Tensor``  the timed layer call, bf16 [T, H] on the GPU
* ``moe_forward(data, weights)``        prepare-once-and-call, the ref_kernel signature
* ``route_topk(scores, K)``             the caller-side router: topk_ids / topk_weights on the GPU

The compute runs in hand-written sm_100a CUDA kernels behind a C ABI (include/muse_moe.h),
loaded from the in-tree shared library ``libmusemoe.so``. There is no CPU fallback: without
the library (or without a GPU) every entry point raises.
"""

from .layer import Config, Inputs, Weights, kernel_fn, moe_forward, prepare, route_topk  # noqa: F401
from ._lib import MuseError, library_path, load_library  # noqa: F401

__all__ = ["prepare", "kernel_fn", "moe_forward", "route_topk", "Weights", "Inputs", "Config",
           "MuseError", "library_path", "load_library"]
