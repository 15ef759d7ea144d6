"""An expert-parallel call that raises before its exchange leaves the exchange in step: the
host's generation count advances only after the exchange kernel was launched, so the next call
still writes the share buffer the device reads and matches the oracle (decode and prefill).
One GPU, a one-rank process group in a child process."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import moe_oracle as orc
from tests.gpu_util import oracle_out, to_numpy_weights

pytestmark = pytest.mark.gpu
TOL = 1.5e-2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _child(port, result_dir):
    import datetime
    import sys
    from pathlib import Path
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=dev, timeout=datetime.timedelta(seconds=60))
    try:
        sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
        import __graft_entry__
        __graft_entry__.load_package()
        from muse_moe_w4a16_b200 import _lib, ep, synth
        shape = synth.MoEShape(16, 4, 256, 256, router="normal")
        w = {k: v.to(dev) for k, v in synth.baseline_weights(shape, seed=4).items()}
        d = synth.baseline_input(shape, 12, seed=8)
        np.save(os.path.join(result_dir, "ids.npy"), d["topk_ids"].numpy())
        d = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in d.items()}
        bad = {**d, "hidden_states": d["hidden_states"].float()}   # rejected before any launch
        moe = ep.ExpertParallelMoE(w)
        outs = []
        for call in (moe.forward_replicated, moe.forward_sharded):
            first = call(d)
            for _ in range(3):   # a failed call between good ones, on both buffer parities
                with pytest.raises(_lib.MuseError):
                    call(bad)
                again = call(d)
                torch.cuda.synchronize()
                assert torch.equal(again.view(torch.int16), first.view(torch.int16))
            outs.append(first.view(torch.uint16).cpu().numpy())
        moe.check_status()
        np.save(os.path.join(result_dir, "outs.npy"), np.stack(outs))
    finally:
        dist.destroy_process_group()


def test_failed_call_keeps_the_exchange_in_step(pkg, tmp_path):
    import importlib
    synth = importlib.import_module("muse_moe_w4a16_b200.synth")
    ctx = mp.get_context("spawn")
    p = ctx.Process(target=_child, args=(_free_port(), str(tmp_path)))
    p.start()
    p.join(timeout=300)
    if p.is_alive():
        p.kill()
        pytest.fail("child did not finish")
    assert p.exitcode == 0
    outs = np.load(tmp_path / "outs.npy")
    shape = synth.MoEShape(16, 4, 256, 256, router="normal")
    d = synth.baseline_input(shape, 12, seed=8)
    ref = oracle_out(d, to_numpy_weights(synth.baseline_weights(shape, seed=4)))
    for o in outs:   # decode and prefill rows of the same tokens
        ok, msg, _, _ = orc.compare(o, ref, TOL)
        assert ok, msg
