"""Expert parallelism on 2+ GPUs of one node: the decode exchange (all-reduce) and the prefill
exchange (reduce-scatter, after an NCCL all-gather of the inputs) over NVLink peer memory,
every rank's output against the oracle over all experts. Skipped with fewer than two GPUs."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import moe_oracle as orc
from tests.gpu_util import oracle_out, to_numpy_weights

pytestmark = pytest.mark.gpu
TOL = 1.5e-2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shape():
    import importlib
    synth = importlib.import_module("muse_moe_w4a16_b200.synth")
    return synth, synth.MoEShape(32, 8, 512, 256, router="normal")


def _rank_main(rank, world, port, T, result_dir):
    import datetime
    import sys
    from pathlib import Path
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
        import __graft_entry__
        __graft_entry__.load_package()
        from muse_moe_w4a16_b200 import ep
        synth, shape = _shape()
        w = synth.baseline_weights(shape, seed=3)            # same bytes on every rank (CPU generator)
        w = {k: v.to(dev) for k, v in w.items()}
        d = synth.baseline_input(shape, T, seed=T)
        d = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in d.items()}
        moe = ep.ExpertParallelMoE(w)
        rep = moe.forward_replicated(d)
        for _ in range(2):   # both share buffers (generation parity) and a fresh generation
            again = moe.forward_replicated(d)
            assert torch.equal(again.view(torch.int16), rep.view(torch.int16))
        graphs = moe.decode_graphs(d)   # captured decode calls, replayed in parity order
        for _ in range(3):
            got = graphs.replay()
            torch.cuda.synchronize()
            assert torch.equal(got.view(torch.int16), rep.view(torch.int16))
        again = moe.forward_replicated(d)   # eager calls and replays share the generation count
        assert torch.equal(again.view(torch.int16), rep.view(torch.int16))
        t_r = T // world
        sl = slice(rank * t_r, (rank + 1) * t_r)
        mine = {**d, "hidden_states": d["hidden_states"][sl], "topk_ids": d["topk_ids"][sl],
                "topk_weights": d["topk_weights"][sl]}
        shard = moe.forward_sharded(mine)
        again = moe.forward_sharded(mine)     # the other share buffer
        assert torch.equal(again.view(torch.int16), shard.view(torch.int16))
        again = moe.forward_replicated(d)     # decode and prefill calls share the generation count
        assert torch.equal(again.view(torch.int16), rep.view(torch.int16))
        # the two-round exchange (reduce-scatter, then all-gather of the bf16 slices) gives the
        # same bits: every element is still summed once, in rank order
        moe.one_round_bytes = 0
        assert moe.exchange_mode(T * shape.hidden) == 2
        for _ in range(2):
            again = moe.forward_replicated(d)
            assert torch.equal(again.view(torch.int16), rep.view(torch.int16))
        graphs2 = moe.decode_graphs(d)
        for _ in range(3):
            got = graphs2.replay()
            torch.cuda.synchronize()
            assert torch.equal(got.view(torch.int16), rep.view(torch.int16))
        moe.check_status()
        del graphs, graphs2
        torch.cuda.synchronize()
        np.save(os.path.join(result_dir, f"rep{rank}.npy"), rep.view(torch.uint16).cpu().numpy())
        np.save(os.path.join(result_dir, f"shard{rank}.npy"), shard.view(torch.uint16).cpu().numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
@pytest.mark.parametrize("T", [16, 64])
def test_expert_parallel_matches_oracle(pkg, tmp_path, T):
    world = min(torch.cuda.device_count(), 4)
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, T, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    synth, shape = _shape()
    d = synth.baseline_input(shape, T, seed=T)
    ref = oracle_out(d, to_numpy_weights(synth.baseline_weights(shape, seed=3)))
    rep0 = np.load(tmp_path / "rep0.npy")
    for r in range(world):
        got = np.load(tmp_path / f"rep{r}.npy")
        ok, msg, _, _ = orc.compare(got, ref, TOL)
        assert ok, f"rank {r} replicated: {msg}"
        np.testing.assert_array_equal(got, rep0)   # every rank sums the shares in rank order
    T_used = (T // world) * world
    got = np.concatenate([np.load(tmp_path / f"shard{r}.npy") for r in range(world)])
    ok, msg, _, _ = orc.compare(got, ref[:T_used], TOL)
    assert ok, f"sharded: {msg}"
    if T_used == T:   # same tokens in the same order: the same shares, summed in the same order
        np.testing.assert_array_equal(got, rep0)
