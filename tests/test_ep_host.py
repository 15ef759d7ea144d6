"""Expert-parallel host logic on CPU ranks (gloo): the expert split and the exchange.

Each rank's local share is computed by the oracle here (its fp32 sum before the bf16 cast),
standing in for the CUDA partial forward, so what these tests check is the plumbing of
`ep.ExpertParallelMoE`: which experts a rank owns, the all-reduce of the decode layout, and the
all-gather / reduce-scatter of the prefill layout, against the single-process oracle over all
experts (the reference's ep8 layer computed in one place, reference.py:93-107).
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import moe_oracle as orc

TOL = 1.5e-2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_expert_block_partitions(pkg):
    from muse_moe_w4a16_b200 import ep
    for E, R in [(256, 8), (128, 2), (130, 4), (8, 8), (9, 2)]:
        blocks = [ep.expert_block(E, r, R) for r in range(R)]
        assert blocks[0].start == 0 and blocks[-1].stop == E
        assert all(a.stop == b.start for a, b in zip(blocks, blocks[1:]))
        assert max(map(len, blocks)) - min(map(len, blocks)) <= 1
    assert ep.expert_block(256, 3, 8) == range(96, 128)   # reference.py:22 LOCAL for rank 3
    with pytest.raises(Exception):
        ep.expert_block(4, 0, 8)


def _problem(seed: int, T: int):
    import importlib
    synth = importlib.import_module("muse_moe_w4a16_b200.synth")
    shape = synth.MoEShape(12, 3, 128, 128, router="normal")
    w = synth.baseline_weights(shape, seed=seed)
    d = synth.baseline_input(shape, T, seed=seed + T)
    wn = {k: (v.view(torch.uint8) if v.dtype == torch.float8_e4m3fn else
              v.view(torch.uint16) if v.dtype == torch.bfloat16 else v).numpy() for k, v in w.items()}
    return shape, w, d, wn


def _oracle_partial(wn, inter):
    def local(d):
        cfg = d["config"]
        out = orc.ref_kernel(d["hidden_states"].view(torch.uint16).numpy(), d["topk_ids"].numpy(),
                             d["topk_weights"].numpy(), wn, cfg["local_start"], cfg["local_count"],
                             inter, return_f32=True)
        return torch.from_numpy(np.ascontiguousarray(out))
    return local


def _oracle_cast(t: torch.Tensor) -> torch.Tensor:
    return torch.from_numpy(orc.f32_to_bf16(t.numpy())).view(torch.bfloat16)


def _rank_main(rank, world, port, layout, T, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        from pathlib import Path
        repo = Path(__file__).resolve().parent.parent
        sys.path.insert(0, str(repo))
        import __graft_entry__
        __graft_entry__.load_package()
        from muse_moe_w4a16_b200 import ep
        shape, w, d, wn = _problem(11, T)
        moe = ep.ExpertParallelMoE(w, n_experts=shape.n_experts, local_fn=_oracle_partial(wn, shape.inter),
                                   cast_fn=_oracle_cast)
        empty = {**d, "hidden_states": d["hidden_states"][:0], "topk_ids": d["topk_ids"][:0],
                 "topk_weights": d["topk_weights"][:0]}
        call = moe.forward_replicated if layout == "replicated" else moe.forward_sharded
        none = call(empty)   # an empty batch on every rank: empty result, no exchange
        assert none.shape == (0, d["hidden_states"].shape[1]) and none.dtype == torch.bfloat16
        if layout == "replicated":
            out = moe.forward_replicated(d)
        else:
            t_r = T // world
            sl = slice(rank * t_r, (rank + 1) * t_r)
            mine = {**d, "hidden_states": d["hidden_states"][sl], "topk_ids": d["topk_ids"][sl],
                    "topk_weights": d["topk_weights"][sl]}
            out = moe.forward_sharded(mine)
        np.save(os.path.join(result_dir, f"r{rank}.npy"), out.view(torch.uint16).numpy())
        np.save(os.path.join(result_dir, f"e{rank}.npy"), np.array([moe.experts.start, moe.experts.stop]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("layout,world,T", [("replicated", 2, 7), ("replicated", 3, 5),
                                            ("sharded", 2, 8), ("sharded", 4, 12)])
def test_ep_exchange_matches_single_process_oracle(pkg, tmp_path, layout, world, T):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, layout, T, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:   # a rank still running after the limit is a failure; end it
        if p.is_alive():
            p.kill()
            p.join()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    shape, w, d, wn = _problem(11, T)
    ref = orc.ref_kernel(d["hidden_states"].view(torch.uint16).numpy(), d["topk_ids"].numpy(),
                         d["topk_weights"].numpy(), wn, 0, shape.n_experts, shape.inter)
    blocks = [tuple(np.load(tmp_path / f"e{r}.npy")) for r in range(world)]
    assert blocks[0][0] == 0 and blocks[-1][1] == shape.n_experts
    if layout == "replicated":
        for r in range(world):
            ok, msg, err, _ = orc.compare(np.load(tmp_path / f"r{r}.npy"), ref, TOL)
            assert ok and err < 1e-5, msg
    else:
        got = np.concatenate([np.load(tmp_path / f"r{r}.npy") for r in range(world)])
        ok, msg, err, _ = orc.compare(got, ref, TOL)
        assert ok and err < 1e-5, msg
