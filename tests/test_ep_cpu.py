"""Expert-parallel exchange logic on CPU: world_size-2 gloo ranks run
nki_moe_7013_b200.ep.ExpertParallelMoE with CPU stand-in kernels and must
reproduce the single-process oracle MoE block on their own tokens; a rank that
leaves before a collective makes its peer fail with an error, not hang."""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _ep_worker(rank, world, port, result_dir, mode):
    sys.path[:0] = [REPO, HERE]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    from ep_reference import CpuEPKernels

    from nki_moe_7013_b200.config import Qwen3MoeConfig
    from nki_moe_7013_b200.ep import ExpertParallelMoE
    from nki_moe_7013_b200.moe import MoEWeights
    from nki_moe_7013_b200.synth import normal_bf16
    from oracle import oracle

    T, H, E, k, I = 20, 256, 32, 4, 128
    cfg = Qwen3MoeConfig(hidden_size=H, num_experts=E, num_experts_per_tok=k, moe_intermediate_size=I)
    wr = normal_bf16(1, "w_router", (E, H), 0.02)
    wgu = normal_bf16(1, "w_gate_up", (E, 2 * I, H), 0.02)
    wd = normal_bf16(1, "w_down", (E, H, I), 0.02)
    el = E // world
    local = MoEWeights(wr, wgu[rank * el:(rank + 1) * el].contiguous(), wd[rank * el:(rank + 1) * el].contiguous())
    x = normal_bf16(100 + rank, "x", (T, H))
    res = normal_bf16(200 + rank, "res", (T, H))
    moe = ExpertParallelMoE(cfg, wr, local, kernels=CpuEPKernels())
    if mode == "drop" and rank == 1:
        os._exit(0)  # leaves before the first collective
    try:
        out = moe(x, residual=res)
        ref = oracle.moe_block(x, wr, wgu, wd, k) + res.float().numpy()
        err = float(np.abs(out.float().numpy() - ref).max() / np.abs(ref).max())
        np.save(os.path.join(result_dir, f"err{rank}.npy"), np.array([err, moe.last_recv_rows]))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # the failure test expects this on the surviving rank
        with open(os.path.join(result_dir, f"exc{rank}.txt"), "w") as f:
            f.write(type(exc).__name__ + ": " + str(exc)[:200])


def test_ep_two_gloo_ranks_match_single_process_oracle(tmp_path):
    mp.start_processes(_ep_worker, args=(2, _free_port(), str(tmp_path), "ok"), nprocs=2,
                       start_method="spawn", join=True)
    errs = [np.load(tmp_path / f"err{r}.npy") for r in range(2)]
    for e in errs:
        assert e[0] < 2e-2
    assert sum(int(e[1]) for e in errs) == 2 * 20 * 4  # every (token, slot) row was served once


def test_ep_rank_leaving_fails_the_peer_cleanly(tmp_path):
    ctx = mp.start_processes(_ep_worker, args=(2, _free_port(), str(tmp_path), "drop"), nprocs=2,
                             start_method="spawn", join=False)
    for p in ctx.processes:
        p.join(timeout=120)
    assert all(not p.is_alive() for p in ctx.processes), "a rank hung"
    assert (tmp_path / "exc0.txt").exists(), "surviving rank did not report the failure"
