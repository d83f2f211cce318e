"""GPU parity on 2 or 4 GPUs: tensor-parallel MLP and token sharding vs one GPU.

Each rank runs in its own spawned process with one GPU. The tensor-parallel MLP
(fc1 column-split, the row absmax max-reduced over the ranks, fc2 row-split with its
int32 partial sums reduced exactly) in all three exchange forms -- inside the kernels
over NVLink peer memory ("p2p": IPC-mapped regions, flag barriers), NCCL int32
reduce-scatter + bf16 all-gather, NCCL int32 all-reduce -- and the token-sharded MLP
must all reproduce the single-GPU fused MLP bit for bit. A cross-GPU barrier that the
other ranks never enter must expire on rank 0 with status 0x201 (bounded wait, no
fault). Skipped when fewer than 2 GPUs are visible.
"""

import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, outdir):
    sys.path.insert(0, os.path.join(ROOT, "x-minimaxh3_b200"))
    import torch.distributed as dist

    import h3b200
    from h3b200 import parallel as P

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        d, ffn, m = 512, 2048, 1000
        g = torch.Generator().manual_seed(11)           # identical weights and inputs on every rank
        w1 = (torch.randn(ffn, d, generator=g) * 0.02).to(torch.bfloat16).to(dev)
        w2 = (torch.randn(d, ffn, generator=g) * 0.02).to(torch.bfloat16).to(dev)
        x = torch.randn(m, d, generator=g).to(torch.bfloat16).to(dev)
        res = torch.randn(m, d, generator=g).to(torch.bfloat16).to(dev)
        gate = torch.randn(d, generator=g).to(torch.bfloat16).to(dev)
        wt = h3b200.W8A8MLPWeights.from_float(w1, w2)
        ref = h3b200.fused_gated_mlp(res, x, wt.w1q, wt.s1, wt.w2q, wt.s2, gate)

        shard = P.TPShard.from_full(wt.w1q, wt.s1, wt.w2q, wt.s2, world, rank)
        # chunks of 383 rows (383, 383, 234): reduce-scatter rows padded to the world size
        tp = all(bool(torch.equal(P.tp_gated_mlp(x, res, gate, shard, chunk_tokens=383, collective=c), ref))
                 for c in P.COLLECTIVES)

        lo, hi = P.shard_range(m, world, rank)
        local = P.token_sharded_mlp(x[lo:hi], res[lo:hi], gate, wt.w1q, wt.s1, wt.w2q, wt.s2)
        ts = P.gather_tokens(local, m)
        torch.cuda.synchronize()
        ok = {
            "tp": tp,
            "token_shard": bool(torch.equal(ts, ref)),
            "status": h3b200.device_status(rank),
        }
        P.close_tp_comms()
        # a barrier that only rank 0 enters: its 20 ms bounded wait expires, the kernel
        # records 0x201 and returns; the other ranks never launch anything on it
        comm = P.TPComm(64, d, ffn // world, barrier_timeout_s=0.02)
        expired = 0x201
        if rank == 0:
            comm.barrier()
            torch.cuda.synchronize()
            expired = h3b200.device_status(rank, clear=True)
        comm.close()
        ok["barrier_expiry"] = expired == 0x201
        with open(os.path.join(outdir, f"rank{rank}.txt"), "w") as f:
            f.write(repr(ok))
    finally:
        dist.destroy_process_group()


def test_tp_mlp_and_token_sharding_multi_gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    world = 4 if torch.cuda.device_count() >= 4 else 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(world):
        res = eval((tmp_path / f"rank{r}.txt").read_text())
        assert res == {"tp": True, "token_shard": True, "status": 0, "barrier_expiry": True}, (r, res)
