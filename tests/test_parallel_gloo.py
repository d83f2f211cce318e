"""Multi-rank logic on CPU: 2 gloo ranks, oracle ops standing in for the CUDA kernels.

Checks that token sharding and the tensor-parallel MLP reproduce the
single-rank result bit for bit, and that a rank that fails before a collective
makes the other rank error out (short process-group timeout) instead of hanging.
"""

import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _paths():
    for p in (ROOT, os.path.join(ROOT, "x-minimaxh3_b200"), os.path.join(ROOT, "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)


def _u(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _t(u):
    return torch.from_numpy(np.ascontiguousarray(u).view(np.int16)).view(torch.bfloat16)


class OracleOps:
    """CPU stand-ins for the stage kernels (test infrastructure only)."""

    def __init__(self):
        import oracle

        self.O = oracle

    def quantize(self, x):
        q, s = self.O.quantize_int8_rowwise(_u(x))
        return torch.from_numpy(q), torch.from_numpy(s)

    def fc1_gelu_absmax(self, xq, xs, w1q, s1, absmax):
        O = self.O
        acc = O.int8_matmul_accumulate(xq.numpy(), w1q.numpy())
        a = O.gelu_tanh_bf16(O.dequant_epilogue(acc, xs.numpy(), s1.numpy()))
        am = np.abs(O.bf16_to_f32(a)).max(-1)
        absmax.copy_(torch.maximum(absmax, torch.from_numpy(am)))
        return _t(a)

    def quantize_absmax(self, a, absmax):
        q, s = self.O.quantize_int8_rowwise_given_absmax(_u(a), absmax.numpy().reshape(-1, 1))
        return torch.from_numpy(q), torch.from_numpy(s)

    def gemm_i32(self, q, w):
        return torch.from_numpy(self.O.int8_matmul_accumulate(q.numpy(), w.numpy()))

    def dequant_gated_residual(self, acc, xs, ws, gate, residual, out):
        O = self.O
        y = O.dequant_epilogue(acc.numpy(), xs.numpy(), ws.numpy())
        out.copy_(_t(O.gated_residual(_u(residual), y, _u(gate))))
        return out

    def fused_mlp(self, residual, x, w1q, s1, w2q, s2, gate, out):
        o = self.O.w8a8_gelu_mlp(_u(x), w1q.numpy(), s1.numpy(), w2q.numpy(), s2.numpy(), _u(gate), _u(residual))
        out.copy_(_t(o))
        return out

    def norm_rope(self, q, k, table, wq, wk, scale, shift, eps, span):
        qo, ko = self.O.adaln_rms_rope(_u(q), _u(k), table.numpy(), _u(wq), _u(wk), _u(scale), _u(shift), eps, span)
        return _t(qo), _t(ko)


def _inputs(m=96, d=128, ffn=512, seed=7):
    import oracle as O

    g = torch.Generator().manual_seed(seed)
    w1 = (torch.randn(ffn, d, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(d, ffn, generator=g) * 0.02).to(torch.bfloat16)
    w1q, s1 = O.quantize_int8_rowwise(_u(w1))
    w2q, s2 = O.quantize_int8_rowwise(_u(w2))
    x = (torch.randn(m, d, generator=g)).to(torch.bfloat16)
    res = (torch.randn(m, d, generator=g)).to(torch.bfloat16)
    gate = (torch.randn(d, generator=g)).to(torch.bfloat16)
    return (x, res, gate, torch.from_numpy(w1q), torch.from_numpy(s1.reshape(-1)), torch.from_numpy(w2q),
            torch.from_numpy(s2.reshape(-1)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    _paths()
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
        from h3b200 import parallel as P

        ops = OracleOps()
        x, res, gate, w1q, s1, w2q, s2 = _inputs()
        m = x.shape[0]
        if mode.startswith("tp"):
            # 96 tokens in chunks of 37 (37, 37, 22 rows): no chunk splits evenly over 2 or 4
            # ranks, so the reduce-scatter pads rows and the gather copies back
            shard = P.TPShard.from_full(w1q, s1, w2q, s2, world, rank)
            full = ops.fused_mlp(res, x, w1q, s1, w2q, s2, gate, torch.empty_like(res))
            ok = True
            for coll in P.PG_COLLECTIVES:
                out = P.tp_gated_mlp(x, res, gate, shard, chunk_tokens=37, ops=ops, collective=coll)
                ok = ok and bool(torch.equal(out.view(torch.int16), full.view(torch.int16)))
            q.put((rank, ok))
        elif mode == "dp":
            lo, hi = P.shard_range(m, world, rank)
            y = P.token_sharded_mlp(x[lo:hi], res[lo:hi], gate, w1q, s1, w2q, s2, ops=ops)
            allv = P.gather_tokens(y, m)
            full = ops.fused_mlp(res, x, w1q, s1, w2q, s2, gate, torch.empty_like(res))
            q.put((rank, bool(torch.equal(allv.view(torch.int16), full.view(torch.int16)))))
        elif mode == "fail":
            if rank == 1:
                raise RuntimeError("injected failure before the collective")
            t = torch.zeros(4)
            try:
                dist.all_reduce(t)
                q.put((rank, "no-error"))
            except Exception as e:  # the surviving rank must see an error, not hang
                q.put((rank, f"error:{type(e).__name__}"))
    except RuntimeError as e:
        if "injected" in str(e):
            q.put((rank, "injected"))
        else:
            q.put((rank, f"crash:{e}"))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def _run(mode, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, v = q.get(timeout=timeout)
        results[r] = v
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return results


def test_shard_range_covers_tokens():
    _paths()
    from h3b200.parallel import column_shard, shard_range

    for m, w in ((196560, 8), (32760, 3), (5, 8), (0, 2)):
        ranges = [shard_range(m, w, r) for r in range(w)]
        assert ranges[0][0] == 0 and ranges[-1][1] == m
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
        assert max(h - l for l, h in ranges) - min(h - l for l, h in ranges) <= 1
    assert column_shard(12288, 8, 3) == (4608, 6144)
    with pytest.raises(ValueError):
        column_shard(12288, 5, 0)


def test_tensor_parallel_mlp_bit_exact_two_ranks():
    res = _run("tp")
    assert res == {0: True, 1: True}


def test_tensor_parallel_mlp_bit_exact_four_ranks():
    """ffn 512 over 4 ranks (128 columns each), ragged chunks of 37 and 22 rows."""
    res = _run("tp", world=4)
    assert res == {0: True, 1: True, 2: True, 3: True}


def test_tensor_parallel_mlp_without_process_group():
    """One rank and no process group: the same chunked path, no collective."""
    _paths()
    from h3b200 import parallel as P

    ops = OracleOps()
    x, res, gate, w1q, s1, w2q, s2 = _inputs(m=50)
    shard = P.TPShard.from_full(w1q, s1, w2q, s2, 1, 0)
    out = P.tp_gated_mlp(x, res, gate, shard, chunk_tokens=16, ops=ops)
    full = ops.fused_mlp(res, x, w1q, s1, w2q, s2, gate, torch.empty_like(res))
    assert torch.equal(out.view(torch.int16), full.view(torch.int16))
    with pytest.raises(ValueError):
        P.tp_gated_mlp(x, res, gate, shard, ops=ops, collective="ring")


def test_token_sharded_mlp_bit_exact_two_ranks():
    res = _run("dp")
    assert res == {0: True, 1: True}


def test_failed_rank_surfaces_as_error_not_hang():
    res = _run("fail")
    assert res[1] == "injected"
    assert res[0].startswith("error:")
