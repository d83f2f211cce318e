"""GPU parity: the tensor-parallel MLP whose exchanges run inside the kernels (peer memory).

On one GPU, ``TPComm.linked_local`` makes ``world`` communicators of one process each
other's peers (no IPC, no barrier), and the test runs every rank's stages in order:
1 quantize + fc1 + absmax push, 2 absmax max + fc2 storing each int32 partial row at its
owner, 3 owner rows (sum, dequant + gated residual, rows pushed to every rank), 4 the
other owners' rows into out. Every rank's output must equal the single-GPU fused MLP bit
for bit (int32 sums are exact, the requant uses the global absmax). The same kernels run
across GPUs, with IPC mappings and flag barriers, in tests/test_gpu_multi.py."""

import pytest
import torch

import h3b200
from h3b200 import parallel as P

pytestmark = pytest.mark.gpu


def _problem(m, d, ffn, seed):
    g = torch.Generator().manual_seed(seed)
    w1 = (torch.randn(ffn, d, generator=g) * 0.02).to(torch.bfloat16).cuda()
    w2 = (torch.randn(d, ffn, generator=g) * 0.02).to(torch.bfloat16).cuda()
    x = torch.randn(m, d, generator=g).to(torch.bfloat16).cuda()
    res = torch.randn(m, d, generator=g).to(torch.bfloat16).cuda()
    gate = torch.randn(d, generator=g).to(torch.bfloat16).cuda()
    wt = h3b200.W8A8MLPWeights.from_float(w1, w2)
    return x, res, gate, wt


# rows are owned in 128-row blocks round-robin: chunks of 1 to 11 blocks, partial last blocks,
# ranks that own nothing in a chunk
@pytest.mark.parametrize("world,m,chunk", [(2, 1000, 383), (4, 700, 256), (8, 383, 383), (4, 5, 3),
                                           (2, 2048, 1024), (4, 3000, 1500), (8, 2500, 1300)])
def test_linked_ranks_match_single_gpu_mlp(world, m, chunk):
    d, ffn = 512, 2048
    x, res, gate, wt = _problem(m, d, ffn, seed=world * 100 + m)
    ref = h3b200.fused_gated_mlp(res, x, wt.w1q, wt.s1, wt.w2q, wt.s2, gate)
    comms = P.TPComm.linked_local(world, chunk, d, ffn // world)
    shards = [P.TPShard.from_full(wt.w1q, wt.s1, wt.w2q, wt.s2, world, r) for r in range(world)]
    outs = [torch.full_like(res, float("nan")) for _ in range(world)]
    try:
        for i, lo in enumerate(range(0, m, chunk)):
            hi = min(m, lo + chunk)
            for stage in (1, 2, 3, 4):
                for r in range(world):
                    comms[r].stage(stage, i, x, res, gate, shards[r], outs[r], lo, hi)
        torch.cuda.synchronize()
        assert h3b200.device_status(0) == 0
        for r in range(world):
            assert torch.equal(outs[r], ref), f"rank {r}"
    finally:
        for c in comms:
            c.close()


def test_strided_rows_and_large_chunk_two_ranks():
    """Row strides above d (views into wider buffers) and the config-1 width."""
    d, ffn, m, world = 3072, 12288, 600, 2
    x0, res0, gate, wt = _problem(m, d, ffn, seed=5)
    xb = torch.zeros(m, d + 64, dtype=torch.bfloat16, device="cuda")
    xb[:, :d] = x0
    rb = torch.zeros(m, d + 128, dtype=torch.bfloat16, device="cuda")
    rb[:, :d] = res0
    x, res = xb[:, :d], rb[:, :d]
    ref = h3b200.fused_gated_mlp(res0, x0, wt.w1q, wt.s1, wt.w2q, wt.s2, gate)
    comms = P.TPComm.linked_local(world, 512, d, ffn // world)
    shards = [P.TPShard.from_full(wt.w1q, wt.s1, wt.w2q, wt.s2, world, r) for r in range(world)]
    ob = [torch.zeros(m, d + 32, dtype=torch.bfloat16, device="cuda") for _ in range(world)]
    outs = [o[:, :d] for o in ob]
    try:
        for i, lo in enumerate(range(0, m, 512)):
            hi = min(m, lo + 512)
            for stage in (1, 2, 3, 4):
                for r in range(world):
                    comms[r].stage(stage, i, x, res, gate, shards[r], outs[r], lo, hi)
        torch.cuda.synchronize()
        for r in range(world):
            assert torch.equal(outs[r], ref)
    finally:
        for c in comms:
            c.close()


def test_contract_errors():
    d, ffn = 512, 2048
    x, res, gate, wt = _problem(64, d, ffn, seed=1)
    comms = P.TPComm.linked_local(2, 64, d, ffn // 2)
    shard = P.TPShard.from_full(wt.w1q, wt.s1, wt.w2q, wt.s2, 2, 0)
    try:
        with pytest.raises(NotImplementedError):       # linked ranks run stage by stage
            comms[0].run(x, res, gate, shard, torch.empty_like(res))
        with pytest.raises(ValueError):                 # chunk above max_rows
            comms[0].stage(1, 0, x, res, gate, shard, torch.empty_like(res), 0, 65)
        with pytest.raises(ValueError):                 # stage out of range
            comms[0].stage(5, 0, x, res, gate, shard, torch.empty_like(res), 0, 8)
        with pytest.raises(ValueError):                 # the other rank's shard width
            comms[0].stage(1, 0, x, res, gate, P.TPShard.from_full(wt.w1q, wt.s1, wt.w2q, wt.s2, 4, 0),
                           torch.empty_like(res), 0, 8)
    finally:
        for c in comms:
            c.close()
    with pytest.raises(ValueError):
        P.TPComm(64, d, ffn, _local=(9, 0))             # more ranks than the kernels route
    with pytest.raises(ValueError):
        P.TPComm(64, d + 8, ffn, _local=(1, 0))         # d not a multiple of 16


def test_one_rank_p2p_is_the_fused_mlp():
    d, ffn, m = 512, 2048, 900
    x, res, gate, wt = _problem(m, d, ffn, seed=9)
    shard = P.TPShard.from_full(wt.w1q, wt.s1, wt.w2q, wt.s2, 1, 0)
    out = P.tp_gated_mlp(x, res, gate, shard, chunk_tokens=256)
    ref = h3b200.fused_gated_mlp(res, x, wt.w1q, wt.s1, wt.w2q, wt.s2, gate)
    assert torch.equal(out, ref)
