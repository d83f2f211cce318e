"""GPU parity: fc2 with its input requantization inside the GEMM (h3b200_requant_gemm_gated_residual).

The GEMM's spare warps quantize h's rows (given the row absmax) while the tensor cores run;
the result must be bit-identical to the two-kernel chain quantize_int8_rowwise_absmax ->
epilogue 3 of int8_gemm_fused, which the other MLP tests pin to the oracle."""

import numpy as np
import pytest
import torch

import h3b200
from h3b200 import ops
from gpu_util import randn_bf16

pytestmark = pytest.mark.gpu


def _case(m, n, k, seed, hscale=1.0):
    gen = torch.Generator().manual_seed(seed)
    h = (randn_bf16((m, k), gen) * hscale).to(torch.bfloat16).cuda()
    w = randn_bf16((n, k), gen, std=0.02).cuda()
    wq, ws = ops.quantize_int8_rowwise(w)
    gate = randn_bf16((n,), gen).cuda()
    res = randn_bf16((m, n), gen).cuda()
    amax = h.float().abs().amax(dim=1)
    return h, amax, wq, ws.reshape(-1), gate, res


def _chain(h, amax, wq, ws, gate, res, bias=None):
    q, xs = ops.quantize_int8_rowwise_absmax(h, amax)
    return ops.int8_gemm_fused(q, wq, ops.EPI_GATED_RESIDUAL, xs, ws, bias=bias, gate=gate, residual=res)


@pytest.mark.parametrize("m,n,k", [(1, 256, 4096), (77, 512, 2048), (300, 3072, 12288), (1000, 1024, 5008),
                                   (4096, 3072, 12288), (32760, 3072, 12288)])
def test_requant_gemm_matches_chain(m, n, k):
    h, amax, wq, ws, gate, res = _case(m, n, k, seed=m + n + k)
    got = h3b200.requant_gemm_gated_residual(h, amax, wq, ws, gate, res)
    want = _chain(h, amax, wq, ws, gate, res)
    assert torch.equal(got, want)
    assert h3b200.device_status(0) == 0


def test_requant_gemm_bias_inplace_strided_and_extreme_rows():
    m, n, k = 700, 768, 3072
    h, amax, wq, ws, gate, res = _case(m, n, k, seed=11)
    big = torch.zeros(m, k + 64, dtype=torch.bfloat16, device="cuda")
    big[:, 32:32 + k] = h
    hv = big[:, 32:32 + k]                     # strided rows, 16-byte aligned
    hv[3].zero_()                              # an all-zero row (scale 1e-30)
    hv[5] *= 1e30                              # huge values
    hv[6] *= 1e-30                             # tiny values
    amax = hv.float().abs().amax(dim=1)
    bias = randn_bf16((n,), torch.Generator().manual_seed(3)).cuda()
    want = _chain(hv, amax, wq, ws, gate, res, bias=bias)
    out = res.clone()
    h3b200.requant_gemm_gated_residual(hv, amax, wq, ws, gate, out, out=out, bias=bias)
    assert torch.equal(out, want)


def test_requant_gemm_row_map_segments():
    m, n, k = 1500, 1024, 4096
    h, amax, wq, ws, _, res = _case(m, n, k, seed=21)
    gen = torch.Generator().manual_seed(5)
    gate_rows = randn_bf16((3, n), gen).cuda()
    row_map = torch.tensor(np.repeat([0, 1, 2], [400, 700, 400]), dtype=torch.int32, device="cuda")
    got = h3b200.requant_gemm_gated_residual(h, amax, wq, ws, gate_rows, res, row_map=row_map)
    for r in range(3):
        sel = row_map == r
        want = _chain(h, amax, wq, ws, gate_rows[r].contiguous(), res)
        assert torch.equal(got[sel], want[sel])


def test_requant_gemm_reuses_workspace():
    m, n, k = 2048, 3072, 12288
    h, amax, wq, ws, gate, res = _case(m, n, k, seed=31)
    work = torch.empty(int(h3b200.library().h3b200_requant_gemm_workspace_bytes(m, k)), dtype=torch.uint8,
                       device="cuda")
    a = h3b200.requant_gemm_gated_residual(h, amax, wq, ws, gate, res, workspace=work)
    b = h3b200.requant_gemm_gated_residual(h, amax, wq, ws, gate, res, workspace=work)
    assert torch.equal(a, b)
    assert torch.equal(a, _chain(h, amax, wq, ws, gate, res))
