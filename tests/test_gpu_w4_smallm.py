"""GPU parity: the small-M W4A8 linear that unpacks the int4 weight in shared memory.

For up to 32 rows (16 with the asymmetric correction) ``w4a8_int8_linear`` without a pre-decoded grid reads the packed weight
through TMA and unpacks it to int8 inside the GEMM (h3b200_w4a8_int8_linear_packed). The
decode is the standalone decode kernel's, bit for bit, so for symmetric weights the result
must equal the decode-then-GEMM path exactly; the asymmetric correction is summed on CUDA
cores there (fp32, one rounding), so it agrees within the float tolerance."""

import numpy as np
import pytest
import torch

import h3b200
import oracle as O
from gpu_util import np_, randn_bf16, t2u

pytestmark = pytest.mark.gpu


def _packed(n, k, group, seed, e4m3=False, extreme=False):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randint(0, 256, (n, k // 2), generator=gen, dtype=torch.int32).to(torch.uint8).view(torch.int8)
    s = torch.rand(n, k // group, generator=gen) * 12.0 + 0.05
    if extreme:  # scales past the table's fast range, and NaN (decodes to 0)
        s[0, 0] = 3000.0
        s[1, 1 % (k // group)] = float("nan")
        s[2, :] = 1e-6
    s_rel = s.to(torch.float8_e4m3fn) if e4m3 else s
    s_ch = torch.rand(n, generator=gen) * 0.01 + 1e-4
    return q.cuda(), s_rel.cuda(), s_ch.cuda()


def _grid_path(x, q, s_rel, s_ch, group, codebook=None, bias=None, correction=None):
    grid = h3b200.dequant_int4_grouped_to_int8(q, s_rel, group, codebook)
    return h3b200.w4a8_int8_linear(x, q, s_rel, s_ch, codebook, correction, bias, group, 256, grid=grid)


@pytest.mark.parametrize("m,n,k,group", [(1, 3072, 3072, 128), (17, 1000, 3072, 128), (32, 12288, 3072, 128),
                                         (3, 3072, 12288, 128), (32, 768, 1024, 32), (20, 512, 5376, 128),
                                         (64, 1024, 3072, 128)])
def test_smallm_symmetric_uniform_matches_grid_path(m, n, k, group):
    q, s_rel, s_ch = _packed(n, k, group, seed=m + n)
    gen = torch.Generator().manual_seed(7 + m)
    x = randn_bf16((m, k), gen).cuda()
    bias = randn_bf16((n,), gen).cuda()
    y = h3b200.w4a8_int8_linear(x, q, s_rel, s_ch, None, None, bias, group, 256)
    assert h3b200.device_status(0) == 0
    assert torch.equal(y, _grid_path(x, q, s_rel, s_ch, group, bias=bias))


@pytest.mark.parametrize("m", [5, 32])
def test_smallm_release_format_extreme_scales(m):
    """H3 release format: group 16, fp8-e4m3 scales, 16-level codebook; scales past the
    table's fast range and a NaN scale take the exact decode."""
    n, k, group = 768, 5376, 16
    q, s_rel, s_ch = _packed(n, k, group, seed=31, e4m3=True, extreme=True)
    from h3b200.weights import W4A8_FIXED_CODEBOOK

    cb = torch.tensor(W4A8_FIXED_CODEBOOK, dtype=torch.float32).cuda()
    gen = torch.Generator().manual_seed(3)
    x = randn_bf16((m, k), gen).cuda()
    y = h3b200.w4a8_int8_linear(x, q, s_rel, s_ch, cb, None, None, group, 256)
    assert h3b200.device_status(0) == 0
    assert torch.equal(y, _grid_path(x, q, s_rel, s_ch, group, codebook=cb))


@pytest.mark.parametrize("m", [1, 7, 16, 40])
def test_smallm_asymmetric_correction_vs_grid_path_and_oracle(m):
    """Config-2 format (asymmetric, group 128, fp32 s_rel) with correction and bias: up to 16
    rows on the in-smem path, 40 rows on the decode path."""
    gen = torch.Generator().manual_seed(61 + m)
    k, n = 3072, 3072
    w = randn_bf16((n, k), gen, std=0.02)
    x = randn_bf16((m, k), gen).cuda()
    bias = randn_bf16((n,), gen).cuda()
    q, s_rel, s_ch, corr = h3b200.quantize_w4a8_weight(w.cuda(), 128)
    y = h3b200.w4a8_int8_linear(x, q, s_rel, s_ch, correction=corr, bias=bias, group_size=128)
    assert h3b200.device_status(0) == 0
    yg = _grid_path(x, q, s_rel, s_ch, 128, bias=bias, correction=corr)
    d = (y.float() - yg.float()).abs()
    assert float(d.max()) <= 2e-2 * max(1.0, float(yg.float().abs().max()))
    assert float((y != yg).float().mean()) < 0.02        # one fp32 sum order against another
    o = O.w4a8_int8_linear_quantized(t2u(x), np_(q), np_(s_rel), np_(s_ch), t2u(corr), 128, 256,
                                     bias_bf16=t2u(bias))
    rel = float(np.linalg.norm(O.bf16_to_f32(t2u(y)) - O.bf16_to_f32(o)) / np.linalg.norm(O.bf16_to_f32(o)))
    assert rel <= 2e-3


def test_smallm_input_act_and_strided_rows():
    n, k, group = 1024, 3072, 128
    q, s_rel, s_ch = _packed(n, k, group, seed=5)
    gen = torch.Generator().manual_seed(9)
    big = randn_bf16((40, 2 * k + 64), gen).cuda()
    x = big[:, :2 * k]                               # strided [gate | up] rows
    y = h3b200.w4a8_int8_linear(x, q, s_rel, s_ch, None, None, None, group, 256, input_act="swiglu")
    yg = _grid_path(h3b200.apply_input_act(x.contiguous(), "swiglu"), q, s_rel, s_ch, group)
    assert torch.equal(y, yg)
