"""GPU parity: W4A8 decode (bit-exact), ConvRot quantizer and W4A8 linear (tolerance)."""

import numpy as np
import pytest
import torch

import h3b200
import oracle as O
from gpu_util import np_, randn_bf16, t2u, u2t

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a = O.bf16_to_f32(a).astype(np.float64)
    b = O.bf16_to_f32(b).astype(np.float64)
    return np.linalg.norm(a - b) / np.linalg.norm(b), float(np.abs(a - b).max())


def test_decode_golden_bit_exact(golden):
    g = golden("w4a8_small")
    grid = h3b200.dequant_int4_grouped_to_int8(torch.from_numpy(g["qdata"]).cuda(),
                                               torch.from_numpy(g["s_rel"]).cuda(), 128)
    np.testing.assert_array_equal(np_(grid), g["grid"])


def test_convrot_quantize_vs_golden(golden):
    """Against the oracle (the correctly rounded rotation): bit-exact. Against the reference's
    own output, whose rotation is a bf16 CPU matmul summed in its BLAS order: the rows whose
    fp32 sums happen to round like the exact value agree bit for bit."""
    g = golden("w4a8_small")
    xq, xs = h3b200.quantize_int8_rowwise_convrot(u2t(g["x"]), 256)
    oq, os_ = O.quantize_int8_rowwise(O.rotate_activation(g["x"], 256))
    np.testing.assert_array_equal(np_(xq), oq)
    np.testing.assert_array_equal(np_(xs), os_)
    same = (np_(xq) == g["xq"]).all(-1)
    assert same.mean() >= 0.95
    np.testing.assert_array_equal(np_(xs)[same], g["xs"][same])


@pytest.mark.parametrize("m,k,ldx", [(1001, 3072, 3072), (37, 12288, 12288), (250, 6144, 6208), (13, 1024, 1024),
                                     (29, 2048, 2048), (45, 4096, 4096), (7, 2304, 2304), (300, 5376, 5376),
                                     (3, 256, 256), (61, 9216, 9216), (40, 11008, 11008), (9, 14336, 14336),
                                     (401, 12544, 12544), (1500, 14336, 14336), (77, 15360, 15424),
                                     (5, 15616, 15616), (33, 18432, 18432), (20, 24576, 24576)])
def test_convrot_quantize_shapes_vs_oracle(m, k, ldx):
    """Bit-exact int8 values and scales for 1 to 96 groups per row (1-8 groups per half-warp,
    partly filled slots such as H3's 21 groups), row counts that leave a stage partly filled,
    strided rows and rings that wrap many times (1,500 rows of H3's 56-group fc2 input)."""
    gen = torch.Generator().manual_seed(k + m)
    xfull = randn_bf16((m, ldx), gen)
    x = xfull[:, :k]
    q, xs = h3b200.quantize_int8_rowwise_convrot(xfull.cuda()[:, :k], 256)
    oq, os_ = O.quantize_int8_rowwise(O.rotate_activation(t2u(x.contiguous()), 256))
    np.testing.assert_array_equal(np_(q), oq)
    np.testing.assert_array_equal(np_(xs), os_)


def test_convrot_quantize_rejects_rows_past_the_limit():
    x = torch.zeros(2, 24832, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(NotImplementedError):
        h3b200.quantize_int8_rowwise_convrot(x, 256)


@pytest.mark.parametrize("k", [3072, 12288])
def test_convrot_quantize_cfg2_full_size_bit_exact(k):
    """Config 2's two activation quantizers at the full token count (32,760 x 3,072 and x 12,288):
    every token of the GPU result, compared bit for bit with the oracle on 2,048 rows spread over
    the whole range plus the first and last rows (the math is per token)."""
    gen = torch.Generator().manual_seed(3 + k)
    m = 32760
    x = randn_bf16((m, k), gen)
    xq, xs = h3b200.quantize_int8_rowwise_convrot(x.cuda(), 256)
    rows = np.unique(np.concatenate([np.linspace(0, m - 1, 2048).astype(np.int64), [0, 1, m - 2, m - 1]]))
    xs_np = t2u(x)[rows]
    oq, os_ = O.quantize_int8_rowwise(O.rotate_activation(xs_np, 256))
    np.testing.assert_array_equal(np_(xq)[rows], oq)
    np.testing.assert_array_equal(np_(xs)[rows], os_)


def _extreme_rows(k, seed):
    """Rows whose 256-groups leave the fast path: exponent spreads beyond 37 bits (1e30 with
    1e-30, 2^100 with 2^-40, 2 with 2^-40), subnormal-only groups, values of 2^-120 with one
    of 2^-84, exact cancellations, zeros; each row's other groups are ordinary."""
    rng = np.random.default_rng(seed)
    rows = O.f32_to_bf16(rng.standard_normal((8, k)).astype(np.float32))
    b = lambda v: O.f32_to_bf16(np.array([v], np.float32))[0]
    g = lambda r, i: (r, slice(256 * i, 256 * i + 256))
    rows[g(0, 0)][5] = b(1e30)
    rows[g(0, 0)][9] = b(-1e-30)
    rows[g(1, 1)] = O.f32_to_bf16((rng.standard_normal(256) * 1e-39).astype(np.float32))
    rows[g(2, 2 % (k // 256))] = O.f32_to_bf16((rng.standard_normal(256) * 2.0 ** 100).astype(np.float32))
    rows[g(2, 2 % (k // 256))][40] = b(2.0 ** -40)
    rows[g(3, 0)] = b(2.0)
    rows[g(3, 0)][0:256:2] = b(2.0 ** -40)
    rows[g(4, 0)] = O.f32_to_bf16((rng.standard_normal(256) * 2.0 ** -120).astype(np.float32))
    rows[g(4, 0)][17] = b(2.0 ** -84)
    rows[g(5, 0)] = b(1.0)                      # every output but one cancels exactly
    rows[6, :] = 0                              # an all-zero row: scale 1e-30, q = 0
    rows[g(7, 0)] = b(3.0)
    rows[g(7, 0)][100] = b(-3.0e-38)
    return rows


@pytest.mark.parametrize("k", [3072, 14336])
def test_convrot_slow_path_groups_bit_exact(k):
    """Groups outside the double-precision fast path take the exact integer-accumulator path;
    the result is still the correctly rounded rotation, so int8 values and scales match the
    oracle (whose own exact path sums those groups with rationals)."""
    ex = _extreme_rows(k, 7)
    gen = torch.Generator().manual_seed(11)
    base = t2u(randn_bf16((300, k), gen))
    base[[3, 150, 299, 40, 41, 200, 201, 77]] = ex
    q, s = h3b200.quantize_int8_rowwise_convrot(u2t(base), 256)
    oq, os_ = O.quantize_int8_rowwise(O.rotate_activation(base, 256))
    np.testing.assert_array_equal(np_(q), oq)
    np.testing.assert_array_equal(np_(s), os_)


def test_w4a8_linear_vs_reference(golden):
    g = golden("w4a8_small")
    y = h3b200.w4a8_int8_linear(u2t(g["x"]), torch.from_numpy(g["qdata"]).cuda(), torch.from_numpy(g["s_rel"]).cuda(),
                                torch.from_numpy(g["s_channel"]).cuda(), correction=u2t(g["correction"]),
                                group_size=128, convrot_groupsize=256)
    rel, mx = rel_l2(t2u(y), g["y_eager"])
    assert rel <= 1e-2 and mx <= 2e-2
    o = O.w4a8_int8_linear_quantized(g["x"], g["qdata"], g["s_rel"], g["s_channel"], g["correction"], 128, 256)
    rel, mx = rel_l2(t2u(y), o)
    assert rel <= 2e-3


@pytest.mark.parametrize("m", [200, 2048])
def test_w4a8_linear_bias_with_correction(m):
    """Asymmetric weights with a bias: bf16(bf16(bf16(dequant) + bias) + correction) on the single-CTA
    (200 rows) and CTA-pair (2,048 rows) GEMMs, against the oracle composition within the float
    tolerance, and the bias-free result plus bias within one bf16 rounding step."""
    gen = torch.Generator().manual_seed(51 + m)
    k, n = 3072, 1024
    w = randn_bf16((n, k), gen, std=0.02)
    x = randn_bf16((m, k), gen).cuda()
    bias = randn_bf16((n,), gen).cuda()
    q, s_rel, s_ch, corr = h3b200.quantize_w4a8_weight(w.cuda(), 128)
    y = h3b200.w4a8_int8_linear(x, q, s_rel, s_ch, correction=corr, bias=bias, group_size=128)
    y0 = h3b200.w4a8_int8_linear(x, q, s_rel, s_ch, correction=corr, group_size=128)
    assert h3b200.device_status(0) == 0
    rows = slice(0, 64)
    o = O.w4a8_int8_linear_quantized(t2u(x[rows]), np_(q), np_(s_rel), np_(s_ch), t2u(corr), 128, 256,
                                     bias_bf16=t2u(bias))
    rel, mx = rel_l2(t2u(y[rows]), o)
    assert rel <= 2e-3 and mx <= 2e-2
    d = (y.float() - (y0.float() + bias.float())).abs()
    assert float(d.max()) <= 2e-2 * float(y.float().abs().max())


def test_w4a8_int32_accumulators_exact(golden):
    g = golden("w4a8_small")
    acc = h3b200.mm_int8(torch.from_numpy(g["xq"]).cuda(), torch.from_numpy(g["grid"]).cuda().t())
    np.testing.assert_array_equal(np_(acc), g["acc"])


def test_fused_w4a8_mlp_matches_op_chain_and_oracle():
    """Config-2 MLP: the fused entry point equals the chain of single W4A8 ops bit for bit,
    and the oracle composition within the north-star tolerance."""
    gen = torch.Generator().manual_seed(3)
    d, ffn, m = 512, 1024, 200
    w1 = randn_bf16((ffn, d), gen, std=0.02)
    w2 = randn_bf16((d, ffn), gen, std=0.02)
    x = randn_bf16((m, d), gen)
    gate = randn_bf16((d,), gen)
    res = randn_bf16((m, d), gen)
    wt = h3b200.W4A8MLPWeights.from_float(w1, w2).to("cuda")
    out = h3b200.fused_gated_mlp_w4a8(res.cuda(), x.cuda(), wt, gate.cuda())
    assert h3b200.device_status(0) == 0
    h = h3b200.w4a8_int8_linear(x.cuda(), wt.q1, wt.s_rel1, wt.s_ch1, correction=wt.corr1, group_size=128)
    y = h3b200.w4a8_int8_linear(h, wt.q2, wt.s_rel2, wt.s_ch2, correction=wt.corr2, group_size=128,
                                input_act="gelu_tanh")
    f = O.bf16_to_f32
    expect = O.f32_to_bf16(f(t2u(res)) + f(t2u(y)) * f(t2u(gate))[None, :])
    np.testing.assert_array_equal(t2u(out), expect)
    # oracle composition (exact rotation, float64 correction)
    q1, q2 = np_(wt.q1), np_(wt.q2)
    oh = O.w4a8_int8_linear_quantized(t2u(x), q1, np_(wt.s_rel1), np_(wt.s_ch1), t2u(wt.corr1), 128, 256)
    oy = O.w4a8_int8_linear_quantized(O.gelu_tanh_bf16(oh), q2, np_(wt.s_rel2), np_(wt.s_ch2), t2u(wt.corr2), 128, 256)
    ref = O.gated_residual(t2u(res), oy, t2u(gate))
    rel, mx = rel_l2(t2u(out), ref)
    assert rel <= 1e-2 and mx <= 2e-2
    # in place on the residual
    r2 = res.cuda()
    h3b200.fused_gated_mlp_w4a8(r2, x.cuda(), wt, gate.cuda(), out=r2)
    np.testing.assert_array_equal(t2u(r2), t2u(out))


def test_w4a8_linear_cta_pair_path_matches_single_cta_and_oracle():
    """Large M takes the CTA-pair GEMM (cta_group::2, correction MMA over both CTAs' rows);
    row slices of <= 256 rows take the single-CTA GEMM. The tensor-core correction sums
    each output element in the same k order on both paths, so they agree bit for bit;
    a row subset is checked against the oracle within the north-star tolerance."""
    gen = torch.Generator().manual_seed(41)
    m, k, n = 2048, 3072, 3072
    w = randn_bf16((n, k), gen, std=0.02)
    x = randn_bf16((m, k), gen).cuda()
    q, s_rel, s_ch, corr = h3b200.quantize_w4a8_weight(w.cuda(), 128)
    grid = h3b200.dequant_int4_grouped_to_int8(q, s_rel, 128)
    y = h3b200.w4a8_int8_linear(x, q, s_rel, s_ch, correction=corr, group_size=128, grid=grid)
    parts = [h3b200.w4a8_int8_linear(x[s:s + 200], q, s_rel, s_ch, correction=corr, group_size=128, grid=grid)
             for s in range(0, m, 200)]
    assert h3b200.device_status(0) == 0
    np.testing.assert_array_equal(t2u(y), t2u(torch.cat(parts)))
    rows = slice(1000, 1064)
    o = O.w4a8_int8_linear_quantized(t2u(x[rows]), np_(q), np_(s_rel), np_(s_ch), t2u(corr), 128, 256)
    rel, mx = rel_l2(t2u(y[rows]), o)
    assert rel <= 2e-3 and mx <= 2e-2


def test_fused_w4a8_mlp_cta_pair_path_matches_op_chain():
    """Config-2 shapes (d 3072, ffn 12288) at 2048 tokens: both fused GEMMs (correction + GELU,
    correction + gated residual) run on CTA pairs; the result equals the chain of single ops."""
    gen = torch.Generator().manual_seed(43)
    d, ffn, m = 3072, 12288, 2048
    w1 = randn_bf16((ffn, d), gen, std=0.02).cuda()
    w2 = randn_bf16((d, ffn), gen, std=0.02).cuda()
    x = randn_bf16((m, d), gen).cuda()
    gate = randn_bf16((d,), gen).cuda()
    res = randn_bf16((m, d), gen).cuda()
    wt = h3b200.W4A8MLPWeights.from_float(w1, w2)
    out = h3b200.fused_gated_mlp_w4a8(res, x, wt, gate)
    h = h3b200.w4a8_int8_linear(x, wt.q1, wt.s_rel1, wt.s_ch1, correction=wt.corr1, group_size=128)
    y = h3b200.w4a8_int8_linear(h, wt.q2, wt.s_rel2, wt.s_ch2, correction=wt.corr2, group_size=128,
                                input_act="gelu_tanh")
    assert h3b200.device_status(0) == 0
    f = O.bf16_to_f32
    expect = O.f32_to_bf16(f(t2u(res)) + f(t2u(y)) * f(t2u(gate))[None, :])
    np.testing.assert_array_equal(t2u(out), expect)
