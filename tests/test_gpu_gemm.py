"""GPU parity: tcgen05 INT8 GEMM (int32 accumulators bit-exact) and the dequant epilogue."""

import numpy as np
import pytest
import torch

import h3b200
import oracle as O
from gpu_util import np_, randn_bf16, t2u, u2t

pytestmark = pytest.mark.gpu


def rand_i8(shape, gen):
    return torch.randint(-128, 128, shape, generator=gen, dtype=torch.int16).to(torch.int8)


# (300, 12288, 3072) and (1000, 12288, 2064) have enough 256 x 256 tiles to run on
# CTA pairs (cta_group::2); the others run on single CTAs
@pytest.mark.parametrize("m,n,k", [(1, 256, 128), (128, 256, 128), (130, 264, 48), (257, 512, 3072),
                                   (1000, 1024, 12288), (37, 8, 16), (300, 12288, 3072), (1000, 12288, 2064)])
def test_mm_int8_exact(m, n, k):
    gen = torch.Generator().manual_seed(m + 3 * n + 7 * k)
    a = rand_i8((m, k), gen)
    w = rand_i8((n, k), gen)
    out = h3b200.mm_int8(a.cuda(), w.cuda().t())
    np.testing.assert_array_equal(np_(out), O.int8_matmul_accumulate(np_(a), np_(w)))


def test_mm_int8_saturating_values_exact():
    # all -128 operands: largest-magnitude accumulators (2^14 * K)
    m, n, k = 128, 256, 12288
    a = torch.full((m, k), -128, dtype=torch.int8)
    w = torch.full((n, k), -128, dtype=torch.int8)
    out = h3b200.mm_int8(a.cuda(), w.cuda().t())
    assert int(out.min()) == int(out.max()) == 128 * 128 * k


def test_int8_linear_cfg0_slice_golden(golden):
    g = golden("linear_cfg0_slice")
    x, wq, ws = u2t(g["x"]), torch.from_numpy(g["wq"]).cuda(), torch.from_numpy(g["ws"]).cuda()
    np.testing.assert_array_equal(t2u(h3b200.int8_linear(x, wq, ws)), g["y"])
    np.testing.assert_array_equal(t2u(h3b200.int8_linear(x, wq, ws, u2t(g["bias"]))), g["y_bias"])
    np.testing.assert_array_equal(t2u(h3b200.int8_linear(x, wq, ws, input_act="gelu_tanh")), g["y_gelu_in"])
    # weight quantization on the GPU matches the reference's per-channel quantizer
    wq2, ws2 = h3b200.quantize_int8_weight(u2t(g["w_bf16"]))
    np.testing.assert_array_equal(np_(wq2), g["wq"])
    np.testing.assert_array_equal(np_(ws2), g["ws"])
    # int32 accumulators of the same activations are bit-exact
    xq = torch.from_numpy(g["xq"]).cuda()
    np.testing.assert_array_equal(np_(h3b200.mm_int8(xq, wq.t())), g["acc"])


def test_int8_linear_cfg0_full_shape():
    """Config 0: M=256, K=3072, N=12288; W ~ N(0, 0.02) seed 0, x ~ N(0, 1) seed 1."""
    w = randn_bf16((12288, 3072), torch.Generator().manual_seed(0), std=0.02)
    x = randn_bf16((256, 3072), torch.Generator().manual_seed(1))
    wq, ws = h3b200.quantize_int8_weight(w.cuda())
    y = h3b200.int8_linear(x.cuda(), wq, ws)
    owq, ows = O.quantize_int8_rowwise(t2u(w))
    np.testing.assert_array_equal(np_(wq), owq)
    np.testing.assert_array_equal(t2u(y), O.int8_linear(t2u(x), owq, ows.reshape(-1)))


def test_int8_linear_prequantized_tensorwise_scale_and_3d():
    gen = torch.Generator().manual_seed(9)
    x = randn_bf16((2, 70, 512), gen)
    w = rand_i8((384, 512), gen)
    ws = torch.tensor([0.0037])
    xq, xs = h3b200.quantize_int8_rowwise(x.cuda())
    y = h3b200.int8_linear_prequantized(xq, xs, w.cuda(), ws.cuda())
    assert y.shape == (2, 70, 384)
    oq, os_ = O.quantize_int8_rowwise(t2u(x).reshape(140, 512))
    ref = O.dequant_epilogue(O.int8_matmul_accumulate(oq, np_(w)), os_, np_(ws).repeat(384))
    np.testing.assert_array_equal(t2u(y).reshape(140, 384), ref)


def test_large_m_sampled_rows_exact():
    """M = 32760 (config 1 fc1 shape): rows are independent, so sampled rows are checked exactly."""
    gen = torch.Generator().manual_seed(21)
    x = randn_bf16((32760, 3072), gen)
    w = randn_bf16((12288, 3072), gen, std=0.02)
    wq, ws = h3b200.quantize_int8_weight(w.cuda())
    y = h3b200.int8_linear(x.cuda(), wq, ws)
    rows = np.sort(np.random.default_rng(0).choice(32760, 40, replace=False))
    rows = np.concatenate([rows, [0, 127, 128, 32639, 32640, 32759]])
    ref = O.int8_linear(t2u(x)[rows], np_(wq), np_(ws))
    np.testing.assert_array_equal(t2u(y)[rows], ref)


def test_contract_errors():
    a = torch.zeros(4, 24, dtype=torch.int8, device="cuda")     # k % 16 != 0
    with pytest.raises(NotImplementedError):
        h3b200.mm_int8(a, torch.zeros(24, 8, dtype=torch.int8, device="cuda"))
    x = torch.zeros(4, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="inner dimensions"):
        h3b200.int8_linear(x, torch.zeros(8, 32, dtype=torch.int8, device="cuda"), torch.ones(8, device="cuda"))
    with pytest.raises(ValueError, match="scalar or per-output-channel"):
        h3b200.int8_linear(x, torch.zeros(8, 64, dtype=torch.int8, device="cuda"), torch.ones(3, device="cuda"))


@pytest.mark.parametrize("m,n,k", [(300, 512, 256), (600, 12288, 128)])
def test_gelu_absmax_epilogue_outside_the_table(m, n, k):
    """The fc1 epilogue (dequant -> tanh-GELU -> bf16, row absmax) on rows whose values fall
    outside the shared-memory table: zero rows, a tiny row scale (|x| < 2^-16), a large one
    (|x| >= 8, both signs), beside ordinary rows; single CTAs and CTA pairs. Output bits and
    row absmax equal the oracle's."""
    gen = torch.Generator().manual_seed(m + n + k)
    a = rand_i8((m, k), gen)
    a[::7] = 0                                                  # acc = 0: gelu(+0) = +0
    w = rand_i8((n, k), gen)
    xs = torch.full((m,), 1e-4, dtype=torch.float32)
    xs[1::5] = 1e-9                                            # |x| < 2^-16: 0.5 x
    xs[2::5] = 1.0                                             # |x| >= 8: x or -0
    ws = (torch.rand(n, generator=gen) * 1e-3 + 1e-4).to(torch.float32)
    amax = torch.zeros(m, dtype=torch.float32, device="cuda")
    out = h3b200.ops.int8_gemm_fused(a.cuda(), w.cuda(), h3b200.ops.EPI_GELU_ABSMAX, xs.cuda(), ws.cuda(),
                                     row_absmax=amax)
    acc = O.int8_matmul_accumulate(np_(a), np_(w))
    ref = O.gelu_tanh_bf16(O.dequant_epilogue(acc, np_(xs), np_(ws)))
    np.testing.assert_array_equal(t2u(out), ref)
    np.testing.assert_array_equal(np_(amax), np.abs(O.bf16_to_f32(ref)).max(axis=1))
    assert h3b200.device_status(0) == 0
