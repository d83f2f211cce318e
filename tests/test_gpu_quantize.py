"""GPU parity: per-token INT8 quantizer and the bf16 tanh-GELU (bit-exact)."""

import numpy as np
import pytest
import torch

import h3b200
import oracle as O
from gpu_util import np_, randn_bf16, t2u, u2t

pytestmark = pytest.mark.gpu


def test_gelu_all_bf16_inputs_bit_exact(golden):
    ref = golden("gelu_tanh_bf16_all")["y"]
    allx = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    y = t2u(h3b200.apply_input_act(u2t(allx), "gelu_tanh"))
    finite = np.isfinite(O.bf16_to_f32(allx))
    assert int((y[finite] != ref[finite]).sum()) == 0


def test_quantize_golden_bit_exact(golden):
    g = golden("quantize_rowwise")
    for sfx in ("", "_ragged", "_one"):
        q, s = h3b200.quantize_int8_rowwise(u2t(g["x" + sfx]))
        np.testing.assert_array_equal(np_(q), g["q" + sfx])
        np.testing.assert_array_equal(np_(s), g["s" + sfx])


@pytest.mark.parametrize("m,k", [(32760, 3072), (1000, 12288), (7, 40), (3, 16392), (5, 8), (1, 2048)])
def test_quantize_random_vs_oracle(m, k):
    gen = torch.Generator().manual_seed(m * 7 + k)
    x = randn_bf16((m, k), gen, std=2.0)
    q, s = h3b200.quantize_int8_rowwise(x.cuda())
    oq, os_ = O.quantize_int8_rowwise(t2u(x))
    np.testing.assert_array_equal(np_(q), oq)
    np.testing.assert_array_equal(np_(s), os_)


def test_quantize_strided_rows_and_act():
    gen = torch.Generator().manual_seed(3)
    big = randn_bf16((300, 4096), gen).cuda()
    x = big[:, 1024:1024 + 3072]                 # row stride 4096
    q, s = h3b200.quantize_int8_rowwise(x, input_act="gelu_tanh")
    a = O.gelu_tanh_bf16(t2u(x))
    oq, os_ = O.quantize_int8_rowwise(a)
    np.testing.assert_array_equal(np_(q), oq)
    np.testing.assert_array_equal(np_(s), os_)


def test_quantize_given_absmax():
    gen = torch.Generator().manual_seed(4)
    x = randn_bf16((129, 12288), gen)
    am = torch.from_numpy(np.abs(O.bf16_to_f32(t2u(x))).max(-1, keepdims=True))
    q, s = h3b200.quantize_int8_rowwise_absmax(x.cuda(), am.cuda())
    oq, os_ = O.quantize_int8_rowwise(t2u(x))
    np.testing.assert_array_equal(np_(q), oq)
    np.testing.assert_array_equal(np_(s), os_)


def test_quantize_empty_rows():
    q, s = h3b200.quantize_int8_rowwise(torch.empty(0, 64, dtype=torch.bfloat16, device="cuda"))
    assert q.shape == (0, 64) and s.shape == (0, 1)


@pytest.mark.parametrize("m,k,seed", [(300, 3072, 1), (7, 40, 99), (64, 12288, 2 ** 40 + 5), (1, 8, 3)])
def test_quantize_stochastic_vs_oracle(m, k, seed):
    gen = torch.Generator().manual_seed(m + k)
    x = randn_bf16((m, k), gen, std=3.0)
    x[0, : min(k, 4)] = 0.0
    if m > 2:
        x[2] = 0.0                                   # a zero row: scale 1e-30, divisor bf16 tiny
    q, s = h3b200.quantize_int8_rowwise(x.cuda(), stochastic_rounding=seed)
    oq, os_ = O.quantize_int8_rowwise_stochastic(t2u(x), seed)
    np.testing.assert_array_equal(np_(q), oq)
    np.testing.assert_array_equal(np_(s), os_)
    q0, _ = h3b200.quantize_int8_rowwise(x.cuda())
    if m * k > 1000:
        assert (np_(q) != np_(q0)).mean() > 0.1      # rounding differs from nearest-even
