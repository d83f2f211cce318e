"""GPU parity: fp16 activations and outputs of the INT8 quantizer and linear.

The reference's eager code takes any activation dtype and ``out_dtype``
(eager/quantization.py:815-826, 857-875, 971-1056); with fp16 the quantizer's divisor
and quotient are fp16 values and the dequantized output (plus the bias, converted to
the output dtype) is rounded to fp16. Bit-exact against the reference fixture and the
oracle pinned to it."""

import numpy as np
import pytest
import torch

import h3b200
import oracle as O
from gpu_util import np_

pytestmark = pytest.mark.gpu


def _h16(u16: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.float16).cuda()


def _b16(u16: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.bfloat16).cuda()


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def test_fp16_against_reference_fixture(golden):
    g = golden("fp16_linear")
    x16 = _h16(g["x16"])
    q, s = h3b200.quantize_int8_rowwise(x16)
    np.testing.assert_array_equal(np_(q), g["q16"])
    np.testing.assert_array_equal(np_(s), g["s16"])
    wq = torch.from_numpy(g["wq"]).cuda()
    ws = torch.from_numpy(g["ws"]).cuda()
    y = h3b200.int8_linear(x16, wq, ws, None, torch.float16)
    assert y.dtype == torch.float16
    np.testing.assert_array_equal(_bits(y), g["y16"])
    yb = h3b200.int8_linear(x16, wq, ws, _h16(g["bias16"]), torch.float16)
    np.testing.assert_array_equal(_bits(yb), g["y16_bias"])
    ym = h3b200.int8_linear(_b16(g["xbf"]), wq, ws, _b16(g["biasbf"]), torch.float16)
    np.testing.assert_array_equal(_bits(ym), g["y_bf_in_f16_out"])
    yf = h3b200.int8_linear(x16, wq, ws, None, torch.bfloat16)
    assert yf.dtype == torch.bfloat16
    np.testing.assert_array_equal(_bits(yf), g["y_f16_in_bf_out"])
    assert h3b200.device_status(0) == 0


@pytest.mark.parametrize("m,n,k,stride_pad", [(1, 256, 64, 0), (37, 200, 40, 8), (1000, 3072, 3072, 0),
                                              (8192, 2048, 1024, 64)])
def test_fp16_linear_matches_oracle(m, n, k, stride_pad):
    """Ragged K and rows, strided rows, single-CTA and CTA-pair GEMM tiles, bias."""
    gen = torch.Generator().manual_seed(m + n)
    xb = (torch.randn(m, k + stride_pad, generator=gen) * 3).to(torch.float16)
    x = xb.cuda()[:, :k]
    w = (torch.randn(n, k, generator=gen) * 0.02).to(torch.bfloat16).cuda()
    wq, ws = h3b200.quantize_int8_rowwise(w)
    ws = ws.reshape(-1)
    bias = torch.randn(n, generator=gen).to(torch.float16).cuda()
    q, s = h3b200.quantize_int8_rowwise(x)
    oq, osc = O.quantize_int8_rowwise_f16(xb[:, :k].numpy())
    np.testing.assert_array_equal(np_(q), oq)
    np.testing.assert_array_equal(np_(s), osc)
    if k % 16 or n % 8:
        return  # the GEMM's contract (k % 16, n % 8); the quantizer has none
    y = h3b200.int8_linear(x, wq, ws, bias, torch.float16)
    oy = O.int8_linear_f16(xb[:, :k].numpy(), np_(wq), np_(ws), bias.cpu().numpy())
    np.testing.assert_array_equal(_bits(y), oy.view(np.uint16))
    assert h3b200.device_status(0) == 0


def test_fp16_unsupported_combinations_raise():
    x = torch.randn(4, 64, device="cuda").to(torch.float16)
    w = torch.zeros(32, 64, dtype=torch.int8, device="cuda")
    ws = torch.ones(32, device="cuda")
    with pytest.raises(NotImplementedError):
        h3b200.int8_linear(x, w, ws, None, torch.float16, input_act="gelu_tanh")
    with pytest.raises(NotImplementedError):
        h3b200.int8_linear(x, w, ws, None, torch.float16, convrot=True)
    with pytest.raises(NotImplementedError):
        h3b200.int8_linear(x, w, ws, None, torch.float32)
    with pytest.raises(NotImplementedError):
        h3b200.quantize_int8_rowwise(x, stochastic_rounding=3)
