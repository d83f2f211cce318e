"""GPU parity: the SwiGLU input activation (input_act="swiglu", rows [gate | up]).

SiLU is bit-exact against the reference's CPU result on all 65,536 bf16 inputs; the
activated rows, their quantization and the plain INT8 linear are bit-exact against
the reference fixtures and the oracle; the ConvRot variant is within the north-star
tolerance (its rotation is a bf16 matmul in the reference).
"""

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


def test_silu_all_bf16_inputs_bit_exact(golden):
    ref = golden("silu_bf16_all")["y"]
    allx = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    ones = np.full(65536, 0x3F80, dtype=np.uint16)          # up = 1.0: the product is the silu itself
    y = t2u(h3b200.apply_input_act(u2t(np.concatenate([allx, ones]).reshape(1, -1)), "swiglu")).reshape(-1)
    finite = np.isfinite(O.bf16_to_f32(allx))
    assert int((y[finite] != ref[finite]).sum()) == 0
    assert np.isnan(O.bf16_to_f32(y[np.isnan(O.bf16_to_f32(allx))])).all()


def test_swiglu_golden(golden):
    g = golden("swiglu_linear")
    x = u2t(g["x"])
    np.testing.assert_array_equal(t2u(h3b200.apply_input_act(x, "swiglu")), g["act"])
    q, s = h3b200.quantize_int8_rowwise(x, input_act="swiglu")
    np.testing.assert_array_equal(np_(q), g["aq"])
    np.testing.assert_array_equal(np_(s), g["as"])
    y = h3b200.int8_linear(x, torch.from_numpy(g["wq"]).cuda(), torch.from_numpy(g["ws"]).cuda(), input_act="swiglu")
    np.testing.assert_array_equal(t2u(y), g["y"])
    yc = h3b200.int8_linear(x, torch.from_numpy(g["wq_convrot"]).cuda(), torch.from_numpy(g["ws_convrot"]).cuda(),
                            convrot=True, convrot_groupsize=256, input_act="swiglu")
    rel, mx = rel_l2(t2u(yc), g["y_convrot"])
    assert rel <= 1e-2 and mx <= 2e-2
    assert h3b200.device_status(0) == 0


@pytest.mark.parametrize("m,k,pad", [(37, 36, 6), (300, 1024, 0), (65, 14336, 16), (3, 16384, 0)])
def test_swiglu_quantizer_paths_vs_oracle(m, k, pad):
    """Every quantizer path (scalar, warp-per-row, CTA-per-row) with strided [gate | up] rows."""
    gen = torch.Generator().manual_seed(k + m)
    xfull = randn_bf16((m, 2 * k + pad), gen, std=2.0)
    x = xfull.cuda()[:, :2 * k]
    q, s = h3b200.quantize_int8_rowwise(x, input_act="swiglu")
    oq, os_ = O.quantize_int8_rowwise(O.swiglu_bf16(t2u(xfull[:, :2 * k].contiguous())))
    np.testing.assert_array_equal(np_(q), oq)
    np.testing.assert_array_equal(np_(s), os_)


def test_swiglu_convrot_quantizer_vs_oracle():
    """ConvRot-256 after SwiGLU at the H3 fc2 width (ffn 14,336 = 56 groups, per-row kernel)."""
    gen = torch.Generator().manual_seed(51)
    m, k = 400, 14336
    x = randn_bf16((m, 2 * k), gen, std=2.0)
    q, s = h3b200.quantize_int8_rowwise_convrot(x.cuda(), 256, input_act="swiglu")
    oq, os_ = O.quantize_int8_rowwise(O.rotate_activation(O.swiglu_bf16(t2u(x)), 256))
    rows = (np_(q) == oq).all(-1)
    assert rows.mean() >= 0.9                    # fp32 butterfly vs exact rotation: rare bf16 flips
    assert np.abs(np_(q).astype(np.int32) - oq).max() <= 1
    assert h3b200.device_status(0) == 0
