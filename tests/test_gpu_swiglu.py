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
    assert rel <= 1e-2 and mx <= 2e-2                 # the reference's rotation is a bf16 CPU matmul
    qc, sc = O.quantize_int8_rowwise(O.rotate_activation(O.apply_input_act(g["x"], "swiglu"), 256))
    np.testing.assert_array_equal(t2u(yc), O.dequant_epilogue(O.int8_matmul_accumulate(qc, g["wq_convrot"]), sc,
                                                              g["ws_convrot"]))
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


@pytest.mark.parametrize("k", [14336, 5376])
def test_swiglu_convrot_quantizer_vs_oracle(k):
    """ConvRot-256 after SwiGLU ([gate | up] rows, exact SiLU and product) at the H3 fc2 width
    (ffn 14,336 = 56 groups) and at 5,376: bit-exact int8 values and scales."""
    gen = torch.Generator().manual_seed(51)
    m = 400
    x = randn_bf16((m, 2 * k), gen, std=2.0)
    q, s = h3b200.quantize_int8_rowwise_convrot(x.cuda(), 256, input_act="swiglu")
    oq, os_ = O.quantize_int8_rowwise(O.rotate_activation(O.swiglu_bf16(t2u(x)), 256))
    np.testing.assert_array_equal(np_(q), oq)
    np.testing.assert_array_equal(np_(s), os_)
    assert h3b200.device_status(0) == 0


def _chain(x, wt, gate_rows, row_map, res):
    """The reference's composition through h3b200's single ops, gated residual in numpy fp32."""
    raw = h3b200.int8_linear(x, wt.w1q, wt.s1, wt.b1, convrot=wt.fc1_convrot)
    y = h3b200.int8_linear(raw, wt.w2q, wt.s2, wt.b2, convrot=True, input_act="swiglu")
    f = O.bf16_to_f32
    g = f(t2u(gate_rows)).reshape(-1, y.shape[-1])[row_map]
    return O.f32_to_bf16(f(t2u(res)) + f(t2u(y)) * g)


def test_convrot_weight_prep_vs_reference(golden):
    """Offline ConvRot weight rotation + per-channel quantization against the reference's
    quantize_int8_convrot_weight (its rotation is a bf16 CPU matmul: rare last-bit flips)."""
    g = golden("swiglu_mlp_small")
    for w, wq_ref, s_ref in ((g["w1"], g["w1q"], g["s1"]), (g["w2"], g["w2q"], g["s2"])):
        wq, s = h3b200.quantize_int8_convrot_weight(u2t(w))
        same = (np_(wq) == wq_ref).all(-1)
        assert same.mean() >= 0.95
        assert np.abs(np_(wq).astype(np.int32) - wq_ref).max() <= 1
        np.testing.assert_array_equal(np_(s)[same], s_ref[same])


def test_swiglu_mlp_vs_reference_and_chain(golden):
    g = golden("swiglu_mlp_small")
    wt = h3b200.SwiGLUMLPWeights(torch.from_numpy(g["w1q"]).cuda(), torch.from_numpy(g["s1"]).cuda(),
                                 torch.from_numpy(g["w2q"]).cuda(), torch.from_numpy(g["s2"]).cuda(),
                                 u2t(g["b1"]), u2t(g["b2"]))
    segs = [tuple(int(v) for v in s) for s in g["segments"]]
    x, res, gate = u2t(g["x"]), u2t(g["residual"]), u2t(g["gate"])
    out = h3b200.fused_gated_mlp_swiglu(res, x, wt, gate, segments=segs)
    assert h3b200.device_status(0) == 0
    rel, mx = rel_l2(t2u(out), g["out"])
    assert rel <= 1e-2 and mx <= 2e-2
    row_map = np.concatenate([np.full(b - a, r) for a, b, r in segs])
    np.testing.assert_array_equal(t2u(out), _chain(x, wt, gate, row_map, res))
    ref = O.swiglu_mlp(g["x"], g["w1q"], g["s1"], g["b1"], g["w2q"], g["s2"], g["b2"], g["gate"], row_map,
                       g["residual"])
    rel, mx = rel_l2(t2u(out), ref)
    assert rel <= 1e-2 and mx <= 2e-2


def test_swiglu_mlp_h3_dims_chunked_in_place():
    """H3 dims (d 5,376, fc1 28,672, ffn 14,336) at 600 tokens (CTA-pair GEMMs), two modulation
    segments and biases: equal to the op chain bit for bit, the same in 256-token chunks, and
    in place on the residual."""
    gen = torch.Generator().manual_seed(61)
    d, ffn, m = 5376, 14336, 600
    w1 = randn_bf16((2 * ffn, d), gen, std=0.02).cuda()
    w2 = randn_bf16((d, ffn), gen, std=0.02).cuda()
    b1 = randn_bf16((2 * ffn,), gen, std=0.1).cuda()
    b2 = randn_bf16((d,), gen, std=0.1).cuda()
    x = randn_bf16((m, d), gen).cuda()
    res = randn_bf16((m, d), gen).cuda()
    gate = randn_bf16((2, d), gen).cuda()
    segs = [(0, 217, 1), (217, m, 0)]
    wt = h3b200.SwiGLUMLPWeights.from_float(w1, w2, b1, b2)
    out = h3b200.fused_gated_mlp_swiglu(res, x, wt, gate, segments=segs)
    assert h3b200.device_status(0) == 0
    row_map = np.concatenate([np.full(b - a, r) for a, b, r in segs])
    np.testing.assert_array_equal(t2u(out), _chain(x, wt, gate, row_map, res))
    chunked = h3b200.fused_gated_mlp_swiglu(res, x, wt, gate, segments=segs, chunk_tokens=256)
    np.testing.assert_array_equal(t2u(chunked), t2u(out))
    r2 = res.clone()
    h3b200.fused_gated_mlp_swiglu(r2, x, wt, gate, segments=segs, out=r2, chunk_tokens=256)
    np.testing.assert_array_equal(t2u(r2), t2u(out))
