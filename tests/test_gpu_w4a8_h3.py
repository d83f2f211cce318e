"""GPU parity: the H3 release W4A8 format (group 16, fp8-e4m3 s_rel, 16-level codebook).

The decode is bit-exact against the reference's fixtures and the oracle for every
scale type, level table and group size (vector and unaligned scalar kernels, all 256
fp8 scale patterns). The linear with a bias equals the ConvRot INT8 linear on the
decoded grid bit for bit and is within the north-star tolerance of the reference (its
rotation is a bf16 matmul). The fused W4 SwiGLU MLP equals the chain of single ops and
the INT8 SwiGLU MLP on the decoded grids bit for bit, and is within tolerance of the
reference's own W4A8 MLP driver.
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


def s_rel_t(a):
    """fixture s_rel (uint8 e4m3 bits or fp32) -> CUDA tensor of the matching dtype"""
    t = torch.from_numpy(np.ascontiguousarray(a))
    return (t.view(torch.float8_e4m3fn) if a.dtype == np.uint8 else t).cuda()


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_decode_vs_reference_all_variants(golden):
    fx = golden("w4a8_h3")
    cases = [("a", 16, True), ("b", 16, True), ("g4_e4m3_cb", 4, True), ("g8_e4m3_cb", 8, True),
             ("g32_f32_cb", 32, True), ("g16_f32_uni", 16, False), ("g8_e4m3_uni", 8, False)]
    for tag, gsz, use_cb in cases:
        cb = cuda(fx[f"codebook_{tag}"]) if use_cb else None
        grid = h3b200.dequant_int4_grouped_to_int8(cuda(fx[f"q_{tag}"]), s_rel_t(fx[f"s_rel_{tag}"]), gsz, cb)
        np.testing.assert_array_equal(np_(grid), fx[f"grid_{tag}"], err_msg=tag)
    assert h3b200.device_status(0) == 0


@pytest.mark.parametrize("group", [4, 8, 16, 32, 128])
@pytest.mark.parametrize("e4m3", [True, False])
@pytest.mark.parametrize("use_cb", [True, False])
def test_decode_vs_oracle(group, e4m3, use_cb):
    gen = torch.Generator().manual_seed(group * 4 + 2 * e4m3 + use_cb)
    n, k = 300, 1024
    q = torch.randint(-128, 128, (n, k // 2), generator=gen, dtype=torch.int8)
    s = torch.rand(n, k // group, generator=gen) * 140.0
    s_rel = s.to(torch.float8_e4m3fn) if e4m3 else s
    cb = torch.sort(torch.rand(16, generator=gen) * 2 - 1).values if use_cb else None
    grid = h3b200.dequant_int4_grouped_to_int8(q.cuda(), s_rel.cuda(), group, None if cb is None else cb.cuda())
    ref = O.decode_int4_grouped_to_int8(q.numpy(), s_rel.view(torch.uint8).numpy() if e4m3 else s.numpy(), group,
                                        None if cb is None else cb.numpy())
    np.testing.assert_array_equal(np_(grid), ref)


def test_decode_every_e4m3_scale_and_unaligned_buffers():
    """All 256 fp8 patterns as group scales (NaN scales decode to 0), through the vector kernel
    and, with buffers off their 8/16-byte alignment, the scalar kernel."""
    gen = torch.Generator().manual_seed(77)
    n, group = 256, 16
    k = 16 * group
    q = torch.randint(-128, 128, (n, k // 2), generator=gen, dtype=torch.int8)
    sb = torch.arange(256, dtype=torch.int32).to(torch.uint8).reshape(256, 1).repeat(1, k // group)
    sb = sb[torch.randperm(256, generator=gen)]
    cb = torch.linspace(-0.99, 0.97, 16)
    s_rel = sb.view(torch.float8_e4m3fn)
    lib = h3b200.library()
    for use_cb in (True, False):
        # NaN scales (0x7F, 0xFF) decode to 0, as a zero scale does
        finite_bits = np.where(np.isin(sb.numpy(), (0x7F, 0xFF)), 0, sb.numpy()).astype(np.uint8)
        ref = O.decode_int4_grouped_to_int8(q.numpy(), finite_bits, group, cb.numpy() if use_cb else None)
        grid = h3b200.dequant_int4_grouped_to_int8(q.cuda(), s_rel.cuda(), group, cb.cuda() if use_cb else None)
        np.testing.assert_array_equal(np_(grid), ref)
        # unaligned: qdata at a 1-byte offset, output at a 1-byte offset
        qbuf = torch.zeros(n * k // 2 + 1, dtype=torch.int8, device="cuda")
        qu = qbuf[1:].view(n, k // 2)
        qu.copy_(q.cuda())
        obuf = torch.zeros(n * k + 1, dtype=torch.int8, device="cuda")
        cbd = cb.cuda() if use_cb else None
        st = lib.h3b200_dequant_int4_grouped_to_int8_ex(qu.data_ptr(), s_rel.cuda().contiguous().data_ptr(), 5,
                                                        cbd.data_ptr() if cbd is not None else None, n, k, group,
                                                        obuf.data_ptr() + 1, torch.cuda.current_stream().cuda_stream)
        assert st == 0
        np.testing.assert_array_equal(np_(obuf[1:]).reshape(n, k), ref)
    assert h3b200.device_status(0) == 0


def test_decode_rejects_bad_arguments():
    q = torch.zeros(4, 256, dtype=torch.int8, device="cuda")
    with pytest.raises(ValueError):
        h3b200.dequant_int4_grouped_to_int8(q, torch.zeros(4, 32, dtype=torch.float16, device="cuda"), 16)
    with pytest.raises(ValueError):
        h3b200.dequant_int4_grouped_to_int8(q, torch.zeros(4, 32, device="cuda"), 16,
                                            torch.zeros(8, device="cuda"))
    lib = h3b200.library()
    assert lib.h3b200_dequant_int4_grouped_to_int8_ex(q.data_ptr(), q.data_ptr(), 2, None, 4, 512, 16, q.data_ptr(),
                                                      None) == 1
    assert lib.h3b200_dequant_int4_grouped_to_int8_ex(q.data_ptr(), q.data_ptr(), 5, None, 4, 512, 12, q.data_ptr(),
                                                      None) == 1


def test_w4a8_linear_release_format_vs_reference(golden):
    fx = golden("w4a8_h3")
    x, b = u2t(fx["x_a"]), u2t(fx["b_a"])
    q, s_rel, s_ch, cb = cuda(fx["q_a"]), s_rel_t(fx["s_rel_a"]), cuda(fx["s_ch_a"]), cuda(fx["codebook_a"])
    y = h3b200.w4a8_int8_linear(x, q, s_rel, s_ch, cb, None, b, 16, 256)
    assert h3b200.device_status(0) == 0
    rel, mx = rel_l2(t2u(y), fx["y_a"])
    assert rel <= 1e-2 and mx <= 2e-2
    grid = h3b200.dequant_int4_grouped_to_int8(q, s_rel, 16, cb)
    same = h3b200.int8_linear(x, grid, s_ch, b, convrot=True, convrot_groupsize=256)
    np.testing.assert_array_equal(t2u(y), t2u(same))
    ref = O.w4a8_symmetric_linear(fx["x_a"], fx["q_a"], fx["s_rel_a"], fx["s_ch_a"], fx["codebook_a"], fx["b_a"])
    rel, mx = rel_l2(t2u(y), ref)
    assert rel <= 1e-2 and mx <= 2e-2
    # a bias with an (all-zero) asymmetric correction: the correction adds exactly 0 to the
    # bf16 dequant + bias value, so the result is the symmetric one bit for bit
    yc = h3b200.w4a8_int8_linear(x, q, s_rel, s_ch, cb, torch.zeros(32, 384, dtype=torch.bfloat16, device="cuda"), b)
    np.testing.assert_array_equal(t2u(yc), t2u(y))


def _w4(fx):
    return h3b200.W4A8SwiGLUMLPWeights(cuda(fx["mlp_q1"]), s_rel_t(fx["mlp_s_rel1"]), cuda(fx["mlp_s_ch1"]),
                                       cuda(fx["mlp_q2"]), s_rel_t(fx["mlp_s_rel2"]), cuda(fx["mlp_s_ch2"]),
                                       cuda(fx["mlp_codebook1"]), cuda(fx["mlp_codebook2"]), u2t(fx["mlp_b1"]),
                                       u2t(fx["mlp_b2"]), 16)


def _grids(w4):
    g1 = h3b200.dequant_int4_grouped_to_int8(w4.q1, w4.s_rel1, w4.group_size, w4.codebook1)
    g2 = h3b200.dequant_int4_grouped_to_int8(w4.q2, w4.s_rel2, w4.group_size, w4.codebook2)
    return h3b200.SwiGLUMLPWeights(g1, w4.s_ch1, g2, w4.s_ch2, w4.b1, w4.b2, True)


def _chain(x, w4, gate_rows, row_map, res):
    """The reference's W4A8 driver through h3b200's single ops (fc1, SwiGLU, fc2), gated
    residual in numpy fp32."""
    raw = h3b200.w4a8_int8_linear(x, w4.q1, w4.s_rel1, w4.s_ch1, w4.codebook1, None, w4.b1, w4.group_size)
    act = h3b200.apply_input_act(raw, "swiglu")
    y = h3b200.w4a8_int8_linear(act, w4.q2, w4.s_rel2, w4.s_ch2, w4.codebook2, None, w4.b2, w4.group_size)
    f = O.bf16_to_f32
    g = f(t2u(gate_rows)).reshape(-1, y.shape[-1])[row_map]
    return O.f32_to_bf16(f(t2u(res)) + f(t2u(y)) * g)


def test_w4_swiglu_mlp_vs_reference_chain_and_int8_path(golden):
    fx = golden("w4a8_h3")
    w4 = _w4(fx)
    segs = [tuple(int(v) for v in s) for s in fx["mlp_segments"]]
    x, res, gate = u2t(fx["mlp_x"]), u2t(fx["mlp_residual"]), u2t(fx["mlp_gate"])
    out = h3b200.fused_gated_mlp_swiglu_w4a8(res, x, w4, gate, segments=segs, chunk_tokens=64)
    assert h3b200.device_status(0) == 0
    rel, mx = rel_l2(t2u(out), fx["mlp_out"])
    assert rel <= 1e-2 and mx <= 2e-2
    row_map = np.concatenate([np.full(b - a, r) for a, b, r in segs])
    np.testing.assert_array_equal(t2u(out), _chain(x, w4, gate, row_map, res))
    np.testing.assert_array_equal(t2u(out), t2u(h3b200.fused_gated_mlp_swiglu(res, x, _grids(w4), gate,
                                                                              segments=segs)))
    w4np = {"q1": fx["mlp_q1"], "s_rel1": fx["mlp_s_rel1"], "s_ch1": fx["mlp_s_ch1"], "codebook1": fx["mlp_codebook1"],
            "b1": fx["mlp_b1"], "q2": fx["mlp_q2"], "s_rel2": fx["mlp_s_rel2"], "s_ch2": fx["mlp_s_ch2"],
            "codebook2": fx["mlp_codebook2"], "b2": fx["mlp_b2"], "group_size": 16}
    rel, mx = rel_l2(t2u(out), O.w4a8_swiglu_mlp(fx["mlp_x"], w4np, fx["mlp_gate"], row_map, fx["mlp_residual"]))
    assert rel <= 1e-2 and mx <= 2e-2


def test_w4_swiglu_mlp_h3_dims_chunked_in_place():
    """H3 dims (d 5,376, fc1 28,672, ffn 14,336) at 600 tokens with weights prepared on the GPU
    in the release format: equal to the INT8 SwiGLU MLP on the decoded grids and to the op
    chain, the same in 256-token chunks and in place."""
    gen = torch.Generator().manual_seed(62)
    d, ffn, m = 5376, 14336, 600
    w1 = randn_bf16((2 * ffn, d), gen, std=0.02).cuda()
    w2 = randn_bf16((d, ffn), gen, std=0.02).cuda()
    b1 = randn_bf16((2 * ffn,), gen, std=0.1).cuda()
    b2 = randn_bf16((d,), gen, std=0.1).cuda()
    x = randn_bf16((m, d), gen).cuda()
    res = randn_bf16((m, d), gen).cuda()
    gate = randn_bf16((2, d), gen).cuda()
    segs = [(0, 333, 1), (333, m, 0)]
    w4 = h3b200.W4A8SwiGLUMLPWeights.from_float(w1, w2, b1, b2)
    assert w4.s_rel1.dtype == torch.float8_e4m3fn and w4.codebook1 is not None
    out = h3b200.fused_gated_mlp_swiglu_w4a8(res, x, w4, gate, segments=segs)
    assert h3b200.device_status(0) == 0
    np.testing.assert_array_equal(t2u(out), t2u(h3b200.fused_gated_mlp_swiglu(res, x, _grids(w4), gate,
                                                                              segments=segs)))
    row_map = np.concatenate([np.full(b - a, r) for a, b, r in segs])
    np.testing.assert_array_equal(t2u(out), _chain(x, w4, gate, row_map, res))
    chunked = h3b200.fused_gated_mlp_swiglu_w4a8(res, x, w4, gate, segments=segs, chunk_tokens=256)
    np.testing.assert_array_equal(t2u(chunked), t2u(out))
    r2 = res.clone()
    h3b200.fused_gated_mlp_swiglu_w4a8(r2, x, w4, gate, segments=segs, out=r2, chunk_tokens=256)
    np.testing.assert_array_equal(t2u(r2), t2u(out))
