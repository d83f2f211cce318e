"""Generate golden vectors by running X-MinimaxH3's own eager implementation.

Run once in a container where the reference checkout is importable:

    python tests/golden/make_golden.py --reference <path-to-X-MinimaxH3>

It imports the reference's vendored ``comfy_kitchen`` eager backend and the
``h3serve`` model helpers (nothing is copied), draws seeded synthetic inputs,
runs the reference functions on CPU and writes compressed ``.npz`` fixtures next
to this file. bf16 tensors are stored as uint16 bit patterns. The tests and the
GPU parity checks read only the fixtures; the reference is never needed at run
time.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def b16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--only", nargs="*", default=None, help="write only these fixtures (names without .npz)")
    args = ap.parse_args()
    ref = os.path.abspath(args.reference)
    sys.path.insert(0, os.path.join(ref, "backends", "turbo", "vendor"))
    sys.path.insert(0, ref)

    from comfy_kitchen.backends._activations import apply_input_act
    from comfy_kitchen.backends.eager import quantization as eq
    from comfy_kitchen.backends.eager import rope as erope
    from comfy_kitchen.backends.eager import w4a8_int8 as ew4
    from comfy_kitchen.tensor.int8_utils import _build_hadamard
    from h3serve.native_engine.model import layers as h3layers

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    out = {}

    # 1. tanh-GELU on every bf16 bit pattern.
    allb = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    out["gelu_tanh_bf16_all"] = {"y": b16(apply_input_act(allb.clone(), "gelu_tanh"))}

    # 2. Row quantizer: config-0 activations plus edge rows.
    g = torch.Generator().manual_seed(1)
    x = torch.randn(256, 3072, generator=g).to(torch.bfloat16)
    x[3] = 0                      # all-zero row -> scale clamps to 1e-30
    x[5, 7] = 1e4                 # one dominant value
    x[6] *= 1e-20                 # tiny row
    x[7, :] = -2.5                # constant row, ties at the clamp
    x[8, ::2] = 0.5
    x[9, 100] = -3.0e38           # near bf16 max
    q, s = eq.quantize_int8_rowwise(x)
    g2 = torch.Generator().manual_seed(11)
    ragged = (torch.randn(37, 40, generator=g2) * 3).to(torch.bfloat16)   # odd rows, K % 16 != 0
    rq, rs = eq.quantize_int8_rowwise(ragged)
    one = (torch.randn(1, 12288, generator=g2)).to(torch.bfloat16)
    oq, os_ = eq.quantize_int8_rowwise(one)
    out["quantize_rowwise"] = {
        "x": b16(x), "q": q.numpy(), "s": s.numpy(),
        "x_ragged": b16(ragged), "q_ragged": rq.numpy(), "s_ragged": rs.numpy(),
        "x_one": b16(one), "q_one": oq.numpy(), "s_one": os_.numpy(),
    }

    # 3. W8A8 linear, config-0 slice: x [256,3072] seed 1, W rows 0..383 of the seed-0 weight.
    gw = torch.Generator().manual_seed(0)
    w = (torch.randn(12288, 3072, generator=gw) * 0.02).to(torch.bfloat16)[:384].contiguous()
    wq, ws = eq.quantize_int8_rowwise(w)
    ws = ws.reshape(-1)
    gx = torch.Generator().manual_seed(1)
    x0 = torch.randn(256, 3072, generator=gx).to(torch.bfloat16)
    xq, xs = eq.quantize_int8_rowwise(x0)
    acc = eq._int8_matmul_accumulate(xq, wq.T.contiguous())
    y = eq.int8_linear(x0, wq, ws, None, torch.bfloat16)
    gb = torch.Generator().manual_seed(5)
    bias = torch.randn(384, generator=gb).to(torch.bfloat16)
    yb = eq.int8_linear(x0, wq, ws, bias, torch.bfloat16)
    ya = eq.int8_linear(x0, wq, ws, None, torch.bfloat16, input_act="gelu_tanh")
    out["linear_cfg0_slice"] = {
        "w_bf16": b16(w), "wq": wq.numpy(), "ws": ws.numpy(), "x": b16(x0), "xq": xq.numpy(),
        "xs": xs.numpy(), "acc": acc.numpy(), "y": b16(y), "bias": b16(bias), "y_bias": b16(yb),
        "y_gelu_in": b16(ya),
    }

    # 4. Gated tanh-GELU W8A8 MLP at reduced width (d=256, ffn=1024, M=100).
    gm = torch.Generator().manual_seed(2)
    d, ffn, m = 256, 1024, 100
    w1 = (torch.randn(ffn, d, generator=gm) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(d, ffn, generator=gm) * 0.02).to(torch.bfloat16)
    xm = torch.randn(m, d, generator=gm).to(torch.bfloat16)
    gate = torch.randn(d, generator=gm).to(torch.bfloat16)
    resid = torch.randn(m, d, generator=gm).to(torch.bfloat16)
    w1q, s1 = eq.quantize_int8_rowwise(w1)
    w2q, s2 = eq.quantize_int8_rowwise(w2)
    s1, s2 = s1.reshape(-1), s2.reshape(-1)
    h = eq.int8_linear(xm, w1q, s1, None, torch.bfloat16)
    a = apply_input_act(h, "gelu_tanh")
    q2, xs2 = eq.quantize_int8_rowwise(a)
    acc2 = eq._int8_matmul_accumulate(q2, w2q.T.contiguous())
    ym = eq.int8_linear(h, w2q, s2, None, torch.bfloat16, input_act="gelu_tanh")
    om = resid.clone().addcmul_(ym, gate)
    out["mlp_small"] = {
        "x": b16(xm), "w1q": w1q.numpy(), "s1": s1.numpy(), "w2q": w2q.numpy(), "s2": s2.numpy(),
        "gate": b16(gate), "residual": b16(resid), "h": b16(h), "a": b16(a), "q2": q2.numpy(),
        "xs2": xs2.numpy(), "acc2": acc2.numpy(), "y": b16(ym), "out": b16(om),
    }

    # 5. AdaLN-modulate + RMSNorm + 3-D split-half RoPE, 24x128 heads, grid (2,5,8).
    gr = torch.Generator().manual_seed(4)
    grid = (2, 5, 8)
    mt = grid[0] * grid[1] * grid[2]
    qn = torch.randn(mt, 24, 128, generator=gr).to(torch.bfloat16)
    kn = torch.randn(mt, 24, 128, generator=gr).to(torch.bfloat16)
    shift = (torch.randn(3072, generator=gr) * 0.1).to(torch.bfloat16)
    scale = (torch.randn(3072, generator=gr) * 0.1).to(torch.bfloat16)
    wq_ = (1 + 0.02 * torch.randn(3072, generator=gr)).to(torch.bfloat16)
    wk_ = (1 + 0.02 * torch.randn(3072, generator=gr)).to(torch.bfloat16)
    wqh = (1 + 0.02 * torch.randn(128, generator=gr)).to(torch.bfloat16)
    wkh = (1 + 0.02 * torch.randn(128, generator=gr)).to(torch.bfloat16)
    tt, hh, ww = torch.meshgrid(torch.arange(grid[0]), torch.arange(grid[1]), torch.arange(grid[2]), indexing="ij")
    pos = torch.stack([tt.reshape(-1), hh.reshape(-1), ww.reshape(-1)], dim=1)
    invs = [1.0 / (10000.0 ** (torch.arange(0, dd, 2, dtype=torch.float32) / dd)) for dd in (44, 42, 42)]
    half = torch.cat([pos[:, i:i + 1].float() * invs[i].reshape(1, -1) for i in range(3)], dim=-1)
    angles = torch.cat((half, half), dim=-1)
    table = h3layers.rope_rotation_table(angles, torch.float32)   # [1, M, 1, 64, 2, 2]

    class _Norm:  # the RMSNorm call used by kernels.rms_adaln's eager branch
        def __init__(self, weight):
            self.weight = weight

        def __call__(self, value):
            return torch.nn.functional.rms_norm(value, (self.weight.shape[0],), weight=self.weight, eps=1e-6)

    def adaln_rope(xx, wgt):
        hid = _Norm(wgt)(xx.reshape(mt, 3072))
        hid.mul_(1.0 + scale.to(hid.dtype)).add_(shift.to(hid.dtype))
        return erope.apply_rope_split_half1(hid.reshape(1, mt, 24, 128), table)[0]

    qo, ko = adaln_rope(qn, wq_), adaln_rope(kn, wk_)
    qh, kh = erope.rms_rope_split_half(qn.unsqueeze(0), kn.unsqueeze(0), table, wqh, wkh, 1e-6, 0)
    qp, kp = erope.rms_rope_split_half(qn.unsqueeze(0), kn.unsqueeze(0), table[..., :48, :, :], wqh, wkh, 1e-6, 96)
    out["norm_rope"] = {
        "q": b16(qn), "k": b16(kn), "shift": b16(shift), "scale": b16(scale), "wq": b16(wq_),
        "wk": b16(wk_), "wq_head": b16(wqh), "wk_head": b16(wkh), "grid": np.array(grid),
        "table": table.reshape(mt, 64, 2, 2).numpy(), "q_out": b16(qo), "k_out": b16(ko),
        "q_head": b16(qh[0]), "k_head": b16(kh[0]), "q_partial96": b16(qp[0]), "k_partial96": b16(kp[0]),
    }

    # 6. W4A8 asymmetric group-128, fp32 s_rel, ConvRot-256 (N=256, K=512, M=64).
    g4 = torch.Generator().manual_seed(3)
    w4 = (torch.randn(256, 512, generator=g4) * 0.02).to(torch.bfloat16)
    x4 = torch.randn(64, 512, generator=g4).to(torch.bfloat16)
    qd, srel, sch, corr, cb = ew4.quantize_w4a8_int8_weight(
        w4, group_size=128, convrot_groupsize=256, symmetric=False, scale_dtype=torch.float32, codebook=False)
    assert cb is None
    grid8 = ew4._dequant_int4_grouped_to_int8(qd, srel, None, 128)
    hmat = _build_hadamard(256, dtype=torch.bfloat16)
    xr = torch.matmul(x4.reshape(-1, 2, 256), hmat).reshape(64, 512)
    xq4, xs4 = eq.quantize_and_rotate_rowwise(x4, hmat, 256)
    acc4 = eq._int8_matmul_accumulate(xq4, grid8.T.contiguous())
    y4 = ew4.w4a8_int8_linear(x4, qd, srel, sch, None, corr, None, 128, 256, torch.bfloat16)
    out["w4a8_small"] = {
        "w_bf16": b16(w4), "x": b16(x4), "qdata": qd.numpy(), "s_rel": srel.numpy(), "s_channel": sch.numpy(),
        "correction": b16(corr), "grid": grid8.numpy(), "x_rot": b16(xr), "xq": xq4.numpy(), "xs": xs4.numpy(),
        "acc": acc4.numpy(), "y_eager": b16(y4),
    }

    # 7. SiLU on every bf16 bit pattern (the swiglu gate, up = 1 so the product is exact).
    ones = torch.ones(65536, dtype=torch.bfloat16)
    out["silu_bf16_all"] = {"y": b16(apply_input_act(torch.cat([allb, ones]).reshape(1, -1), "swiglu").reshape(-1))}

    # 8. SwiGLU input activation into an INT8 linear (x rows [gate | up], K = 512, N = 192),
    #    plain and ConvRot (weights rotated offline by the reference's own helper).
    gs_ = torch.Generator().manual_seed(6)
    xs_ = (torch.randn(64, 1024, generator=gs_) * 2).to(torch.bfloat16)
    wsw = (torch.randn(192, 512, generator=gs_) * 0.02).to(torch.bfloat16)
    swq, sws = eq.quantize_int8_rowwise(wsw)
    sws = sws.reshape(-1)
    act = apply_input_act(xs_, "swiglu")
    aq, as_ = eq.quantize_int8_rowwise(act)
    ysw = eq.int8_linear(xs_, swq, sws, None, torch.bfloat16, input_act="swiglu")
    cwq, cws = eq.quantize_int8_convrot_weight(wsw, 256)
    cws = cws.reshape(-1)
    ysc = eq.int8_linear(xs_, cwq, cws, None, torch.bfloat16, convrot=True, convrot_groupsize=256, input_act="swiglu")
    out["swiglu_linear"] = {
        "x": b16(xs_), "wq": swq.numpy(), "ws": sws.numpy(), "act": b16(act), "aq": aq.numpy(), "as": as_.numpy(),
        "y": b16(ysw), "wq_convrot": cwq.numpy(), "ws_convrot": cws.numpy(), "y_convrot": b16(ysc),
    }

    # 9. H3 SwiGLU MLP at reduced width (d=256, ffn=512, M=96): ConvRot INT8 fc1 with bias,
    #    fused-act ConvRot fc2 with bias, gated residual over three modulation segments
    #    (the INT8 path of try_fused_gated_mlp, h3serve/native_engine/model/fused_mlp.py:366-424).
    gq = torch.Generator().manual_seed(7)
    d9, f9, m9 = 256, 512, 96
    w91 = (torch.randn(2 * f9, d9, generator=gq) * 0.02).to(torch.bfloat16)
    w92 = (torch.randn(d9, f9, generator=gq) * 0.02).to(torch.bfloat16)
    b91 = (torch.randn(2 * f9, generator=gq) * 0.1).to(torch.bfloat16)
    b92 = (torch.randn(d9, generator=gq) * 0.1).to(torch.bfloat16)
    x9 = torch.randn(m9, d9, generator=gq).to(torch.bfloat16)
    r9 = torch.randn(m9, d9, generator=gq).to(torch.bfloat16)
    g9 = torch.randn(3, d9, generator=gq).to(torch.bfloat16)
    segs = ((0, 40, 2), (40, 70, 0), (70, 96, 1))
    w91q, s91 = eq.quantize_int8_convrot_weight(w91, 256)
    w92q, s92 = eq.quantize_int8_convrot_weight(w92, 256)
    s91, s92 = s91.reshape(-1), s92.reshape(-1)
    raw9 = eq.int8_linear(x9, w91q, s91, b91, torch.bfloat16, convrot=True, convrot_groupsize=256)
    proj9 = eq.int8_linear(raw9, w92q, s92, b92, torch.bfloat16, convrot=True, convrot_groupsize=256,
                           input_act="swiglu")
    out9 = r9.clone()
    for a9, z9, row9 in segs:
        out9[a9:z9].addcmul_(proj9[a9:z9], g9[row9])
    out["swiglu_mlp_small"] = {
        "w1": b16(w91), "w2": b16(w92), "b1": b16(b91), "b2": b16(b92), "x": b16(x9), "residual": b16(r9),
        "gate": b16(g9), "segments": np.array(segs, dtype=np.int64), "w1q": w91q.numpy(), "s1": s91.numpy(),
        "w2q": w92q.numpy(), "s2": s92.numpy(), "raw": b16(raw9), "proj": b16(proj9), "out": b16(out9),
    }

    # 10. H3 release W4A8 format (quantize_w4a8_int8_weight defaults: group 16, symmetric,
    #     fp8-e4m3 s_rel, 16-level codebook, no correction; ConvRot-256).
    #     a) Gaussian weight (fixed codebook), its decode and its linear with a bias through
    #        the top-level comfy_kitchen.w4a8_int8_linear (tensor/w4a8_int8.py:89-115);
    #     b) a weight whose rotated groups are heavy-tailed (v^3 rotated back by H), so the
    #        codebook is fitted, with more elements than the kurtosis and fit samples;
    #     c) decode-only cases for the other group sizes, fp32 scales and the uniform
    #        symmetric branch;
    #     d) a reduced-width W4 SwiGLU MLP (d=256, ffn=512, M=96, biases, three modulation
    #        segments, 64-token chunks) through the reference's own W4A8 driver
    #        _chunked_module_gated_mlp (h3serve/native_engine/model/fused_mlp.py:222-266)
    #        with the production binding comfy_kitchen_w4a8_kernel (quantization.py:64-95).
    import types

    import comfy_kitchen as ck
    from h3serve.native_engine.model import fused_mlp as h3fused
    from h3serve.native_engine.model import quantization as h3quant

    def u8(t):
        return t.contiguous().view(torch.uint8).numpy().copy()

    gh = torch.Generator().manual_seed(8)
    wa = (torch.randn(384, 512, generator=gh) * 0.02).to(torch.bfloat16)
    xa = torch.randn(80, 512, generator=gh).to(torch.bfloat16)
    ba = (torch.randn(384, generator=gh) * 0.1).to(torch.bfloat16)
    qa, sra, sca, ca, cba = ew4.quantize_w4a8_int8_weight(wa)
    assert ca is None and cba is not None and sra.dtype == torch.float8_e4m3fn
    grida = ew4._dequant_int4_grouped_to_int8(qa, sra, cba, 16)
    ya = ck.w4a8_int8_linear(xa, qa, sra, sca, cba, None, ba, 16, 256, torch.bfloat16)
    h10 = _build_hadamard(256, dtype=torch.float32)
    zb = torch.randn(1088, 512, generator=gh)
    wb = ((zb * zb * zb * 0.01).reshape(1088, 2, 256) @ h10).reshape(1088, 512).to(torch.bfloat16)
    qb, srb, scb, cb_, cbb = ew4.quantize_w4a8_int8_weight(wb)
    fixed = torch.tensor(ew4._FIXED_LUT)
    assert not torch.equal(cbb, fixed), "the heavy-tailed case must take the fitted codebook"
    gridb = ew4._dequant_int4_grouped_to_int8(qb, srb, cbb, 16)
    arrays10 = {
        "w_a": b16(wa), "x_a": b16(xa), "b_a": b16(ba), "q_a": qa.numpy(), "s_rel_a": u8(sra), "s_ch_a": sca.numpy(),
        "codebook_a": cba.numpy(), "grid_a": grida.numpy(), "y_a": b16(ya),
        "w_b": b16(wb), "q_b": qb.numpy(), "s_rel_b": u8(srb), "s_ch_b": scb.numpy(), "codebook_b": cbb.numpy(),
        "grid_b": gridb.numpy(),
    }
    wc = (torch.randn(64, 512, generator=gh) * 0.02).to(torch.bfloat16)
    for tag, gsz, sdt, use_cb in (("g4_e4m3_cb", 4, torch.float8_e4m3fn, True), ("g8_e4m3_cb", 8, torch.float8_e4m3fn, True),
                                  ("g32_f32_cb", 32, torch.float32, True), ("g16_f32_uni", 16, torch.float32, False),
                                  ("g8_e4m3_uni", 8, torch.float8_e4m3fn, False)):
        qc, src_, scc, cc, cbc = ew4.quantize_w4a8_int8_weight(wc, gsz, 256, True, sdt, use_cb)
        assert cc is None and (cbc is not None) == use_cb
        arrays10[f"q_{tag}"] = qc.numpy()
        arrays10[f"s_rel_{tag}"] = u8(src_) if sdt != torch.float32 else src_.numpy()
        arrays10[f"s_ch_{tag}"] = scc.numpy()
        if use_cb:
            arrays10[f"codebook_{tag}"] = cbc.numpy()
        arrays10[f"grid_{tag}"] = ew4._dequant_int4_grouped_to_int8(qc, src_, cbc, gsz).numpy()
    arrays10["w_c"] = b16(wc)
    d10, f10, m10 = 256, 512, 96
    w101 = (torch.randn(2 * f10, d10, generator=gh) * 0.02).to(torch.bfloat16)
    w102 = (torch.randn(d10, f10, generator=gh) * 0.02).to(torch.bfloat16)
    b101 = (torch.randn(2 * f10, generator=gh) * 0.1).to(torch.bfloat16)
    b102 = (torch.randn(d10, generator=gh) * 0.1).to(torch.bfloat16)
    x10 = torch.randn(m10, d10, generator=gh).to(torch.bfloat16)
    r10 = torch.randn(m10, d10, generator=gh).to(torch.bfloat16)
    g10 = torch.randn(3, d10, generator=gh).to(torch.bfloat16)
    segs10 = ((0, 40, 2), (40, 70, 0), (70, 96, 1))
    p1 = ew4.quantize_w4a8_int8_weight(w101)
    p2 = ew4.quantize_w4a8_int8_weight(w102)

    def w4_linear(prep, bias):
        def run(v):
            return h3quant.comfy_kitchen_w4a8_kernel(v, prep[0], prep[1], prep[2], prep[4], prep[3], bias, 16, 256,
                                                     v.dtype)
        return run

    mlp10 = types.SimpleNamespace(fc1=w4_linear(p1, b101), fc2=w4_linear(p2, b102))
    out10 = r10.clone()
    h3fused._chunked_module_gated_mlp(out10, x10, mlp10, g10, segs10, chunk_tokens=64)
    raw10 = mlp10.fc1(x10)
    arrays10.update({
        "mlp_w1": b16(w101), "mlp_w2": b16(w102), "mlp_b1": b16(b101), "mlp_b2": b16(b102), "mlp_x": b16(x10),
        "mlp_residual": b16(r10), "mlp_gate": b16(g10), "mlp_segments": np.array(segs10, dtype=np.int64),
        "mlp_q1": p1[0].numpy(), "mlp_s_rel1": u8(p1[1]), "mlp_s_ch1": p1[2].numpy(), "mlp_codebook1": p1[4].numpy(),
        "mlp_q2": p2[0].numpy(), "mlp_s_rel2": u8(p2[1]), "mlp_s_ch2": p2[2].numpy(), "mlp_codebook2": p2[4].numpy(),
        "mlp_raw": b16(raw10), "mlp_out": b16(out10),
    })
    #     e) a heavy-tailed [640, 8192] weight regenerated from its seed by the test (too big
    #        to store): more rows than the codebook row sample (rows are then strided) and two
    #        preparation chunks; SHA-256 digests of the weight and of the outputs.
    import hashlib

    def digest(t):
        return np.frombuffer(hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).digest(), np.uint8)

    ge = torch.Generator().manual_seed(9)
    ze = torch.randn(640, 8192, generator=ge)
    we = ((ze * ze * ze * 0.01).reshape(640, 32, 256) @ h10).reshape(640, 8192).to(torch.bfloat16)
    qe, sre, sce, _, cbe = ew4.quantize_w4a8_int8_weight(we)
    assert not torch.equal(cbe, fixed)
    arrays10.update({"big_seed": np.array(9), "big_w_sha": digest(we), "big_q_sha": digest(qe),
                     "big_s_rel_sha": digest(sre), "big_s_ch": sce.numpy(), "big_codebook": cbe.numpy()})
    out["w4a8_h3"] = arrays10

    # 11. H3 QK-norm + partial RoPE at the H3 head layout (56 heads x 128, rot_dim 96 = 3 axes
    #     x 16 pairs, eps 1e-5), table from H3's own rope_frequencies / rope_rotation_table
    #     (layers.py:51-69) on a (t, h, w) grid, fp32 and bf16. Reference outputs: comfy eager
    #     rms_rope_split_half (fp32 table), the same with the bf16 table, and H3's CPU
    #     single-side path _apply_single_qknorm_rope (layers.py:152-231, bf16 table) for Q and K.
    gr = torch.Generator().manual_seed(10)
    m11, h11 = 16, 56
    inv11 = 1.0 / (10000.0 ** (torch.arange(0, 32, 2, dtype=torch.float32) / 32.0))
    tt, hh, ww = torch.meshgrid(torch.arange(2) + 3, torch.arange(2) + 17, torch.arange(4) + 29, indexing="ij")
    pos11 = torch.stack([tt.reshape(-1), hh.reshape(-1), ww.reshape(-1)], dim=-1)
    ang11 = h3layers.rope_frequencies(pos11, inv11)
    tab32 = h3layers.rope_rotation_table(ang11, torch.float32)
    tab16 = h3layers.rope_rotation_table(ang11, torch.bfloat16)
    q11 = (torch.randn(m11, h11, 128, generator=gr) * 1.5).to(torch.bfloat16)
    k11 = (torch.randn(m11, h11, 128, generator=gr) * 0.7).to(torch.bfloat16)
    wq11 = (1 + 0.02 * torch.randn(128, generator=gr)).to(torch.bfloat16)
    wk11 = (1 + 0.02 * torch.randn(128, generator=gr)).to(torch.bfloat16)
    q32, k32 = erope.rms_rope_split_half(q11.unsqueeze(0), k11.unsqueeze(0), tab32, wq11, wk11, 1e-5, 96)
    q16, k16 = erope.rms_rope_split_half(q11.unsqueeze(0), k11.unsqueeze(0), tab16, wq11, wk11, 1e-5, 96)
    qh3 = h3layers._apply_single_qknorm_rope(q11, weight=wq11, frequencies=tab16, eps=1e-5, query_slot=True)
    kh3 = h3layers._apply_single_qknorm_rope(k11, weight=wk11, frequencies=tab16, eps=1e-5, query_slot=False)
    out["qknorm_rope_h3"] = {
        "q": b16(q11), "k": b16(k11), "wq": b16(wq11), "wk": b16(wk11), "table_f32": tab32.reshape(m11, 48, 2, 2).numpy(),
        "table_bf16": b16(tab16.reshape(m11, 48, 2, 2)), "q_f32tab": b16(q32[0]), "k_f32tab": b16(k32[0]),
        "q_bf16tab": b16(q16[0]), "k_bf16tab": b16(k16[0]), "q_h3": b16(qh3), "k_h3": b16(kh3),
    }

    # 12. RMS-AdaLN on the hidden stream.
    #  (a) H3 rms_adaln(value, norm, shift, scale, segments) (kernels.py:7586-7634, eager branch on
    #      CPU) at the H3 width 5,376 with three modulation segments: an RMSNorm module with an fp32
    #      weight (cast to bf16 in its forward), shift/scale as the fp32 [rows, hidden] views that
    #      split_adaln cuts from a [1, 18 * hidden] projection (cast by .to(bf16)), and edge rows
    #      (zero, tiny, one huge value, constant).
    #  (b) comfy_kitchen rms_adaln(x, scale, shift, eps) (eager/adaln.py:17-20, no weight) with
    #      per-sample [B, 1, D] modulation.
    import importlib

    from h3serve.native_engine.model import kernels as h3kernels

    eadaln = importlib.import_module("comfy_kitchen.backends.eager.adaln")  # the package re-exports a function

    gm = torch.Generator().manual_seed(12)
    m12, d12 = 96, 5376
    v12 = (torch.randn(m12, d12, generator=gm) * 1.3).to(torch.bfloat16)
    v12[4] = 0
    v12[9] = (v12[9].float() * 1e-30).to(torch.bfloat16)
    v12[11, 5] = 3.0e38
    v12[17] = -2.0
    norm12 = h3layers.RMSNorm(d12, eps=1e-6)
    with torch.no_grad():
        norm12.weight.copy_(1 + 0.05 * torch.randn(d12, generator=gm))
    proj = torch.randn(1, 18 * d12, generator=gm) * 0.2
    shift_a, scale_a = h3layers.split_adaln(proj, hidden_size=d12)[:2]
    segs12 = ((0, 25, 2), (25, 60, 0), (60, m12, 1))
    o12 = h3kernels.rms_adaln(v12.clone(), norm12, shift_a, scale_a, segs12)
    xb = torch.randn(2, 48, 3072, generator=gm).to(torch.bfloat16)
    scb = (torch.randn(2, 1, 3072, generator=gm) * 0.1).to(torch.bfloat16)
    shb = (torch.randn(2, 1, 3072, generator=gm) * 0.1).to(torch.bfloat16)
    ob = eadaln.rms_adaln(xb, scb, shb, 1e-6)
    assert o12.dtype == torch.bfloat16 and ob.dtype == torch.bfloat16
    out["rms_adaln"] = {
        "x_h3": b16(v12), "w_h3": b16(norm12.weight.detach().to(torch.bfloat16)),
        "shift_rows": shift_a.contiguous().numpy(), "scale_rows": scale_a.contiguous().numpy(),
        "segments": np.array(segs12, dtype=np.int64), "eps_h3": np.float32(norm12.eps), "out_h3": b16(o12),
        "x_cf": b16(xb), "scale_cf": b16(scb), "shift_cf": b16(shb), "out_cf": b16(ob),
    }

    # fp16 activations and outputs: the same eager quantizer and linear with x in fp16
    # (edge rows: zero, a scale that underflows fp16, values near the fp16 maximum) and
    # out_dtype fp16, plus bf16 x -> fp16 out and fp16 x -> bf16 out.
    g16 = torch.Generator().manual_seed(16)
    x16 = (torch.randn(96, 512, generator=g16) * 2).to(torch.float16)
    x16[1] = 0
    x16[2] = (torch.randn(512, generator=g16) * 1e-7).to(torch.float16)   # fp16 subnormals
    x16[3, 5] = 6.0e4
    x16[4, :] = -1.5
    w16 = (torch.randn(160, 512, generator=g16) * 0.02).to(torch.bfloat16)
    wq16, ws16 = eq.quantize_int8_rowwise(w16)
    ws16 = ws16.reshape(-1)
    q16, s16 = eq.quantize_int8_rowwise(x16)
    bias16 = torch.randn(160, generator=g16).to(torch.float16)
    xbf = torch.randn(96, 512, generator=g16).to(torch.bfloat16)
    biasbf = torch.randn(160, generator=g16).to(torch.bfloat16)
    y16 = eq.int8_linear(x16, wq16, ws16, None, torch.float16)
    y16b = eq.int8_linear(x16, wq16, ws16, bias16, torch.float16)
    ymix = eq.int8_linear(xbf, wq16, ws16, biasbf, torch.float16)
    y16bf = eq.int8_linear(x16, wq16, ws16, None, torch.bfloat16)
    assert y16.dtype == torch.float16 and ymix.dtype == torch.float16 and y16bf.dtype == torch.bfloat16

    def h16(t):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()

    out["fp16_linear"] = {
        "x16": h16(x16), "q16": q16.numpy(), "s16": s16.numpy(), "wq": wq16.numpy(), "ws": ws16.numpy(),
        "bias16": h16(bias16), "xbf": b16(xbf), "biasbf": b16(biasbf),
        "y16": h16(y16), "y16_bias": h16(y16b), "y_bf_in_f16_out": h16(ymix), "y_f16_in_bf_out": b16(y16bf),
    }

    for name, arrays in out.items():
        if args.only is not None and name not in args.only:
            continue
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **arrays)
        print(f"wrote {path} ({os.path.getsize(path)} bytes)")


if __name__ == "__main__":
    main()
