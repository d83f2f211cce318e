"""GPU parity: standalone RMS-AdaLN (segmented and per-sample modulation), the
segmented modulation of the fused norm-RoPE, and segmented gates of the W8A8 MLP.

Bit-exact against the oracle (pinned to the reference's eager outputs in
tests/golden/rms_adaln.npz) on the reference fixture, on seeded inputs at H3's
width 5,376 and config 3's 3,072, on widths that take the predicated kernel
instances, in place, on strided rows and strided modulation views, and at the
full config-3 token count.
"""

import numpy as np
import pytest
import torch

import h3b200
import oracle as O
from gpu_util import randn_bf16, t2u, u2t

pytestmark = pytest.mark.gpu


class _Norm:
    """Stands in for H3's RMSNorm module: a weight and an eps (layers.py:33-48)."""

    def __init__(self, weight, eps):
        self.weight = weight
        self.eps = eps


def _row_map(m, segments):
    rm = np.zeros(m, np.int64)
    for a, b, r in segments:
        rm[a:b] = r
    return rm


def test_rms_adaln_golden_h3_segments(golden):
    g = golden("rms_adaln")
    segs = [tuple(int(v) for v in s) for s in g["segments"]]
    # shift / scale arrive as the fp32 views split_adaln cuts; the op casts them like scale[row].to(bf16)
    proj = torch.zeros(g["shift_rows"].shape[0], 6 * g["shift_rows"].shape[1])
    d = g["shift_rows"].shape[1]
    proj[:, :d] = torch.from_numpy(g["shift_rows"])
    proj[:, d:2 * d] = torch.from_numpy(g["scale_rows"])
    proj = proj.cuda()
    shift, scale = proj[:, :d], proj[:, d:2 * d]          # strided fp32 views
    norm = _Norm(u2t(g["w_h3"]), float(g["eps_h3"]))
    out = h3b200.rms_adaln_segmented(u2t(g["x_h3"]), norm, shift, scale, segs)
    np.testing.assert_array_equal(t2u(out), g["out_h3"])


def test_rms_adaln_golden_comfy_per_sample(golden):
    g = golden("rms_adaln")
    out = h3b200.rms_adaln(u2t(g["x_cf"]), u2t(g["scale_cf"]), u2t(g["shift_cf"]), 1e-6)
    np.testing.assert_array_equal(t2u(out), g["out_cf"])


@pytest.mark.parametrize("m,d,rows,with_w", [(1000, 5376, 3, True), (777, 3072, 2, True), (513, 3072, 1, False),
                                             (300, 1000, 3, True), (64, 8192, 2, True), (5, 64, 1, True),
                                             (129, 2056, 4, False)])
def test_rms_adaln_segmented_vs_oracle(m, d, rows, with_w):
    gen = torch.Generator().manual_seed(m + d)
    x = randn_bf16((m, d), gen, std=1.7)
    x[min(3, m - 1)] = 0
    w = randn_bf16((d,), gen, std=0.05, mean=1.0)
    sc = randn_bf16((rows, d), gen, std=0.2)
    sh = randn_bf16((rows, d), gen, std=0.2)
    cuts = sorted(set(int(v) for v in torch.randint(1, max(2, m), (rows - 1,), generator=gen))) if m > 1 else []
    bounds = [0] + cuts + [m]
    segs = [(bounds[i], bounds[i + 1], (i * 7 + 1) % rows) for i in range(len(bounds) - 1)]
    out = h3b200.rms_adaln_segmented(x.cuda(), _Norm(w.cuda() if with_w else None, 1e-6), sh.cuda(), sc.cuda(), segs)
    ref = O.rms_adaln_rows(t2u(x), t2u(w) if with_w else None, t2u(sc), t2u(sh), _row_map(m, segs), 1e-6)
    np.testing.assert_array_equal(t2u(out), ref)


def test_rms_adaln_in_place_strided_rows_and_views():
    gen = torch.Generator().manual_seed(21)
    m, d = 333, 5376
    big = randn_bf16((m, 2 * d), gen).cuda()
    x = big[:, 512:512 + d]                               # strided token rows
    w = randn_bf16((d,), gen, std=0.05, mean=1.0).cuda()
    proj = randn_bf16((3, 6 * d), gen, std=0.2).cuda()
    shift, scale = proj[:, :d], proj[:, d:2 * d]          # split_adaln-style strided bf16 views
    segs = [(0, 100, 1), (100, 101, 2), (101, m, 0)]
    ref = O.rms_adaln_rows(t2u(x), t2u(w), t2u(scale), t2u(shift), _row_map(m, segs), 1e-5)
    before = t2u(big)
    out = h3b200.rms_adaln_segmented(x, _Norm(w, 1e-5), shift, scale, segs, out=x)
    assert out.data_ptr() == x.data_ptr()
    np.testing.assert_array_equal(t2u(x), ref)
    after = t2u(big)
    np.testing.assert_array_equal(after[:, :512], before[:, :512])          # untouched outside the view
    np.testing.assert_array_equal(after[:, 512 + d:], before[:, 512 + d:])


def test_rms_adaln_comfy_broadcast_forms():
    gen = torch.Generator().manual_seed(22)
    x = randn_bf16((3, 40, 1024), gen).cuda()
    xu = t2u(x).reshape(-1, 1024)
    one = randn_bf16((1024,), gen, std=0.1)
    out = h3b200.rms_adaln(x, one.cuda(), (one * 0.5).to(torch.bfloat16).cuda(), 1e-6)
    ref = O.rms_adaln_rows(xu, None, t2u(one)[None], t2u((one * 0.5).to(torch.bfloat16))[None], np.zeros(120, int))
    np.testing.assert_array_equal(t2u(out).reshape(-1, 1024), ref)
    per_tok = randn_bf16((3, 40, 1024), gen, std=0.1)     # one row per token
    shf = randn_bf16((1, 40, 1024), gen, std=0.1)         # broadcast over the batch: needs a row map
    out2 = h3b200.rms_adaln(x, per_tok.cuda(), shf.expand(3, 40, 1024).contiguous().cuda(), 1e-6)
    ref2 = O.rms_adaln_rows(xu, None, t2u(per_tok).reshape(-1, 1024),
                            t2u(shf.expand(3, 40, 1024).contiguous()).reshape(-1, 1024), np.arange(120))
    np.testing.assert_array_equal(t2u(out2).reshape(-1, 1024), ref2)
    sc3 = randn_bf16((1, 40, 1024), gen, std=0.1)
    out3 = h3b200.rms_adaln(x, sc3.cuda(), shf.cuda(), 1e-6)
    rm = np.tile(np.arange(40), 3)
    ref3 = O.rms_adaln_rows(xu, None, t2u(sc3).reshape(-1, 1024), t2u(shf).reshape(-1, 1024), rm)
    np.testing.assert_array_equal(t2u(out3).reshape(-1, 1024), ref3)


def test_rms_adaln_full_cfg3_size_single_row():
    gen = torch.Generator().manual_seed(4)
    m, d = 32760, 3072
    x = randn_bf16((m, d), gen)
    sc = randn_bf16((1, d), gen, std=0.1)
    sh = randn_bf16((1, d), gen, std=0.1)
    w = randn_bf16((d,), gen, std=0.02, mean=1.0)
    out = h3b200.rms_adaln_segmented(x.cuda(), _Norm(w.cuda(), 1e-6), sh.cuda(), sc.cuda(), [(0, m, 0)])
    ref = O.rms_adaln_rows(t2u(x), t2u(w), t2u(sc), t2u(sh), np.zeros(m, int), 1e-6)
    np.testing.assert_array_equal(t2u(out), ref)


def test_rms_adaln_rejects_bad_segments_and_shapes():
    x = torch.zeros(10, 64, dtype=torch.bfloat16, device="cuda")
    rows = torch.zeros(2, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="ordered partition"):
        h3b200.rms_adaln_segmented(x, None, rows, rows, [(0, 4, 0), (5, 10, 1)])
    with pytest.raises(ValueError, match="do not cover"):
        h3b200.rms_adaln_segmented(x, None, rows, rows, [(0, 4, 0)])
    with pytest.raises(ValueError, match="outside"):
        h3b200.rms_adaln_segmented(x, None, rows, rows, [(0, 10, 2)])
    bad = torch.zeros(3, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="broadcast"):
        h3b200.rms_adaln(x, bad, bad, 1e-6)
    with pytest.raises(ValueError, match="same shape"):
        h3b200.rms_adaln(x, bad, rows[:1], 1e-6)


@pytest.mark.parametrize("rot", [0, 96])
def test_norm_rope_segmented_modulation_vs_oracle(rot):
    gen = torch.Generator().manual_seed(31 + rot)
    m, h = 1500, 24
    q = randn_bf16((m, h, 128), gen)
    k = randn_bf16((m, h, 128), gen)
    wq = randn_bf16((h * 128,), gen, std=0.02, mean=1.0)
    wk = randn_bf16((h * 128,), gen, std=0.02, mean=1.0)
    sc = randn_bf16((3, h * 128), gen, std=0.1)
    sh = randn_bf16((3, h * 128), gen, std=0.1)
    segs = [(0, 200, 2), (200, 900, 0), (900, m, 1)]
    table = O.rope_grid_table((1, 30, 50))
    if rot:
        table = np.ascontiguousarray(table[:, :rot // 2])
    qo, ko = h3b200.adaln_rms_rope(q.cuda(), k.cuda(), torch.from_numpy(table).cuda(), wq.cuda(), wk.cuda(),
                                   sc.cuda(), sh.cuda(), 1e-6, "row", rot, segments=segs)
    rm = _row_map(m, segs)
    for x, w, o in ((q, wq, qo), (k, wk, ko)):
        hrow = O.rms_adaln_rows(t2u(x).reshape(m, -1), t2u(w), t2u(sc), t2u(sh), rm, 1e-6).reshape(m, h, 128)
        np.testing.assert_array_equal(t2u(o), O.rope_split_half(hrow, table, rot))


def test_fused_mlp_segmented_gates_vs_oracle():
    gen = torch.Generator().manual_seed(41)
    d, ffn, m = 3072, 12288, 700
    w1 = randn_bf16((ffn, d), gen, std=0.02)
    w2 = randn_bf16((d, ffn), gen, std=0.02)
    wt = h3b200.W8A8MLPWeights.from_float(w1.cuda(), w2.cuda())
    x = randn_bf16((m, d), gen)
    res = randn_bf16((m, d), gen)
    gates = randn_bf16((3, d), gen)
    segs = [(0, 250, 1), (250, 256, 2), (256, m, 0)]
    out = h3b200.fused_gated_mlp(res.cuda(), x.cuda(), wt.w1q, wt.s1, wt.w2q, wt.s2, gates.cuda(), segments=segs)
    got = t2u(out)
    xs, rs, gs = t2u(x), t2u(res), t2u(gates)
    w1q, s1, w2q, s2 = (t.cpu().numpy() for t in (wt.w1q, wt.s1, wt.w2q, wt.s2))
    for a, b, r in segs:
        np.testing.assert_array_equal(got[a:b], O.w8a8_gelu_mlp(xs[a:b], w1q, s1, w2q, s2, gs[r], rs[a:b]))
