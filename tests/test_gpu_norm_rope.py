"""GPU parity: fused AdaLN-modulate + RMSNorm + split-half RoPE on Q/K."""

import numpy as np
import pytest
import torch

import h3b200
import oracle as O
from gpu_util import np_, randn_bf16, t2u, u2t

pytestmark = pytest.mark.gpu


def _close_to_reference(mine, ref):
    a, b = O.bf16_to_f32(mine), O.bf16_to_f32(ref)
    rel = np.linalg.norm((a - b).astype(np.float64)) / np.linalg.norm(b.astype(np.float64))
    assert rel <= 1e-2                          # north-star tolerance for bf16 outputs
    assert float(np.abs(a - b).max()) <= 2e-2
    assert (mine != ref).mean() <= 1e-4        # rare last-bit flips from the reference's fp32 sum order


def test_norm_rope_golden_row_span(golden):
    g = golden("norm_rope")
    q, k = u2t(g["q"]), u2t(g["k"])
    qo, ko = h3b200.adaln_rms_rope(q, k, torch.from_numpy(g["table"]).cuda(), u2t(g["wq"]), u2t(g["wk"]),
                                   u2t(g["scale"]), u2t(g["shift"]), 1e-6, "row")
    _close_to_reference(t2u(qo), g["q_out"])
    _close_to_reference(t2u(ko), g["k_out"])
    oq, ok = O.adaln_rms_rope(g["q"], g["k"], g["table"], g["wq"], g["wk"], g["scale"], g["shift"], 1e-6, "row")
    np.testing.assert_array_equal(t2u(qo), oq)
    np.testing.assert_array_equal(t2u(ko), ok)


def test_norm_rope_golden_head_span_full_and_partial(golden):
    g = golden("norm_rope")
    tab = torch.from_numpy(g["table"]).cuda()
    qh, kh = h3b200.rms_rope_split_half(u2t(g["q"]), u2t(g["k"]), tab, u2t(g["wq_head"]), u2t(g["wk_head"]), 1e-6, 0)
    _close_to_reference(t2u(qh), g["q_head"])
    _close_to_reference(t2u(kh), g["k_head"])
    qp, kp = h3b200.rms_rope_split_half(u2t(g["q"]), u2t(g["k"]), tab[:, :48].contiguous(), u2t(g["wq_head"]),
                                        u2t(g["wk_head"]), 1e-6, 96)
    _close_to_reference(t2u(qp), g["q_partial96"])
    _close_to_reference(t2u(kp), g["k_partial96"])
    oq, ok = O.rms_rope_split_half(g["q"], g["k"], g["table"][:, :48], g["wq_head"], g["wk_head"], 1e-6, 96)
    np.testing.assert_array_equal(t2u(qp), oq)
    np.testing.assert_array_equal(t2u(kp), ok)


def _cfg3_inputs(m, grid, seed=4):
    gen = torch.Generator().manual_seed(seed)
    q = randn_bf16((m, 24, 128), gen)
    k = randn_bf16((m, 24, 128), gen)
    shift = randn_bf16((3072,), gen, std=0.1)
    scale = randn_bf16((3072,), gen, std=0.1)
    wq = randn_bf16((3072,), gen, std=0.02, mean=1.0)
    wk = randn_bf16((3072,), gen, std=0.02, mean=1.0)
    table = O.rope_grid_table(grid)
    return q, k, shift, scale, wq, wk, table


def test_norm_rope_cfg3_full_size_exact_vs_oracle():
    """Config 3: M=32760 tokens on the 21x39x40 grid, 24x128 heads, 44/42/42 split, base 10000."""
    q, k, shift, scale, wq, wk, table = _cfg3_inputs(32760, (21, 39, 40))
    qo, ko = h3b200.adaln_rms_rope(q.cuda(), k.cuda(), torch.from_numpy(table).cuda(), wq.cuda(), wk.cuda(),
                                   scale.cuda(), shift.cuda())
    oq, ok = O.adaln_rms_rope(t2u(q), t2u(k), table, t2u(wq), t2u(wk), t2u(scale), t2u(shift))
    np.testing.assert_array_equal(t2u(qo), oq)
    np.testing.assert_array_equal(t2u(ko), ok)


def test_norm_rope_inplace_on_packed_qkv():
    """Q and K as strided views of a packed [M, 3, H, D] projection, updated in place."""
    gen = torch.Generator().manual_seed(12)
    m = 517
    qkv = randn_bf16((m, 3, 24, 128), gen).cuda()
    table = O.rope_grid_table((11, 47, 1))
    wq = randn_bf16((128,), gen, std=0.02, mean=1.0).cuda()
    wk = randn_bf16((128,), gen, std=0.02, mean=1.0).cuda()
    q0, k0, v0 = t2u(qkv[:, 0]), t2u(qkv[:, 1]), t2u(qkv[:, 2])
    h3b200.rms_rope_split_half_(qkv[:, 0], qkv[:, 1], torch.from_numpy(table).cuda(), wq, wk)
    oq, ok = O.rms_rope_split_half(q0, k0, table, t2u(wq), t2u(wk))
    np.testing.assert_array_equal(t2u(qkv[:, 0]), oq)
    np.testing.assert_array_equal(t2u(qkv[:, 1]), ok)
    np.testing.assert_array_equal(t2u(qkv[:, 2]), v0)     # V untouched


def test_norm_rope_head_span_with_modulation_and_odd_heads():
    gen = torch.Generator().manual_seed(13)
    m, h = 200, 5
    q = randn_bf16((m, h, 128), gen)
    k = randn_bf16((m, h, 128), gen)
    wq = randn_bf16((128,), gen, std=0.02, mean=1.0)
    sc = randn_bf16((h * 128,), gen, std=0.1)
    sh = randn_bf16((h * 128,), gen, std=0.1)
    table = O.rope_grid_table((2, 10, 10), dims=(16, 24, 24))
    qo, ko = h3b200.adaln_rms_rope(q.cuda(), k.cuda(), torch.from_numpy(table).cuda(), wq.cuda(), None, sc.cuda(),
                                   sh.cuda(), 1e-6, "head", 64)
    oq, ok = O.adaln_rms_rope(t2u(q), t2u(k), table, t2u(wq), t2u(wq), t2u(sc), t2u(sh), 1e-6, "head", 64)
    np.testing.assert_array_equal(t2u(qo), oq)
    np.testing.assert_array_equal(t2u(ko), ok)


def test_norm_rope_contract():
    q = torch.zeros(4, 2, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(NotImplementedError):
        h3b200.adaln_rms_rope(q, q, torch.zeros(4, 32, 2, 2, device="cuda"), torch.ones(64, device="cuda"), None,
                              None, None, 1e-6, "head")
