"""GPU parity: fused gated W8A8 tanh-GELU MLP (bit-exact against the oracle / reference)."""

import numpy as np
import pytest
import torch

import h3b200
import oracle as O
from gpu_util import np_, randn_bf16, t2u, u2t

pytestmark = pytest.mark.gpu


def test_mlp_golden_bit_exact(golden):
    g = golden("mlp_small")
    out = h3b200.fused_gated_mlp(u2t(g["residual"]), u2t(g["x"]), torch.from_numpy(g["w1q"]).cuda(),
                                 torch.from_numpy(g["s1"]).cuda(), torch.from_numpy(g["w2q"]).cuda(),
                                 torch.from_numpy(g["s2"]).cuda(), u2t(g["gate"]))
    np.testing.assert_array_equal(t2u(out), g["out"])


def _weights(d, ffn, seed):
    gen = torch.Generator().manual_seed(seed)
    w1 = randn_bf16((ffn, d), gen, std=0.02)
    w2 = randn_bf16((d, ffn), gen, std=0.02)
    return gen, h3b200.W8A8MLPWeights.from_float(w1.cuda(), w2.cuda())


def _oracle_rows(x, res, gate, wt, rows):
    return O.w8a8_gelu_mlp(t2u(x)[rows], np_(wt.w1q), np_(wt.s1), np_(wt.w2q), np_(wt.s2), t2u(gate),
                           t2u(res)[rows])


def test_mlp_cfg1_dims_vs_oracle():
    gen, wt = _weights(3072, 12288, 2)
    x = randn_bf16((300, 3072), gen)
    gate = randn_bf16((3072,), gen)
    res = randn_bf16((300, 3072), gen)
    out = h3b200.fused_gated_mlp(res.cuda(), x.cuda(), wt.w1q, wt.s1, wt.w2q, wt.s2, gate.cuda())
    np.testing.assert_array_equal(t2u(out), _oracle_rows(x, res, gate, wt, np.arange(300)))


def test_mlp_inplace_residual_and_strided_hidden():
    gen, wt = _weights(512, 2048, 5)
    xbig = randn_bf16((77, 1024), gen).cuda()
    x = xbig[:, 256:768]                                  # strided rows
    gate = randn_bf16((512,), gen).cuda()
    res = randn_bf16((77, 512), gen).cuda()
    expect = _oracle_rows(x, res, gate, wt, np.arange(77))
    out = h3b200.fused_gated_mlp(res, x, wt.w1q, wt.s1, wt.w2q, wt.s2, gate, out=res)
    assert out.data_ptr() == res.data_ptr()
    np.testing.assert_array_equal(t2u(res), expect)


def test_mlp_cfg1_full_size_sampled_rows():
    """Config 1 at full size (M=32760): per-token math, so sampled rows are compared bit for bit."""
    gen, wt = _weights(3072, 12288, 2)
    x = randn_bf16((32760, 3072), gen)
    gate = randn_bf16((3072,), gen)
    res = randn_bf16((32760, 3072), gen)
    out = h3b200.fused_gated_mlp(res.cuda(), x.cuda(), wt.w1q, wt.s1, wt.w2q, wt.s2, gate.cuda())
    rows = np.sort(np.random.default_rng(1).choice(32760, 24, replace=False))
    rows = np.concatenate([[0, 32759], rows])
    np.testing.assert_array_equal(t2u(out)[rows], _oracle_rows(x, res, gate, wt, rows))
    assert h3b200.device_status(0) == 0


def test_mlp_repeat_is_deterministic():
    gen, wt = _weights(1024, 4096, 8)
    x = randn_bf16((500, 1024), gen).cuda()
    gate = randn_bf16((1024,), gen).cuda()
    res = randn_bf16((500, 1024), gen).cuda()
    a = h3b200.fused_gated_mlp(res, x, wt.w1q, wt.s1, wt.w2q, wt.s2, gate)
    b = h3b200.fused_gated_mlp(res, x, wt.w1q, wt.s1, wt.w2q, wt.s2, gate)
    assert torch.equal(a, b)


def test_mlp_rejects_bad_shapes():
    _, wt = _weights(256, 1024, 1)
    x = torch.zeros(4, 256, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="gate"):
        h3b200.fused_gated_mlp(x, x, wt.w1q, wt.s1, wt.w2q, wt.s2, torch.zeros(3, dtype=torch.bfloat16, device="cuda"))
    with pytest.raises(NotImplementedError):
        h3b200.fused_gated_mlp(x, x, wt.w1q, wt.s1, wt.w2q, wt.s2, x[0], act="swiglu")


def test_mlp_host_pipeline_matches_device_call():
    """Host-buffer entry point: chunked, copy-overlapped, bit-identical to one device call."""
    gen, wt = _weights(512, 2048, 9)
    m = 1000                                               # 3 full chunks of 300 + a ragged one
    x = randn_bf16((m, 512), gen).pin_memory()
    res = randn_bf16((m, 512), gen).pin_memory()
    gate = randn_bf16((512,), gen).cuda()
    expect = h3b200.fused_gated_mlp(res.cuda(), x.cuda(), wt.w1q, wt.s1, wt.w2q, wt.s2, gate)
    out = h3b200.fused_gated_mlp_host(res, x, wt.w1q, wt.s1, wt.w2q, wt.s2, gate, chunk_tokens=300)
    np.testing.assert_array_equal(t2u(out), t2u(expect))
    # a second call reuses the staging slots; in place on the residual buffer
    res2 = res.clone().pin_memory()
    h3b200.fused_gated_mlp_host(res2, x, wt.w1q, wt.s1, wt.w2q, wt.s2, gate, out=res2, chunk_tokens=300)
    np.testing.assert_array_equal(t2u(res2), t2u(expect))
