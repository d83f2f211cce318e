"""Host-side contract of the Python operator surface (CPU, no kernel launches)."""

import pytest
import torch

import h3b200


def test_cpu_tensors_are_rejected_no_fallback():
    x = torch.zeros(4, 16, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA tensors only"):
        h3b200.quantize_int8_rowwise(x)
    w = torch.zeros(8, 16, dtype=torch.int8)
    with pytest.raises(ValueError, match="CUDA tensors only"):
        h3b200.int8_linear(x, w, torch.ones(8))
    with pytest.raises(ValueError, match="CUDA tensors only"):
        h3b200.mm_int8(w, w.t())


def test_input_act_codes_match_reference():
    # backends/cuda/input_act_codes.h:13 -- 0 none, 1 gelu_tanh
    assert h3b200.input_act_code(None) == 0
    assert h3b200.input_act_code("none") == 0
    assert h3b200.input_act_code("gelu_tanh") == 1
    with pytest.raises(ValueError, match="unsupported input_act"):
        h3b200.input_act_code("relu")


def test_stochastic_rounding_oracle_properties():
    """The stochastic rounding restatement: q is floor(t) or floor(t) + 1 of the bf16
    quotient t, unbiased on average, a function of (element index, seed)."""
    import numpy as np

    import oracle as O

    rng = np.random.default_rng(0)
    x = O.f32_to_bf16(rng.standard_normal((64, 1024)).astype(np.float32))
    q1, s1 = O.quantize_int8_rowwise_stochastic(x, 7)
    q1b, _ = O.quantize_int8_rowwise_stochastic(x, 7)
    q2, _ = O.quantize_int8_rowwise_stochastic(x, 8)
    qn, sn = O.quantize_int8_rowwise(x)
    np.testing.assert_array_equal(q1, q1b)
    np.testing.assert_array_equal(s1, sn)            # same row scale as the deterministic quantizer
    assert (q1 != q2).mean() > 0.2
    sb = O.bf16_to_f32(O.f32_to_bf16(s1))
    t = O.bf16_to_f32(O.f32_to_bf16((O.bf16_to_f32(x) / sb).astype(np.float32)))
    d = q1.astype(np.float32) - np.floor(t)
    assert set(np.unique(d)) <= {0.0, 1.0}
    # E[floor(t + u)] = t for u ~ U[0, 1); the sum is rounded to bf16 before the floor (the
    # reference's order), which biases large |t| upward, so check where bf16 resolves the sum
    small = np.abs(t) < 1.0
    assert abs(float((q1[small] - t[small]).mean())) < 0.02
    # the noise is the reference kernel's: a 24-bit hash fraction, rounded to bf16
    u = O.stochastic_noise_bf16(np.arange(100000, dtype=np.uint64), 12345)
    assert u.min() >= 0.0 and u.max() <= 1.0 and abs(float(u.mean()) - 0.5) < 0.01


def test_rope_table_builder_matches_oracle():
    import numpy as np

    import oracle as O
    from h3b200.rope import rope_grid_table

    for grid, sl in (((21, 39, 40), None), ((45, 52, 84), (1000, 1700)), ((2, 5, 8), None)):
        t = rope_grid_table(grid, token_slice=sl, device="cpu").numpy()
        o = O.rope_grid_table(grid, token_slice=sl)
        np.testing.assert_array_equal(t, o)


def test_w4a8_weight_quantizer_matches_reference_golden_and_oracle(golden):
    """Offline W4A8 weight preparation (torch) vs the reference's quantize_w4a8_int8_weight output."""
    import numpy as np
    import torch

    import oracle as O
    from h3b200.weights import quantize_w4a8_weight

    def to_t(u):
        return torch.from_numpy(np.ascontiguousarray(u).view(np.int16)).view(torch.bfloat16)

    def to_u(t):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)

    g = golden("w4a8_small")
    q, s_rel, s_ch, corr = quantize_w4a8_weight(to_t(g["w_bf16"]), 128, 256)
    np.testing.assert_array_equal(q.numpy(), g["qdata"])
    np.testing.assert_array_equal(s_rel.numpy(), g["s_rel"])
    np.testing.assert_array_equal(s_ch.numpy(), g["s_channel"])
    np.testing.assert_array_equal(to_u(corr), g["correction"])
    w = (torch.randn(384, 1024, generator=torch.Generator().manual_seed(3)) * 0.02).to(torch.bfloat16)
    got = quantize_w4a8_weight(w, 128, 256)
    want = O.w4a8_quantize_weight(to_u(w), 128, 256)
    for a, b in zip(got[:3], want[:3]):
        np.testing.assert_array_equal(a.numpy(), b)
    np.testing.assert_array_equal(to_u(got[3]), want[3])
