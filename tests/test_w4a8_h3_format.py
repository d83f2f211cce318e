"""CPU checks of the H3 release W4A8 format (group 16, fp8-e4m3 s_rel, 16-level codebook).

The oracle's decode, linear and W4 SwiGLU MLP, and h3b200's torch weight preparation,
against fixtures made by running the reference (``tests/golden/make_golden.py``,
fixture ``w4a8_h3``): ``quantize_w4a8_int8_weight`` with its release defaults and other
branches, ``_dequant_int4_grouped_to_int8``, ``comfy_kitchen.w4a8_int8_linear`` and the
reference's own W4A8 MLP driver ``_chunked_module_gated_mlp``.
"""

import hashlib

import numpy as np
import pytest
import torch

import oracle as O
from h3b200.weights import W4A8_FIXED_CODEBOOK, quantize_w4a8_int8_weight, regular_hadamard

DECODE_CASES = (("g4_e4m3_cb", 4, torch.float8_e4m3fn, True), ("g8_e4m3_cb", 8, torch.float8_e4m3fn, True),
                ("g32_f32_cb", 32, torch.float32, True), ("g16_f32_uni", 16, torch.float32, False),
                ("g8_e4m3_uni", 8, torch.float8_e4m3fn, False))


@pytest.fixture(scope="module")
def fx():
    from conftest import load_golden

    return load_golden("w4a8_h3")


def bf(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


def bits(t):
    return t.contiguous().view(torch.uint8).numpy() if t.dtype == torch.float8_e4m3fn else t.numpy()


def test_e4m3_widening_all_patterns():
    allb = np.arange(256, dtype=np.uint8)
    ref = torch.from_numpy(allb).view(torch.float8_e4m3fn).float().numpy()
    got = O.e4m3_to_f32(allb)
    nan = np.isnan(ref)
    np.testing.assert_array_equal(np.isnan(got), nan)
    np.testing.assert_array_equal(got[~nan], ref[~nan])
    assert nan.sum() == 2


def test_oracle_decode_vs_reference(fx):
    for tag in ("a", "b"):
        np.testing.assert_array_equal(
            O.decode_int4_grouped_to_int8(fx[f"q_{tag}"], fx[f"s_rel_{tag}"], 16, fx[f"codebook_{tag}"]),
            fx[f"grid_{tag}"])
    for tag, gsz, _, use_cb in DECODE_CASES:
        cb = fx[f"codebook_{tag}"] if use_cb else None
        np.testing.assert_array_equal(O.decode_int4_grouped_to_int8(fx[f"q_{tag}"], fx[f"s_rel_{tag}"], gsz, cb),
                                      fx[f"grid_{tag}"])


def test_oracle_linear_and_mlp_vs_reference(fx):
    y = O.w4a8_symmetric_linear(fx["x_a"], fx["q_a"], fx["s_rel_a"], fx["s_ch_a"], fx["codebook_a"], fx["b_a"], 16)
    np.testing.assert_array_equal(y, fx["y_a"])
    segs = fx["mlp_segments"]
    row_map = np.concatenate([np.full(b - a, r) for a, b, r in segs])
    w4 = {"q1": fx["mlp_q1"], "s_rel1": fx["mlp_s_rel1"], "s_ch1": fx["mlp_s_ch1"], "codebook1": fx["mlp_codebook1"],
          "b1": fx["mlp_b1"], "q2": fx["mlp_q2"], "s_rel2": fx["mlp_s_rel2"], "s_ch2": fx["mlp_s_ch2"],
          "codebook2": fx["mlp_codebook2"], "b2": fx["mlp_b2"], "group_size": 16}
    out, inter = O.w4a8_swiglu_mlp(fx["mlp_x"], w4, fx["mlp_gate"], row_map, fx["mlp_residual"], True)
    np.testing.assert_array_equal(inter["raw"], fx["mlp_raw"])
    np.testing.assert_array_equal(out, fx["mlp_out"])


def test_weight_prep_release_format_vs_reference(fx):
    """Release defaults: Gaussian weight (fixed codebook) and heavy-tailed weight (fitted
    codebook, sampled kurtosis and fit), bit for bit."""
    for tag in ("a", "b"):
        q, s_rel, s_ch, corr, cb = quantize_w4a8_int8_weight(bf(fx[f"w_{tag}"]))
        assert corr is None and s_rel.dtype == torch.float8_e4m3fn
        np.testing.assert_array_equal(q.numpy(), fx[f"q_{tag}"])
        np.testing.assert_array_equal(bits(s_rel), fx[f"s_rel_{tag}"])
        np.testing.assert_array_equal(s_ch.numpy(), fx[f"s_ch_{tag}"])
        np.testing.assert_array_equal(cb.numpy(), fx[f"codebook_{tag}"])
    assert np.array_equal(fx["codebook_a"], np.array(W4A8_FIXED_CODEBOOK, np.float32))
    assert not np.array_equal(fx["codebook_b"], np.array(W4A8_FIXED_CODEBOOK, np.float32))
    for i in (1, 2):
        q, s_rel, _, _, cb = quantize_w4a8_int8_weight(bf(fx[f"mlp_w{i}"]))
        np.testing.assert_array_equal(q.numpy(), fx[f"mlp_q{i}"])
        np.testing.assert_array_equal(bits(s_rel), fx[f"mlp_s_rel{i}"])


@pytest.mark.parametrize("tag,gsz,sdt,use_cb", DECODE_CASES)
def test_weight_prep_other_branches_vs_reference(fx, tag, gsz, sdt, use_cb):
    q, s_rel, s_ch, corr, cb = quantize_w4a8_int8_weight(bf(fx["w_c"]), gsz, 256, True, sdt, use_cb)
    assert corr is None and (cb is not None) == use_cb
    np.testing.assert_array_equal(q.numpy(), fx[f"q_{tag}"])
    np.testing.assert_array_equal(bits(s_rel), fx[f"s_rel_{tag}"])
    np.testing.assert_array_equal(s_ch.numpy(), fx[f"s_ch_{tag}"])
    if use_cb:
        np.testing.assert_array_equal(cb.numpy(), fx[f"codebook_{tag}"])


def test_weight_prep_strided_codebook_rows_and_chunks(fx):
    """[640, 8192] heavy-tailed weight, regenerated from its seed: the codebook is chosen from
    strided rows and the rows are prepared in two chunks; digests of the reference's outputs."""

    def digest(t):
        return np.frombuffer(hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).digest(), np.uint8)

    gen = torch.Generator().manual_seed(int(fx["big_seed"]))
    z = torch.randn(640, 8192, generator=gen)
    h = regular_hadamard(256).float()
    w = ((z * z * z * 0.01).reshape(640, 32, 256) @ h).reshape(640, 8192).to(torch.bfloat16)
    if not np.array_equal(digest(w), fx["big_w_sha"]):
        pytest.fail("torch's CPU generator no longer reproduces the fixture's weight; regenerate the fixture")
    q, s_rel, s_ch, _, cb = quantize_w4a8_int8_weight(w)
    np.testing.assert_array_equal(cb.numpy(), fx["big_codebook"])
    np.testing.assert_array_equal(s_ch.numpy(), fx["big_s_ch"])
    np.testing.assert_array_equal(digest(s_rel), fx["big_s_rel_sha"])
    np.testing.assert_array_equal(digest(q), fx["big_q_sha"])


def test_weight_prep_rejects_bad_shapes():
    with pytest.raises(ValueError):
        quantize_w4a8_int8_weight(torch.zeros(4, 500, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        quantize_w4a8_int8_weight(torch.zeros(4, 512, dtype=torch.bfloat16), group_size=12)
    with pytest.raises(ValueError):
        quantize_w4a8_int8_weight(torch.zeros(4, 512, dtype=torch.bfloat16), scale_dtype=torch.float16)
