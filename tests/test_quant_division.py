"""The quantizer's reciprocal product equals the reference's division (CPU).

The reference quantizes with q = clamp(rne(bf16(fp32(x / sb))), -128, 127)
(backends/eager/quantization.py:815-826, 857-875). The CUDA quantizers compute
t = fp32(x * fp32(1 / sb)) instead, with no fallback: for bf16 x and bf16 sb the
exact quotient is a ratio of two integer mantissas of at most 8 bits, which lies
more than 128 fp32 ulp away from every bf16 rounding midpoint, while t is within
2 ulp of it. This test replays the rule with numpy's IEEE fp32 arithmetic on every
finite bf16 x against a spread of bf16 divisors; the full sweep (all 32,512
positive normal bf16 divisors, 2.1e9 pairs, no mismatch) is the same loop with a
step of 1.
"""

import numpy as np
import pytest


def bf16_round_bits(f32: np.ndarray) -> np.ndarray:
    u = f32.view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32)


def finish(t: np.ndarray) -> np.ndarray:
    b = (bf16_round_bits(t) << 16).view(np.float32)
    with np.errstate(all="ignore"):
        return np.clip(np.rint(b), -128, 127)


@pytest.mark.parametrize("step", [509])
def test_reciprocal_product_matches_division(step):
    x = (np.arange(65536, dtype=np.uint32) << 16).view(np.float32)
    x = x[np.isfinite(x)]
    scales = (np.arange(0x0080, 0x7F80, step, dtype=np.uint32) << 16).view(np.float32)
    # the smallest divisor the quantizers can see (scale >= 1e-30), the zero-absmax
    # divisor, and scales of typical activations
    extra = [np.float32(1e-30), 1.17549435e-38, 1.0, 2.0 ** -20, 1.0 / 127, 3.0 / 127, 0.0171, 1.7e3]
    scales = np.concatenate([scales, np.array(extra, dtype=np.float32)])
    sbs = (bf16_round_bits(scales.astype(np.float32)) << 16).view(np.float32)
    for sb in sbs:
        sb = np.float32(sb)
        with np.errstate(all="ignore"):
            exact = (x / sb).astype(np.float32)
            t = (x * (np.float32(1.0) / sb)).astype(np.float32)
        np.testing.assert_array_equal(finish(t), finish(exact), err_msg=f"divisor {sb!r}")


def test_midpoint_distance_argument():
    """The number-theoretic fact behind the shortcut, checked directly: for integer
    mantissas a, b in [1, 255], a / b is never within 128 fp32 ulp of a bf16 midpoint."""
    a = np.arange(1, 256, dtype=np.float64)[:, None]
    b = np.arange(1, 256, dtype=np.float64)[None, :]
    q = a / b
    e = np.floor(np.log2(q))                      # binade of the quotient
    ulp_bf16 = 2.0 ** (e - 7)
    mid = (np.floor(q / ulp_bf16) + 0.5) * ulp_bf16
    dist = np.abs(q - mid) / 2.0 ** (e - 23)      # in fp32 ulp of that binade
    assert dist.min() > 128
