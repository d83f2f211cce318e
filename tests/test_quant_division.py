"""The quantizer's division shortcut equals the reference's division (CPU).

The reference quantizes with q = clamp(rne(bf16(fp32(x / sb))), -128, 127)
(backends/eager/quantization.py:815-826, 857-875). The CUDA quantizer computes
t = fp32(x * fp32(1 / sb)) instead and falls back to the IEEE division only when
the low 16 bits of t lie within 8 of 0x8000 (a bf16 rounding midpoint). This test
replays that rule with numpy's IEEE fp32 arithmetic on every finite bf16 x against
a spread of bf16 scales; the full 2^31-pair sweep (all positive normal bf16
scales) is the same loop with a step of 1.
"""

import numpy as np
import pytest

WINDOW = 8  # must match kMidWin in x-minimaxh3_b200/csrc/quantize.cu


def bf16_round_bits(f32: np.ndarray) -> np.ndarray:
    u = f32.view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32)


def finish(t: np.ndarray) -> np.ndarray:
    b = (bf16_round_bits(t) << 16).view(np.float32)
    with np.errstate(all="ignore"):
        return np.clip(np.rint(b), -128, 127)


@pytest.mark.parametrize("step", [509])
def test_reciprocal_with_midpoint_fallback_matches_division(step):
    x = (np.arange(65536, dtype=np.uint32) << 16).view(np.float32)
    x = x[np.isfinite(x)]
    scales = (np.arange(0x0080, 0x7F80, step, dtype=np.uint32) << 16).view(np.float32)
    scales = np.concatenate([scales, np.array([1.17549435e-38, 1.0, 2.0 ** -20, 1.0 / 127], dtype=np.float32)])
    fallbacks = 0
    for sb in scales:
        sb = np.float32(sb)
        with np.errstate(all="ignore"):
            exact = (x / sb).astype(np.float32)
            t = (x * (np.float32(1.0) / sb)).astype(np.float32)
        lo = (t.view(np.uint32) & 0xFFFF).astype(np.int64)
        fb = np.abs(lo - 0x8000) <= WINDOW
        fallbacks += int(fb.sum())
        fast = np.where(fb, exact, t)
        np.testing.assert_array_equal(finish(fast), finish(exact), err_msg=f"scale {sb!r}")
    # the shortcut is what runs almost always
    assert fallbacks < 1e-3 * x.size * scales.size
