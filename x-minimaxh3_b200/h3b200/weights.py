"""Weight preparation for the quantized MLP (offline, on the GPU).

W8A8 weights are quantized per output channel with the same row quantizer the
activations use, as the reference does (``quantize_int8_rowwise(W)``,
backends/eager/quantization.py:857-875: fp32 scale = absmax / 127).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .ops import quantize_int8_rowwise


def quantize_int8_weight(w: torch.Tensor):
    """bf16 [N, K] -> (int8 [N, K], fp32 per-channel scale [N])."""
    q, s = quantize_int8_rowwise(w.to(torch.bfloat16).contiguous())
    return q, s.reshape(-1)


@dataclass
class W8A8MLPWeights:
    """Resident quantized weights of one gated MLP: fc1 [ffn, d], fc2 [d, ffn]."""

    w1q: torch.Tensor
    s1: torch.Tensor
    w2q: torch.Tensor
    s2: torch.Tensor

    @classmethod
    def from_float(cls, w1: torch.Tensor, w2: torch.Tensor) -> "W8A8MLPWeights":
        w1q, s1 = quantize_int8_weight(w1)
        w2q, s2 = quantize_int8_weight(w2)
        return cls(w1q, s1, w2q, s2)

    @property
    def d(self) -> int:
        return self.w1q.shape[1]

    @property
    def ffn(self) -> int:
        return self.w1q.shape[0]
