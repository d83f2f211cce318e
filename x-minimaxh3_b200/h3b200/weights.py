"""Weight preparation for the quantized MLP (offline).

W8A8 weights are quantized per output channel with the same row quantizer the
activations use, as the reference does (``quantize_int8_rowwise(W)``,
backends/eager/quantization.py:857-875: fp32 scale = absmax / 127).

W4A8 weights use the reference's asymmetric grouped format
(``quantize_w4a8_int8_weight(symmetric=False, codebook=False,
scale_dtype=float32)``, backends/eager/w4a8_int8.py:315-341 -> :122-209):
ConvRot-256 rotation of W, per-group min/max to uint4, fp32 ``s_rel`` and
``s_channel``, bf16 ``correction``. This is offline preparation written with
torch tensor operations (it runs once per weight, on any device).

ConvRot INT8 weights (the H3 SwiGLU MLP) are rotated along their input dimension
by the regular Hadamard-256 and then quantized per output channel
(``quantize_int8_convrot_weight``, backends/eager/quantization.py:898-906).
"""

from __future__ import annotations

import math
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


def regular_hadamard(size: int = 256, device=None) -> torch.Tensor:
    """Normalised regular Hadamard matrix H4^(x)n / sqrt(size), float64 (tensor/int8_utils.py:11-38)."""
    if size < 4 or size & (size - 1) or (size.bit_length() - 1) % 2:
        raise ValueError(f"regular Hadamard size must be a power of 4, got {size}")
    h4 = torch.tensor([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=torch.float64,
                      device=device)
    h = h4
    while h.shape[0] < size:
        h = torch.kron(h, h4)
    return h / math.sqrt(size)


def quantize_w4a8_weight(w: torch.Tensor, group_size: int = 128, convrot_groupsize: int = 256):
    """bf16 W [N, K] -> (qdata int8 [N, K/2], s_rel fp32 [N, K/g], s_channel fp32 [N], correction bf16 [K/g, N]).

    Steps of eager/w4a8_int8.py:122-209 (asymmetric branch :175-186, scales
    :188-191, packing :200-202, even column in the low nibble) after the offline
    rotation ``W @ H^T`` per 256-group (tensor/int8_utils.py:41-55), whose
    result is rounded to bf16 as the reference's bf16 matmul is."""
    n, k = w.shape
    if k % convrot_groupsize or k % group_size:
        raise ValueError(f"K={k} must be divisible by convrot_groupsize and group_size")
    hm = regular_hadamard(convrot_groupsize, w.device)
    wr = (w.to(torch.float64).reshape(n, k // convrot_groupsize, convrot_groupsize) @ hm.T).reshape(n, k)
    wr = wr.to(torch.float32).to(torch.bfloat16).to(torch.float32)
    g = wr.reshape(n, k // group_size, group_size)
    mn = g.amin(-1, keepdim=True)
    gsc = torch.clamp_min((g.amax(-1, keepdim=True) - mn) / 15.0, 1e-8)
    u = torch.clamp(torch.round((g - mn) / gsc), 0, 15).to(torch.int32)
    shifted = (u - 8).to(torch.float32) * gsc
    corr = (8.0 * gsc + mn).squeeze(-1).t().contiguous().to(torch.bfloat16)
    s_ch = torch.clamp_min(shifted.abs().amax(dim=(1, 2)) / 127.0, 1e-8)
    s_rel = (gsc.squeeze(-1) / s_ch[:, None]).contiguous()
    u = u.reshape(n, k)
    packed = ((u[:, 0::2] & 0xF) | ((u[:, 1::2] & 0xF) << 4)).to(torch.uint8).view(torch.int8).contiguous()
    return packed, s_rel, s_ch.contiguous(), corr


@dataclass
class W4A8MLPWeights:
    """One gated MLP in the reference's W4A8 format: fc1 [ffn, d], fc2 [d, ffn] (int4 at rest)."""

    q1: torch.Tensor
    s_rel1: torch.Tensor
    s_ch1: torch.Tensor
    corr1: torch.Tensor
    q2: torch.Tensor
    s_rel2: torch.Tensor
    s_ch2: torch.Tensor
    corr2: torch.Tensor
    group_size: int = 128

    @classmethod
    def from_float(cls, w1: torch.Tensor, w2: torch.Tensor, group_size: int = 128) -> "W4A8MLPWeights":
        return cls(*quantize_w4a8_weight(w1, group_size), *quantize_w4a8_weight(w2, group_size), group_size)

    def to(self, device) -> "W4A8MLPWeights":
        return W4A8MLPWeights(self.q1.to(device), self.s_rel1.to(device), self.s_ch1.to(device),
                              self.corr1.to(device), self.q2.to(device), self.s_rel2.to(device),
                              self.s_ch2.to(device), self.corr2.to(device), self.group_size)

    @property
    def d(self) -> int:
        return self.q1.shape[1] * 2

    @property
    def ffn(self) -> int:
        return self.q1.shape[0]


def rotate_weight(w: torch.Tensor, group_size: int = 256) -> torch.Tensor:
    """Offline ConvRot rotation ``W @ H^T`` per input group (tensor/int8_utils.py:41-55),
    summed exactly and rounded to bf16 as the reference's bf16 matmul result is stored."""
    n, k = w.shape
    if k % group_size:
        raise ValueError(f"in_features {k} not divisible by group_size {group_size}")
    hm = regular_hadamard(group_size, w.device)
    wr = (w.to(torch.float64).reshape(n, k // group_size, group_size) @ hm.T).reshape(n, k)
    return wr.to(torch.float32).to(torch.bfloat16)


def quantize_int8_convrot_weight(w: torch.Tensor, group_size: int = 256):
    """bf16 [N, K] -> (int8 [N, K], fp32 per-channel scale [N]) of the rotated weight
    (``quantize_int8_convrot_weight`` eager/quantization.py:898-906)."""
    return quantize_int8_weight(rotate_weight(w, group_size))


@dataclass
class SwiGLUMLPWeights:
    """One H3 SwiGLU MLP: fc1 [2 ffn, d] ([gate | up] output rows), fc2 [d, ffn], INT8 with
    per-channel fp32 scales and optional bf16 biases. fc2 is always ConvRot-rotated (the
    reference's fused fc2 requires it, fused_mlp.py:306-312); fc1 is when ``fc1_convrot``."""

    w1q: torch.Tensor
    s1: torch.Tensor
    w2q: torch.Tensor
    s2: torch.Tensor
    b1: torch.Tensor | None = None
    b2: torch.Tensor | None = None
    fc1_convrot: bool = True

    @classmethod
    def from_float(cls, w1: torch.Tensor, w2: torch.Tensor, b1: torch.Tensor | None = None,
                   b2: torch.Tensor | None = None, fc1_convrot: bool = True) -> "SwiGLUMLPWeights":
        w1q, s1 = quantize_int8_convrot_weight(w1) if fc1_convrot else quantize_int8_weight(w1)
        w2q, s2 = quantize_int8_convrot_weight(w2)
        cast = (lambda b: None if b is None else b.to(torch.bfloat16).contiguous())
        return cls(w1q, s1, w2q, s2, cast(b1), cast(b2), fc1_convrot)

    @property
    def d(self) -> int:
        return self.w1q.shape[1]

    @property
    def ffn(self) -> int:
        return self.w1q.shape[0] // 2
