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

The H3 release W4A8 format (``quantize_w4a8_int8_weight`` with its defaults:
group 16, symmetric, fp8-e4m3 ``s_rel``, a 16-level Lloyd-Max codebook; the
``W4A8QuantSpec`` of h3serve/native_engine/model/quantization.py:153-187) is
prepared by :func:`quantize_w4a8_int8_weight`, which covers every branch of the
reference function (asymmetric, symmetric uniform, symmetric codebook) and
returns its five-tuple.
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


# Lloyd-Max levels of a group-normalised Gaussian (16 levels in [-1, 1]): the fixed
# codebook of the H3 release format, backends/eager/w4a8_int8.py:11-16. A shared data
# table (weights quantized against it must decode with the same values).
W4A8_FIXED_CODEBOOK = (
    -0.980602, -0.794529, -0.638165, -0.500986, -0.377321, -0.263187, -0.155210, -0.050720,
    0.052541, 0.156985, 0.265284, 0.379533, 0.502636, 0.638953, 0.794876, 0.980671,
)
_KURTOSIS_GATE = -0.1          # excess kurtosis above this: fit a codebook instead (:19)
_KURTOSIS_SAMPLE = 1 << 19     # elements sampled for the kurtosis test (:20)
_FIT_SAMPLE = 300000           # elements sampled for the Lloyd-Max fit (:69)
_FIT_ITERATIONS = 25           # Lloyd-Max iterations (:68)
_ROW_CHUNK_ELEMS = 1 << 22     # rows per preparation chunk: about 4 M elements (:215)
_CODEBOOK_ROWS_ELEMS = 1 << 22 # rows sampled to choose the codebook: about 4 M elements (:218)


def _nearest_index(values: torch.Tensor, levels: torch.Tensor) -> torch.Tensor:
    """Index of the nearest of 16 levels (``levels`` [16], or [..., 16] broadcast against
    ``values[..., G]`` as [..., 1]); ties keep the lower index (eager/w4a8_int8.py:36-62)."""
    per_group = levels.dim() > 1
    best = None
    index = torch.zeros(values.shape, dtype=torch.int32, device=values.device)
    for i in range(16):
        level = levels[..., i:i + 1].expand_as(values) if per_group else levels[i]
        dist = (values - level).abs()
        if best is None:
            best = dist
            continue
        closer = dist < best
        best = torch.where(closer, dist, best)
        index = torch.where(closer, i, index)
    return index


def _lloyd_max_codebook(normalized: torch.Tensor) -> torch.Tensor:
    """16-level Lloyd-Max fit on a seeded sample (eager/w4a8_int8.py:65-96): quantile
    initialisation, then 25 rounds of nearest-level assignment and mean update."""
    flat = normalized.flatten()
    if flat.numel() > _FIT_SAMPLE:
        gen = torch.Generator(device=flat.device).manual_seed(0)
        pick = torch.randint(0, flat.numel(), (_FIT_SAMPLE,), device=flat.device, generator=gen)
        flat = flat[pick]
    flat = flat.float()
    levels = torch.quantile(flat, torch.linspace(0, 1, 16, device=flat.device))
    for _ in range(_FIT_ITERATIONS):
        nearest = (flat.unsqueeze(-1) - levels).abs().argmin(-1)
        updated = levels.clone()
        for i in range(16):
            members = nearest == i
            if members.any():
                updated[i] = flat[members].mean()
        levels = updated
    return levels.contiguous()


def _choose_codebook(normalized: torch.Tensor) -> torch.Tensor:
    """The fixed table unless the normalised groups are heavy-tailed (excess kurtosis on a
    seeded sample above -0.1), then a fitted one (eager/w4a8_int8.py:23-33)."""
    flat = normalized.detach().flatten()
    if flat.numel() > _KURTOSIS_SAMPLE:
        gen = torch.Generator(device=flat.device).manual_seed(0)
        flat = flat[torch.randint(0, flat.numel(), (_KURTOSIS_SAMPLE,), device=flat.device, generator=gen)]
    flat = flat.float()
    kurtosis = ((flat - flat.mean()) / (flat.std() + 1e-9)).pow(4).mean() - 3.0
    if kurtosis.item() <= _KURTOSIS_GATE:
        return torch.tensor(W4A8_FIXED_CODEBOOK, dtype=torch.float32, device=normalized.device)
    return _lloyd_max_codebook(normalized)


def _tensor_codebook(w: torch.Tensor, group_size: int, convrot_groupsize: int) -> torch.Tensor:
    """One codebook per tensor, chosen from evenly strided rows (at most about 4 M
    elements) so the choice does not depend on the row chunking (eager/w4a8_int8.py:221-239)."""
    n, k = w.shape
    rows = max(1, _CODEBOOK_ROWS_ELEMS // max(k, 1))
    sample = w.index_select(0, torch.linspace(0, n - 1, rows, device=w.device).long()) if n > rows else w
    g = rotate_weight(sample.contiguous(), convrot_groupsize).float().view(sample.shape[0], k // group_size,
                                                                           group_size)
    return _choose_codebook(g / g.abs().amax(dim=-1, keepdim=True).clamp(min=1e-8))


def _w4a8_rows(wr: torch.Tensor, group_size: int, symmetric: bool, scale_dtype, codebook):
    """Quantize rotated rows (eager/w4a8_int8.py:122-209). Returns (codes int32 [n, k],
    s_rel, s_channel fp32 [n], correction bf16 [groups, n] or None)."""
    out_dtype = wr.dtype
    n, k = wr.shape
    g = wr.float().view(n, k // group_size, group_size)
    corr = None
    if codebook is not None:
        # scale per group, refined three times by least squares against the chosen levels
        gsc = g.abs().amax(dim=-1, keepdim=True).clamp(min=1e-8)
        codes = _nearest_index(g / gsc, codebook)
        for _ in range(3):
            lv = codebook[codes]
            gsc = ((g * lv).sum(-1, keepdim=True) / (lv * lv).sum(-1, keepdim=True).clamp(min=1e-8)).clamp(min=1e-8)
            codes = _nearest_index(g / gsc, codebook)
        shifted = codebook[codes] * gsc
    elif symmetric:
        gsc = (g.abs().amax(dim=-1, keepdim=True) / 7.0).clamp(min=1e-8)
        signed = (g / gsc).round().clamp(-8, 7).to(torch.int32)
        codes = signed + 8
        shifted = signed * gsc
    else:
        lo = g.amin(dim=-1, keepdim=True)
        gsc = ((g.amax(dim=-1, keepdim=True) - lo) / 15.0).clamp(min=1e-8)
        codes = ((g - lo) / gsc).round().clamp(0, 15).to(torch.int32)
        shifted = (codes - 8) * gsc
        corr = (8.0 * gsc + lo).squeeze(-1).t().contiguous().to(out_dtype)
    s_ch = (shifted.abs().amax(dim=(1, 2)) / 127.0).clamp(min=1e-8)
    s_rel = (gsc.squeeze(-1) / s_ch.unsqueeze(1)).float().contiguous()
    if scale_dtype != torch.float32:
        s_rel = s_rel.to(scale_dtype).contiguous()
    if codebook is not None:
        # final codes: nearest decoded int8 level of each weight, in units of s_channel
        grid = (codebook.view(1, 1, 16) * s_rel.float().unsqueeze(-1)).round_().clamp_(-127, 127)
        codes = _nearest_index(g / s_ch.view(-1, 1, 1), grid)
    return codes.reshape(n, k), s_rel, s_ch.float().contiguous(), corr


def pack_int4(codes: torch.Tensor) -> torch.Tensor:
    """int32 codes [n, k] in [0, 16) -> int8 [n, k/2], even column in the low nibble
    (eager/w4a8_int8.py:200-202)."""
    return ((codes[:, 0::2] & 0xF) | ((codes[:, 1::2] & 0xF) << 4)).to(torch.int8).contiguous()


def quantize_w4a8_int8_weight(weight: torch.Tensor, group_size: int = 16, convrot_groupsize: int = 256,
                              symmetric: bool = True, scale_dtype: torch.dtype = torch.float8_e4m3fn,
                              codebook: bool = True, codebook_tensor: torch.Tensor | None = None):
    """Rotate and pack a floating weight [N, K] into grouped W4A8 storage.

    ``quantize_w4a8_int8_weight`` (backends/eager/w4a8_int8.py:315-341, rows in chunks of
    about 4 M elements as :242-312): returns ``(qdata int8 [N, K/2], s_rel [N, K/g] in
    ``scale_dtype``, s_channel fp32 [N], correction bf16 [K/g, N] or None, codebook fp32
    [16] or None)``. The defaults are the H3 release format. Offline preparation in torch
    tensor operations; the codebook is chosen once for the whole tensor (or taken from
    ``codebook_tensor``)."""
    if weight.dim() != 2:
        raise ValueError(f"W4A8 weight must be 2D, got shape {tuple(weight.shape)}")
    n, k = weight.shape
    if (k % 16 or k % group_size or k % convrot_groupsize or group_size < 4
            or (16 % group_size and group_size % 16)):
        raise ValueError(f"K={k} must be divisible by 16, group_size={group_size}, and "
                         f"convrot_groupsize={convrot_groupsize}; group_size must be >=4 "
                         f"and divide 16 or be a multiple of 16")
    if scale_dtype not in (torch.float32, torch.float8_e4m3fn):
        raise ValueError(f"scale_dtype must be float32 or float8_e4m3fn, got {scale_dtype}")
    cb = None
    if symmetric and codebook:
        cb = (codebook_tensor.to(device=weight.device, dtype=torch.float32) if codebook_tensor is not None
              else _tensor_codebook(weight, group_size, convrot_groupsize))
    rows = max(1, _ROW_CHUNK_ELEMS // max(k, 1))
    parts = [_w4a8_rows(rotate_weight(weight[r:r + rows].contiguous(), convrot_groupsize), group_size,
                        symmetric, scale_dtype, cb) for r in range(0, n, rows)]
    packed = torch.cat([pack_int4(p[0]) for p in parts], 0)
    s_rel = torch.cat([p[1] for p in parts], 0)
    s_ch = torch.cat([p[2] for p in parts], 0)
    corr = torch.cat([p[3] for p in parts], 1) if parts[0][3] is not None else None
    return packed, s_rel, s_ch, corr, cb


@dataclass
class W4A8SwiGLUMLPWeights:
    """One H3 SwiGLU MLP in the H3 release W4A8 format: fc1 [2 ffn, d] ([gate | up] output
    rows), fc2 [d, ffn], both ConvRot-256 rotated, int4 codes packed two per byte, group
    ``group_size`` scales ``s_rel`` (fp8-e4m3 or fp32), per-channel fp32 ``s_channel``,
    optional 16-level codebooks and optional bf16 biases (ConvRotW4A8Linear,
    h3serve/native_engine/model/quantization.py:416-600; symmetric, no correction)."""

    q1: torch.Tensor
    s_rel1: torch.Tensor
    s_ch1: torch.Tensor
    q2: torch.Tensor
    s_rel2: torch.Tensor
    s_ch2: torch.Tensor
    codebook1: torch.Tensor | None = None
    codebook2: torch.Tensor | None = None
    b1: torch.Tensor | None = None
    b2: torch.Tensor | None = None
    group_size: int = 16

    @classmethod
    def from_float(cls, w1: torch.Tensor, w2: torch.Tensor, b1: torch.Tensor | None = None,
                   b2: torch.Tensor | None = None, group_size: int = 16,
                   scale_dtype: torch.dtype = torch.float8_e4m3fn, codebook: bool = True) -> "W4A8SwiGLUMLPWeights":
        q1, sr1, sc1, c1, cb1 = quantize_w4a8_int8_weight(w1, group_size, 256, True, scale_dtype, codebook)
        q2, sr2, sc2, c2, cb2 = quantize_w4a8_int8_weight(w2, group_size, 256, True, scale_dtype, codebook)
        assert c1 is None and c2 is None
        cast = (lambda b: None if b is None else b.to(torch.bfloat16).contiguous())
        return cls(q1, sr1, sc1, q2, sr2, sc2, cb1, cb2, cast(b1), cast(b2), group_size)

    def to(self, device) -> "W4A8SwiGLUMLPWeights":
        mv = (lambda t: None if t is None else t.to(device))
        return W4A8SwiGLUMLPWeights(mv(self.q1), mv(self.s_rel1), mv(self.s_ch1), mv(self.q2), mv(self.s_rel2),
                                    mv(self.s_ch2), mv(self.codebook1), mv(self.codebook2), mv(self.b1),
                                    mv(self.b2), self.group_size)

    @property
    def d(self) -> int:
        return self.q1.shape[1] * 2

    @property
    def ffn(self) -> int:
        return self.q1.shape[0] // 2


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
