"""torch-CPU restatement of the reference eager hot path, used as the timed CPU baseline.

TEST / BASELINE INFRASTRUCTURE ONLY (see ``oracle/__init__.py``). The reference
(X-MinimaxH3 with its vendored comfy_kitchen) is Python and cannot travel to the
GPU box, so ``bench.py``'s ``cpu_baseline`` and ``--impl reference`` legs time
this port instead: the same torch CPU operators the reference's eager backend
calls, in the same order, on all host threads:

* ``quantize_int8_rowwise``  backends/eager/quantization.py:857-875
* ``int8_linear``            backends/eager/quantization.py:971-1056
  (``torch._int_mm`` int32 GEMM, chunked fp32 dequant, bf16 store)
* ``apply_input_act``        backends/_activations.py:40-53
* gated residual ``addcmul_``  h3serve/native_engine/model/fused_mlp.py:414-425
* ``rms_adaln`` eager order  h3serve/native_engine/model/kernels.py:7623-7631
* ``apply_rope_split_half1`` backends/eager/rope.py:39-42

Its outputs are checked against the golden fixtures in the CPU test suite.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def quantize_int8_rowwise(x: torch.Tensor):
    abs_max = x.abs().amax(dim=-1, keepdim=True)
    scale = (abs_max.float() / 127.0).clamp(min=1e-30)
    sb = scale.to(x.dtype)
    sb = torch.where(sb == 0, torch.full_like(sb, torch.finfo(x.dtype).tiny), sb)
    q = (x / sb).round_().clamp_(-128.0, 127.0).to(torch.int8)
    return q, scale


def int8_linear(x: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor, input_act=None) -> torch.Tensor:
    if input_act == "gelu_tanh":
        x = F.gelu(x, approximate="tanh")
    xq, xs = quantize_int8_rowwise(x)
    acc = torch._int_mm(xq, wq.t().contiguous())
    m, n = acc.shape
    chunk = max(1, min(m, 256 * 1024 * 1024 // (n * 4)))
    ws = ws.reshape(1, -1).float()
    parts = []
    for i in range(0, m, chunk):
        parts.append((acc[i:i + chunk].float() * (xs[i:i + chunk] * ws)).to(torch.bfloat16))
    return torch.cat(parts, dim=0)


def w8a8_gelu_mlp(x, w1q, s1, w2q, s2, gate, residual) -> torch.Tensor:
    h = int8_linear(x, w1q, s1)
    y = int8_linear(h, w2q, s2, input_act="gelu_tanh")
    return residual.clone().addcmul_(y, gate)


def adaln_rms_rope(q, k, table, wq, wk, scale, shift, eps=1e-6):
    """q, k [M, H, D] bf16; table fp32 [M, D/2, 2, 2]; row-span RMSNorm + modulation + RoPE."""
    m, h, d = q.shape
    t = table.reshape(1, m, 1, d // 2, 2, 2)
    outs = []
    for x, w in ((q, wq), (k, wk)):
        hid = F.rms_norm(x.reshape(m, h * d), (h * d,), weight=w, eps=eps)
        hid.mul_(1.0 + scale.to(hid.dtype)).add_(shift.to(hid.dtype))
        x4 = hid.reshape(1, m, h, d)
        t_ = x4.reshape(*x4.shape[:-1], 2, -1).movedim(-2, -1).unsqueeze(-2).to(torch.float32)
        o = t[..., 0] * t_[..., 0] + t[..., 1] * t_[..., 1]
        outs.append(o.movedim(-1, -2).reshape(*x4.shape).type_as(x4)[0])
    return outs[0], outs[1]
