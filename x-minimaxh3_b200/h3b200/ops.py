"""Operator surface of the quantized DiT-block hot path (comfy_kitchen-compatible).

Every function takes CUDA tensors, allocates its outputs with torch on the
tensor's device, and launches the sm_100a kernels of ``libh3b200.so`` through
the C ABI on ``torch.cuda.current_stream()``. Argument names, meanings and
errors follow the reference operators (comfy_kitchen 0.2.28, vendored in
X-MinimaxH3 under ``backends/turbo/vendor/comfy_kitchen``); each function cites
the one it replaces. There is no CPU or library fallback: unsupported inputs
raise.
"""

from __future__ import annotations

import torch

from . import _lib

__all__ = [
    "apply_input_act",
    "quantize_int8_rowwise",
    "quantize_int8_rowwise_absmax",
    "mm_int8",
    "int8_linear_prequantized",
    "int8_linear",
    "int8_gemm_fused",
    "dequant_gated_residual",
    "fused_gated_mlp",
    "fused_gated_mlp_w4a8",
    "fused_gated_mlp_swiglu_w4a8",
    "adaln_rms_rope",
    "adaln_rms_rope_",
    "rms_adaln",
    "rms_adaln_segmented",
    "rms_rope_split_half",
    "rms_rope_split_half_",
    "qknorm_rope_strided_",
    "single_qknorm_rope_",
    "single_qknorm_rope_to_hnd",
    "qkv_qknorm_rope",
    "dequant_int4_grouped_to_int8",
    "quantize_int8_rowwise_convrot",
    "w4a8_int8_linear",
    "input_act_code",
]

_ACT = {None: _lib.ACT_NONE, "none": _lib.ACT_NONE, "gelu_tanh": _lib.ACT_GELU_TANH, "swiglu": _lib.ACT_SWIGLU}


def input_act_code(input_act) -> int:
    """Kernel code for ``input_act`` (backends/_activations.py:19-33)."""
    try:
        return _ACT[input_act]
    except KeyError:
        known = sorted(k for k in _ACT if k is not None)
        raise ValueError(f"unsupported input_act: {input_act!r} (expected one of {known})") from None


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("h3b200 operators take CUDA tensors only (no CPU fallback)")


_OUT_CODES = {torch.bfloat16: 2, torch.float16: 1}  # H3B200_DTYPE_BF16 / H3B200_DTYPE_F16


def _rows(x: torch.Tensor):
    """View x as [rows, K] with unit stride along K; returns (x2d, row_stride)."""
    k = x.shape[-1]
    if x.dim() == 2 and x.stride(1) == 1 and x.stride(0) >= k:
        return x, x.stride(0)
    x2 = x.reshape(-1, k)
    if x2.stride(-1) != 1 or (x2.shape[0] > 1 and x2.stride(0) < k):
        x2 = x2.contiguous()
    return x2, (x2.stride(0) if x2.shape[0] > 1 else k)


def _ptr(t):
    return None if t is None else t.data_ptr()


def input_act_width(input_act) -> int:
    """Raw input columns per activated column (backends/_activations.py:36-38): 2 for swiglu."""
    return 2 if input_act_code(input_act) == _lib.ACT_SWIGLU else 1


def _act_k(x: torch.Tensor, input_act) -> int:
    """Width of the activated row of x."""
    w = input_act_width(input_act)
    if x.shape[-1] % w:
        raise ValueError(f"swiglu needs an even last dimension ([gate | up]), got {x.shape[-1]}")
    return x.shape[-1] // w


def apply_input_act(x: torch.Tensor, input_act) -> torch.Tensor:
    """Pre-quantization activation (backends/_activations.py:40-53), bit-identical to
    the reference's CPU result for every bf16 input: ``gelu(approximate="tanh")``, or
    for ``swiglu`` ``silu(gate) * up`` of the ``[gate | up]`` halves of the last dim."""
    _need_cuda(x)
    code = input_act_code(input_act)
    if code == _lib.ACT_NONE:
        return x
    if x.dtype != torch.bfloat16:
        raise ValueError("apply_input_act expects bf16")
    if code == _lib.ACT_SWIGLU:
        k = _act_k(x, input_act)
        x2, ldx = _rows(x)
        y = torch.empty((x2.shape[0], k), dtype=torch.bfloat16, device=x.device)
        _lib.call("h3b200_swiglu", x2.data_ptr(), ldx, y.data_ptr(), k, x2.shape[0], k, _stream(x))
        return y.reshape(*x.shape[:-1], k)
    xc = x.contiguous()
    y = torch.empty_like(xc)
    _lib.call("h3b200_apply_input_act", xc.data_ptr(), y.data_ptr(), xc.numel(), code, _stream(x))
    return y


# ---------------------------------------------------------------------------
# (a) quantizer
# ---------------------------------------------------------------------------


def quantize_int8_rowwise(x: torch.Tensor, stochastic_rounding: int | None = 0, input_act=None):
    """Per-row absmax INT8 quantization -> (int8 [..., K], fp32 scales [..., 1]).

    Replaces ``comfy_kitchen.quantize_int8_rowwise`` (__init__.py:702-709;
    eager eager/quantization.py:857-875; CUDA backends/cuda/ops/int8_linear.cu:157-200).
    ``stochastic_rounding`` > 0 is the seed of stochastic rounding: the reference CUDA
    kernel's counter-based noise is added to the bf16 quotient, which is then floored
    (``h3b200_quantize_int8_rowwise_stochastic``); <= 0 or None rounds to nearest even.
    An fp16 ``x`` is quantized with the reference's fp16 arithmetic (fp16 divisor and
    quotient, ``h3b200_quantize_int8_rowwise_f16``); it takes no input activation and
    no stochastic rounding."""
    _need_cuda(x)
    if x.dtype == torch.float16:
        if input_act is not None or (stochastic_rounding is not None and stochastic_rounding > 0):
            raise NotImplementedError("fp16 activations are quantized without input_act and stochastic rounding "
                                      "(the exact activation tables are built for bf16 inputs)")
        x2, ldx = _rows(x)
        m, k = x2.shape
        q = torch.empty((m, k), dtype=torch.int8, device=x.device)
        s = torch.empty((m, 1), dtype=torch.float32, device=x.device)
        _lib.call("h3b200_quantize_int8_rowwise_f16", x2.data_ptr(), m, k, ldx, q.data_ptr(), s.data_ptr(), _stream(x))
        return q.reshape(*x.shape[:-1], k), s.reshape(*x.shape[:-1], 1)
    if x.dtype != torch.bfloat16:
        raise ValueError(f"quantize_int8_rowwise expects bf16 or fp16, got {x.dtype}")
    k = _act_k(x, input_act)
    x2, ldx = _rows(x)
    m = x2.shape[0]
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    s = torch.empty((m, 1), dtype=torch.float32, device=x.device)
    if stochastic_rounding is not None and stochastic_rounding > 0:
        _lib.call("h3b200_quantize_int8_rowwise_stochastic", x2.data_ptr(), m, k, ldx, input_act_code(input_act),
                  int(stochastic_rounding), q.data_ptr(), s.data_ptr(), _stream(x))
    else:
        _lib.call("h3b200_quantize_int8_rowwise", x2.data_ptr(), m, k, ldx, input_act_code(input_act), q.data_ptr(),
                  s.data_ptr(), _stream(x))
    return q.reshape(*x.shape[:-1], k), s.reshape(*x.shape[:-1], 1)


def quantize_int8_rowwise_absmax(x: torch.Tensor, absmax: torch.Tensor):
    """Quantizer body with a precomputed fp32 row absmax [..., 1] (same arithmetic)."""
    _need_cuda(x, absmax)
    x2, ldx = _rows(x)
    m, k = x2.shape
    am = absmax.reshape(-1).to(torch.float32).contiguous()
    if am.numel() != m:
        raise ValueError("absmax must have one value per row")
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    s = torch.empty((m, 1), dtype=torch.float32, device=x.device)
    _lib.call("h3b200_quantize_int8_rowwise_absmax", x2.data_ptr(), am.data_ptr(), m, k, ldx, q.data_ptr(),
              s.data_ptr(), _stream(x))
    return q.reshape(x.shape), s.reshape(*x.shape[:-1], 1)


# ---------------------------------------------------------------------------
# (b) INT8 GEMM / linear / fused MLP
# ---------------------------------------------------------------------------


def mm_int8(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """INT8 matmul ``C[M, N] = A[M, K] @ B[K, N]`` with int32 accumulators.

    Replaces ``comfy_kitchen.mm_int8`` / ``_int8_matmul_accumulate``
    (eager/quantization.py:749-800). ``b`` may be a transposed view of a
    row-major [N, K] weight (no copy in that case)."""
    _need_cuda(a, b)
    if a.dtype != torch.int8 or b.dtype != torch.int8 or a.dim() != 2 or b.dim() != 2:
        raise ValueError("mm_int8 takes 2-D int8 tensors")
    if a.size(1) != b.size(0):
        raise ValueError(f"K mismatch: {a.size(1)} vs {b.size(0)}")
    a = a.contiguous()
    w = b.t()
    if not w.is_contiguous():
        w = w.contiguous()
    m, k = a.shape
    n = w.shape[0]
    out = torch.empty((m, n), dtype=torch.int32, device=a.device)
    _lib.call("h3b200_int8_mm", a.data_ptr(), w.data_ptr(), m, n, k, out.data_ptr(), _stream(a))
    return out


def _weight_scale(weight_scale: torch.Tensor, n: int, device) -> torch.Tensor:
    ws = weight_scale.to(device=device, dtype=torch.float32).reshape(-1).contiguous()
    if ws.numel() not in (1, n):
        raise ValueError(f"INT8 weight scale must be scalar or per-output-channel, got {tuple(weight_scale.shape)} "
                         f"for {n} output channels")
    return ws


def int8_linear_prequantized(x_qdata: torch.Tensor, x_scale: torch.Tensor, weight: torch.Tensor,
                             weight_scale: torch.Tensor, bias: torch.Tensor | None = None,
                             out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """INT8 linear from a row-quantized activation (backends/cuda/__init__.py:1934-1957).

    ``out = out_dtype(float(acc) * (x_scale[row] * weight_scale[col])) (+ bias)`` with
    the eager association (eager/quantization.py:1044-1053): bf16 or fp16 out, the bias
    converted to the output dtype and added in it."""
    _need_cuda(x_qdata, x_scale, weight)
    if out_dtype not in _OUT_CODES:
        raise NotImplementedError(f"h3b200 builds bf16 and fp16 outputs, got {out_dtype}")
    xq = x_qdata.reshape(-1, x_qdata.shape[-1]).contiguous()
    m, k = xq.shape
    n, kw = weight.shape
    if k != kw:
        raise ValueError(f"Input and weight inner dimensions must match, got {k} and {kw}")
    w = weight.contiguous()
    xs = x_scale.reshape(-1).to(torch.float32).contiguous()
    ws = _weight_scale(weight_scale, n, xq.device)
    b = None if bias is None else bias.to(device=xq.device, dtype=out_dtype).contiguous()
    out = torch.empty((m, n), dtype=out_dtype, device=xq.device)
    _lib.call("h3b200_int8_linear_prequantized", xq.data_ptr(), xs.data_ptr(), w.data_ptr(), ws.data_ptr(),
              ws.numel(), _ptr(b), _OUT_CODES[out_dtype], out.data_ptr(), m, n, k, _stream(xq))
    return out.reshape(*x_qdata.shape[:-1], n)


EPI_I32, EPI_BF16, EPI_GELU_ABSMAX, EPI_GATED_RESIDUAL = 0, 1, 2, 3


def int8_gemm_fused(a: torch.Tensor, w: torch.Tensor, epilogue: int, a_scale=None, w_scale=None, bias=None,
                    gate=None, residual=None, out=None, row_absmax=None) -> torch.Tensor:
    """One tcgen05 INT8 GEMM with a fused epilogue (the stages of :func:`fused_gated_mlp`).

    ``epilogue``: EPI_I32 (int32 accumulators), EPI_BF16 (dequant + bias),
    EPI_GELU_ABSMAX (dequant -> tanh-GELU -> bf16, row absmax into ``row_absmax``),
    EPI_GATED_RESIDUAL (``residual + dequant * gate``). ``a`` [M, K] and ``w`` [N, K]
    are int8 with unit stride along K."""
    _need_cuda(a, w)
    m, k = a.shape
    n = w.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=torch.int32 if epilogue == EPI_I32 else torch.bfloat16, device=a.device)
    ws = None if w_scale is None else _weight_scale(w_scale, n, a.device)
    xs = None if a_scale is None else a_scale.reshape(-1).to(torch.float32).contiguous()
    _lib.call("h3b200_int8_gemm_fused", a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), m, n, k, int(epilogue),
              _ptr(xs), _ptr(ws), 0 if ws is None else ws.numel(), _ptr(bias), _ptr(gate), _ptr(residual),
              0 if residual is None else residual.stride(0), out.data_ptr(), out.stride(0), _ptr(row_absmax),
              _stream(a))
    return out


def requant_gemm_gated_residual(h: torch.Tensor, h_absmax: torch.Tensor, w: torch.Tensor, w_scale: torch.Tensor,
                                gate: torch.Tensor, residual: torch.Tensor, out: torch.Tensor | None = None,
                                bias: torch.Tensor | None = None, row_map: torch.Tensor | None = None,
                                workspace: torch.Tensor | None = None) -> torch.Tensor:
    """fc2 of the fused MLP with its input requantization inside the GEMM:
    ``residual + bf16(int8_linear_prequantized(quantize_int8_rowwise(h))) * gate``, where
    ``h_absmax[row]`` is max |h[row, :]| (the fc1 GELU epilogue's row absmax). ``gate`` is
    one row [n], or rows [R, n] picked per output row by the int32 ``row_map``."""
    _need_cuda(h, h_absmax, w, w_scale, gate, residual)
    h2, ldh = _rows(h)
    m, k = h2.shape
    n = w.shape[0]
    ws = _weight_scale(w_scale, n, h.device)
    amax = h_absmax.reshape(-1).to(torch.float32).contiguous()
    r2, ldr = _rows(residual)
    if out is None:
        out = torch.empty_like(r2)
    o2, ldo = _rows(out)
    if row_map is not None:
        g2, ldg = _rows(gate)
        rm = row_map.to(torch.int32).contiguous()
    else:
        g2, ldg, rm = gate.reshape(-1).contiguous(), 0, None
    need = int(_lib.load().h3b200_requant_gemm_workspace_bytes(m, k))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=h.device)
    _lib.call("h3b200_requant_gemm_gated_residual", h2.data_ptr(), ldh, amax.data_ptr(), w.data_ptr(), ws.data_ptr(),
              ws.numel(), _ptr(bias), g2.data_ptr(), ldg, _ptr(rm), r2.data_ptr(), ldr, o2.data_ptr(), ldo, m, n, k,
              workspace.data_ptr(), workspace.numel(), _stream(h))
    return out


def dequant_gated_residual(acc: torch.Tensor, x_scale: torch.Tensor, w_scale: torch.Tensor, gate: torch.Tensor,
                           residual: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``residual + bf16(acc * (x_scale * w_scale)) * gate`` on (cross-rank reduced) int32 accumulators."""
    _need_cuda(acc, x_scale, w_scale, gate, residual)
    m, n = acc.shape
    acc = acc.contiguous()
    xs = x_scale.reshape(-1).to(torch.float32).contiguous()
    ws = w_scale.reshape(-1).to(torch.float32).contiguous()
    g = gate.reshape(-1).contiguous()
    r2, ldr = _rows(residual)
    if out is None:
        out = torch.empty_like(r2)
    o2, ldo = _rows(out)
    _lib.call("h3b200_dequant_gated_residual", acc.data_ptr(), xs.data_ptr(), ws.data_ptr(), g.data_ptr(),
              r2.data_ptr(), ldr, o2.data_ptr(), ldo, m, n, _stream(acc))
    return out


def int8_linear(x: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor, bias: torch.Tensor | None = None,
                out_dtype: torch.dtype | None = None, convrot: bool = False, convrot_groupsize: int = 256,
                input_act: str | None = None) -> torch.Tensor:
    """Dynamically quantized INT8 linear.

    Replaces ``comfy_kitchen.int8_linear`` (__init__.py:722-764; CUDA
    backends/cuda/__init__.py:1960-2081; eager eager/quantization.py:971-1056):
    ``input_act`` on x, per-row quantization, INT8 GEMM, dequant (+ bias).
    ``convrot=True`` rotates the activation with the regular Hadamard-256 first."""
    _need_cuda(x, weight)
    if out_dtype is None:
        out_dtype = torch.bfloat16
    if out_dtype not in _OUT_CODES or x.dtype not in _OUT_CODES:
        raise NotImplementedError(f"h3b200 builds bf16 / fp16 activations and outputs, got {x.dtype} -> {out_dtype}")
    if x.dtype == torch.float16:
        if input_act is not None or convrot:
            raise NotImplementedError("fp16 activations: no input_act or convrot (the exact activation tables and "
                                      "the correctly rounded rotation are built for bf16)")
        if x.shape[-1] != weight.shape[-1]:
            raise ValueError(f"Input and weight inner dimensions must match, got {x.shape[-1]} and {weight.shape[-1]}")
        xq, xs = quantize_int8_rowwise(x)
        return int8_linear_prequantized(xq, xs, weight, weight_scale, bias, out_dtype)
    k = _act_k(x, input_act)  # swiglu: x rows are [gate | up], 2 K wide
    if k != weight.shape[-1]:
        raise ValueError(f"Input and weight inner dimensions must match, got {k} and {weight.shape[-1]}")
    act = input_act_code(input_act)
    n = weight.shape[0]
    if convrot:
        xq, xs = quantize_int8_rowwise_convrot(x, convrot_groupsize, input_act)
        return int8_linear_prequantized(xq, xs, weight, weight_scale, bias, out_dtype)
    if out_dtype != torch.bfloat16:        # bf16 x, fp16 out: quantize, then the fp16 epilogue
        xq, xs = quantize_int8_rowwise(x, input_act=input_act)
        return int8_linear_prequantized(xq, xs, weight, weight_scale, bias, out_dtype)
    x2, ldx = _rows(x)
    m = x2.shape[0]
    w = weight.contiguous()
    ws = _weight_scale(weight_scale, n, x.device)
    b = None if bias is None else bias.to(device=x.device, dtype=torch.bfloat16).contiguous()
    out = torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    nbytes = int(_lib.load().h3b200_int8_linear_workspace_bytes(m, k))
    work = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    _lib.call("h3b200_int8_linear", x2.data_ptr(), ldx, w.data_ptr(), ws.data_ptr(), ws.numel(), _ptr(b), act,
              out.data_ptr(), m, n, k, work.data_ptr(), nbytes, _stream(x))
    return out.reshape(*x.shape[:-1], n)


def fused_gated_mlp(residual: torch.Tensor, hidden: torch.Tensor, w1q: torch.Tensor, s1: torch.Tensor,
                    w2q: torch.Tensor, s2: torch.Tensor, gate: torch.Tensor, act: str = "gelu_tanh",
                    out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                    segments=None) -> torch.Tensor:
    """``residual + int8_linear(act(int8_linear(hidden, w1q, s1)), w2q, s2) * gate`` in one launch chain.

    Drop-in for ``try_fused_gated_mlp`` (h3serve/native_engine/model/fused_mlp.py:269-426;
    composition :393-425) with the tanh-GELU activation. ``gate`` is one modulation row [d],
    or with ``segments`` (``(start, stop, row)`` runs partitioning the tokens, the reference's
    modulation segments, ``_segment_row_map`` :34-55) rows [rows, d]: token t is gated by
    ``gate[row of t]`` (the per-segment ``addcmul_``, layers.py:937-953). ``out`` may be
    ``residual`` (in-place ``addcmul_``)."""
    _need_cuda(residual, hidden, w1q, w2q, gate)
    if act != "gelu_tanh":
        raise NotImplementedError(f"fused_gated_mlp builds act='gelu_tanh' only, got {act!r}")
    for name, t in (("residual", residual), ("hidden", hidden), ("gate", gate)):
        if t.dtype != torch.bfloat16:
            raise ValueError(f"{name} must be bf16, got {t.dtype}")
    x2, ldx = _rows(hidden)
    r2, ldr = _rows(residual)
    m, d = x2.shape
    ffn = w1q.shape[0]
    if tuple(w1q.shape) != (ffn, d) or tuple(w2q.shape) != (d, ffn):
        raise ValueError(f"weights must be w1 [ffn, d] and w2 [d, ffn], got {tuple(w1q.shape)} and {tuple(w2q.shape)}")
    if r2.shape != x2.shape:
        raise ValueError("residual and hidden must have the same shape")
    g, row_map, ldg = _gate_rows(gate, segments, m, d, hidden.device)
    ws1 = _weight_scale(s1, ffn, hidden.device)
    ws2 = _weight_scale(s2, d, hidden.device)
    if ws1.numel() != ffn or ws2.numel() != d:
        raise ValueError("fused_gated_mlp needs per-channel weight scales")
    if out is None:
        out = torch.empty_like(r2)
    o2, ldo = _rows(out)
    nbytes = int(_lib.load().h3b200_fused_gated_mlp_workspace_bytes(m, d, ffn))
    if workspace is None or workspace.numel() < nbytes:
        workspace = torch.empty(nbytes, dtype=torch.uint8, device=hidden.device)
    if row_map is None:
        _lib.call("h3b200_fused_gated_mlp", x2.data_ptr(), ldx, w1q.contiguous().data_ptr(), ws1.data_ptr(),
                  w2q.contiguous().data_ptr(), ws2.data_ptr(), g.data_ptr(), r2.data_ptr(), ldr, o2.data_ptr(), ldo,
                  m, d, ffn, _lib.ACT_GELU_TANH, workspace.data_ptr(), workspace.numel(), _stream(hidden))
    else:
        _lib.call("h3b200_fused_gated_mlp_segmented", x2.data_ptr(), ldx, w1q.contiguous().data_ptr(),
                  ws1.data_ptr(), w2q.contiguous().data_ptr(), ws2.data_ptr(), g.data_ptr(), ldg, row_map.data_ptr(),
                  r2.data_ptr(), ldr, o2.data_ptr(), ldo, m, d, ffn, _lib.ACT_GELU_TANH, workspace.data_ptr(),
                  workspace.numel(), _stream(hidden))
    return out


def fused_gated_mlp_w4a8(residual: torch.Tensor, hidden: torch.Tensor, weights, gate: torch.Tensor,
                         act: str = "gelu_tanh", out: torch.Tensor | None = None,
                         workspace: torch.Tensor | None = None) -> torch.Tensor:
    """``residual + w4a8_linear(gelu(w4a8_linear(hidden, W1)), W2) * gate`` (config-2 MLP).

    ``weights`` is a :class:`h3b200.W4A8MLPWeights` (the reference's asymmetric
    group-128 format, int4 at rest); each call decodes it into the workspace.
    Composition of ``w4a8_int8_linear`` (tensor/w4a8_int8.py:89-115), the
    tanh-GELU input activation and the addcmul of ``try_fused_gated_mlp``
    (h3serve/native_engine/model/fused_mlp.py:414-425)."""
    _need_cuda(residual, hidden, gate)
    if act != "gelu_tanh":
        raise NotImplementedError(f"fused_gated_mlp_w4a8 builds act='gelu_tanh' only, got {act!r}")
    for name, t in (("residual", residual), ("hidden", hidden), ("gate", gate)):
        if t.dtype != torch.bfloat16:
            raise ValueError(f"{name} must be bf16, got {t.dtype}")
    x2, ldx = _rows(hidden)
    r2, ldr = _rows(residual)
    m, d = x2.shape
    ffn = weights.ffn
    if weights.d != d or r2.shape != x2.shape:
        raise ValueError(f"hidden/residual [M, {d}] do not match the weights (d={weights.d})")
    g = gate.reshape(-1).contiguous()
    if g.numel() != d:
        raise ValueError(f"gate must have {d} elements (one modulation row)")
    if out is None:
        out = torch.empty_like(r2)
    o2, ldo = _rows(out)
    nbytes = int(_lib.load().h3b200_fused_gated_mlp_w4a8_workspace_bytes(m, d, ffn, weights.group_size))
    if workspace is None or workspace.numel() < nbytes:
        workspace = torch.empty(nbytes, dtype=torch.uint8, device=hidden.device)
    w = weights
    _lib.call("h3b200_fused_gated_mlp_w4a8", x2.data_ptr(), ldx, w.q1.data_ptr(), w.s_rel1.data_ptr(),
              w.s_ch1.data_ptr(), w.corr1.data_ptr(), w.q2.data_ptr(), w.s_rel2.data_ptr(), w.s_ch2.data_ptr(),
              w.corr2.data_ptr(), g.data_ptr(), r2.data_ptr(), ldr, o2.data_ptr(), ldo, m, d, ffn, w.group_size,
              _lib.ACT_GELU_TANH, workspace.data_ptr(), workspace.numel(), _stream(hidden))
    return out


# ---------------------------------------------------------------------------
# (c) AdaLN + RMSNorm + RoPE
# ---------------------------------------------------------------------------


def _qk3(t: torch.Tensor):
    """[1, M, H, D] / [M, H, D] -> ([M, H, D] view, token stride)."""
    if t.dim() == 4:
        if t.shape[0] != 1:
            raise ValueError("batch dimension must be 1 (packed token layout)")
        t = t[0]
    if t.dim() != 3:
        raise ValueError(f"expected [M, H, D] or [1, M, H, D], got {tuple(t.shape)}")
    if t.stride(2) != 1 or t.stride(1) != t.shape[2]:
        raise ValueError("heads x head_dim must be contiguous within a token")
    return t, t.stride(0)


def _freqs(freqs_cis: torch.Tensor, m: int, half: int) -> torch.Tensor:
    f = freqs_cis
    if f.dtype != torch.float32:
        raise ValueError("freqs_cis must be fp32")
    f = f.reshape(-1, f.shape[-3], 2, 2)
    if f.shape[0] != m or f.shape[1] < half:
        raise ValueError(f"freqs_cis must hold [M={m}, >= {half}, 2, 2] rotations, got {tuple(freqs_cis.shape)}")
    if f.shape[1] != half:
        f = f[:, :half]
    return f.contiguous()


def adaln_rms_rope_(q, k, freqs_cis, q_weight, k_weight=None, scale=None, shift=None, eps: float = 1e-6,
                    norm_span: str = "row", rot_dim: int = 0, q_out=None, k_out=None, segments=None):
    """Fused AdaLN-modulate + RMSNorm + split-half RoPE on Q and K, in place by default.

    ``norm_span="row"``: RMSNorm over heads*head_dim with [H*D] weights, then
    ``*(1 + scale)`` and ``+ shift`` (bf16 after each) -- the eager order of H3's
    ``rms_adaln`` (h3serve/native_engine/model/kernels.py:7586-7634) -- then
    per-head split-half RoPE (eager/rope.py:39-42). ``scale``/``shift`` are one row
    [H*D], or with ``segments`` (``(start, stop, row)`` runs partitioning the tokens,
    the reference's modulation segments) rows [rows, H*D] selected per token.
    ``norm_span="head"``: per-head RMSNorm with [D] weights (``rms_rope_split_half``,
    eager/rope.py:67-143), optional single-row modulation after it.
    Returns (q_out, k_out)."""
    _need_cuda(q, k, freqs_cis, q_weight)
    if k_weight is None:
        k_weight = q_weight
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16:
        raise ValueError("q and k must be bf16")
    q3, ldq = _qk3(q)
    k3, ldk = _qk3(k)
    if q3.shape != k3.shape:
        raise ValueError("q and k must have the same [M, H, D] shape")
    m, h, d = q3.shape
    rd = d if rot_dim in (0, None) else int(rot_dim)
    if q_out is None:
        q_out = q
    if k_out is None:
        k_out = k
    qo3, ldqo = _qk3(q_out)
    ko3, ldko = _qk3(k_out)
    span = {"row": 0, "head": 1}.get(norm_span)
    if span is None:
        raise ValueError(f"norm_span must be 'row' or 'head', got {norm_span!r}")
    width = h * d if span == 0 else d
    wq = q_weight.to(device=q.device, dtype=torch.bfloat16).reshape(-1).contiguous()
    wk = k_weight.to(device=q.device, dtype=torch.bfloat16).reshape(-1).contiguous()
    if wq.numel() != width or wk.numel() != width:
        raise ValueError(f"norm weights must have {width} elements for norm_span={norm_span!r}")
    sc = sh = None
    if scale is not None or shift is not None:
        if scale is None or shift is None:
            raise ValueError("scale and shift must be given together")
        if segments is not None:
            if span != 0:
                raise NotImplementedError("per-segment modulation is built for norm_span='row'")
            sc = _mod_rows(scale, h * d, q.device, "scale")
            sh = _mod_rows(shift, h * d, q.device, "shift")
            row_map = segment_row_map(m, segments, q.device)
            if m and max(int(r) for _, _, r in segments) >= min(sc.shape[0], sh.shape[0]):
                raise ValueError("a segment names a modulation row outside scale/shift")
            f = _freqs(freqs_cis, m, rd // 2)
            _lib.call("h3b200_adaln_rms_rope_segmented", q3.data_ptr(), ldq, k3.data_ptr(), ldk, qo3.data_ptr(),
                      ldqo, ko3.data_ptr(), ldko, f.data_ptr(), wq.data_ptr(), wk.data_ptr(), sc.data_ptr(),
                      sc.stride(0) if sc.shape[0] > 1 else h * d, sh.data_ptr(),
                      sh.stride(0) if sh.shape[0] > 1 else h * d, min(sc.shape[0], sh.shape[0]),
                      row_map.data_ptr(), 0, m, h, d, rd, float(eps), _stream(q))
            return q_out, k_out
        sc = scale.to(device=q.device, dtype=torch.bfloat16).reshape(-1).contiguous()
        sh = shift.to(device=q.device, dtype=torch.bfloat16).reshape(-1).contiguous()
        if sc.numel() != h * d or sh.numel() != h * d:
            raise ValueError(f"scale/shift must have {h * d} elements (one modulation row)")
    elif segments is not None:
        raise ValueError("segments need scale and shift")
    f = _freqs(freqs_cis, m, rd // 2)
    _lib.call("h3b200_adaln_rms_rope", q3.data_ptr(), ldq, k3.data_ptr(), ldk, qo3.data_ptr(), ldqo, ko3.data_ptr(),
              ldko, f.data_ptr(), wq.data_ptr(), wk.data_ptr(), _ptr(sc), _ptr(sh), m, h, d, rd, span, float(eps),
              _stream(q))
    return q_out, k_out


def _mod_rows(t, d: int, device, name: str) -> torch.Tensor:
    """Modulation rows as bf16 [rows, d] with unit column stride (a strided row view is kept)."""
    if t.shape[-1] != d:
        raise ValueError(f"{name} must have {d} features in its last dimension, got {tuple(t.shape)}")
    r = t.reshape(-1, d) if t.dim() != 2 else t
    r = r.to(device=device, dtype=torch.bfloat16)
    if r.stride(-1) != 1 or (r.shape[0] > 1 and (r.stride(0) < d or r.stride(0) % 8)) or r.data_ptr() % 16:
        r = r.contiguous()
    return r


def _rms_adaln_launch(x2, ldx, weight, sc, sh, row_map, tokens_per_row, eps, out2, ldo):
    m, d = x2.shape
    lds = sc.stride(0) if sc is not None and sc.shape[0] > 1 else d
    ldh = sh.stride(0) if sh is not None and sh.shape[0] > 1 else d
    _lib.call("h3b200_rms_adaln", x2.data_ptr(), ldx, _ptr(weight), _ptr(sc), lds, _ptr(sh), ldh,
              0 if sc is None else sc.shape[0], _ptr(row_map), int(tokens_per_row), float(eps), out2.data_ptr(),
              ldo, m, d, _stream(x2))


def rms_adaln(x: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor, eps: float = 1e-6,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """``rmsnorm(x) * (1 + scale) + shift`` without an affine weight, bf16 after each step.

    comfy_kitchen ``rms_adaln(x, scale, shift, eps)`` (``__init__.py:130-150``; eager
    ``backends/eager/adaln.py:17-20``). ``x`` bf16 ``[..., D]``; ``scale`` / ``shift`` bf16 and
    broadcastable to ``x`` with a full last dimension D: one row ``[D]``, per-sample rows such as
    ``[B, 1, D]``, or one row per token. Each token's modulation row is found from the broadcast
    shape (a row map, or ``tokens_per_row`` for the per-sample case); nothing is expanded."""
    _need_cuda(x, scale, shift)
    if x.dtype != torch.bfloat16:
        raise ValueError("rms_adaln expects bf16 x")
    if scale.dtype != torch.bfloat16 or shift.dtype != torch.bfloat16:
        raise NotImplementedError("rms_adaln builds bf16 scale/shift (other dtypes promote the result in eager)")
    d = x.shape[-1]
    if scale.shape != shift.shape:
        raise ValueError(f"scale {tuple(scale.shape)} and shift {tuple(shift.shape)} must have the same shape")
    if scale.shape[-1] != d or scale.dim() > x.dim():
        raise ValueError(f"scale/shift {tuple(scale.shape)} do not broadcast to x {tuple(x.shape)} with a full "
                         "last dimension")
    lead_x = tuple(x.shape[:-1])
    lead_s = (1,) * (x.dim() - scale.dim()) + tuple(scale.shape[:-1])
    for a, b in zip(lead_s, lead_x):
        if a not in (1, b):
            raise ValueError(f"scale/shift {tuple(scale.shape)} do not broadcast to x {tuple(x.shape)}")
    x2, ldx = _rows(x)
    n = x2.shape[0]
    sc = _mod_rows(scale, d, x.device, "scale")
    sh = _mod_rows(shift, d, x.device, "shift")
    row_map, tpr = None, 0
    rows = sc.shape[0]
    if rows > 1:
        # the dims scale/shift vary along: a contiguous run of leading 1s then full dims means one
        # row per tokens_per_row tokens; anything else takes an explicit row map
        varying = [i for i, a in enumerate(lead_s) if a != 1]
        tail = 1
        for b in lead_x[varying[-1] + 1:]:
            tail *= b
        if varying == list(range(varying[0], varying[-1] + 1)) and all(lead_s[i] == lead_x[i] for i in varying) \
                and all(a == 1 for a in lead_s[:varying[0]]) and all(b == 1 for b in lead_x[:varying[0]]):
            tpr = tail
        else:
            idx = torch.arange(rows, dtype=torch.int32, device=x.device).reshape(lead_s)
            row_map = idx.expand(lead_x).reshape(-1).contiguous()
    if out is None:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    o2, ldo = _rows(out)
    _rms_adaln_launch(x2, ldx, None, sc, sh, row_map, tpr, eps, o2, ldo)
    return out


def rms_adaln_segmented(value: torch.Tensor, norm, shift: torch.Tensor, scale: torch.Tensor, segments,
                        out: torch.Tensor | None = None) -> torch.Tensor:
    """H3's ``rms_adaln(value, norm, shift, scale, segments)``
    (h3serve/native_engine/model/kernels.py:7586-7634), same argument order.

    ``hidden = norm(value)`` (``F.rms_norm`` with ``norm.weight`` cast to bf16 and ``norm.eps``;
    ``norm=None`` or a norm without weight: no affine weight), then for every
    ``(start, stop, row)`` segment ``hidden[start:stop].mul_(1.0 + scale[row].to(bf16))
    .add_(shift[row].to(bf16))`` -- one pass over ``value`` [M, D] bf16. ``shift``/``scale`` are
    [rows, D] (the strided views ``split_adaln`` returns are read in place when bf16). The segments
    must partition ``[0, M)`` in order (same validation as the reference). ``out`` may be
    ``value``."""
    _need_cuda(value, shift, scale)
    if value.dtype != torch.bfloat16 or value.dim() != 2:
        raise ValueError("rms_adaln_segmented expects a 2-D bf16 value [tokens, hidden]")
    m, d = value.shape
    weight = getattr(norm, "weight", None) if norm is not None else None
    eps = float(getattr(norm, "eps", 1e-6)) if norm is not None else 1e-6
    w = None
    if weight is not None:
        w = weight.detach().to(device=value.device, dtype=torch.bfloat16).reshape(-1).contiguous()
        if w.numel() != d:
            raise ValueError(f"norm weight has {w.numel()} elements, value has {d} features")
    sc = _mod_rows(scale, d, value.device, "scale")
    sh = _mod_rows(shift, d, value.device, "shift")
    row_map = segment_row_map(m, segments, value.device)
    if m and int(max(r for _, _, r in segments)) >= min(sc.shape[0], sh.shape[0]):
        raise ValueError("a segment names a modulation row outside scale/shift")
    x2, ldx = _rows(value)
    if out is None:
        out = torch.empty_like(x2)
    o2, ldo = _rows(out)
    _rms_adaln_launch(x2, ldx, w, sc, sh, row_map, 0, eps, o2, ldo)
    return out


def adaln_rms_rope(q, k, freqs_cis, q_weight, k_weight=None, scale=None, shift=None, eps: float = 1e-6,
                   norm_span: str = "row", rot_dim: int = 0, segments=None):
    """Out-of-place variant of :func:`adaln_rms_rope_`."""
    return adaln_rms_rope_(q, k, freqs_cis, q_weight, k_weight, scale, shift, eps, norm_span, rot_dim,
                           q_out=torch.empty_like(q), k_out=torch.empty_like(k), segments=segments)


_TABLE_DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}   # eager/quantization.py:34-40


def _nhd(t: torch.Tensor, name: str) -> torch.Tensor:
    """[1, T, H, D] / [T, H, D] bf16 with unit stride on D -> [T, H, D] view."""
    if t.dim() == 4:
        if t.shape[0] != 1:
            raise ValueError(f"{name}: batch dimension must be 1 (packed token layout)")
        t = t[0]
    if t.dim() != 3:
        raise ValueError(f"{name}: expected [T, H, D] or [1, T, H, D], got {tuple(t.shape)}")
    if t.dtype != torch.bfloat16:
        raise ValueError(f"{name} must be bf16, got {t.dtype}")
    if t.stride(2) != 1:
        raise ValueError(f"{name}: head_dim must have unit stride")
    return t


def _rope_rows(frequencies: torch.Tensor, tokens: int, heads: int, pairs: int):
    """Rotation table [1, 1|T, 1|H, P, 2, 2] (or [T, P, 2, 2]) with P >= pairs -> (table with
    contiguous [P, 2, 2] rows, token stride, head stride) in elements (0 = broadcast)."""
    f = frequencies
    if f.dim() == 4:
        f = f.unsqueeze(0).unsqueeze(2)
    if f.dim() != 6 or tuple(f.shape[-2:]) != (2, 2):
        raise ValueError(f"frequencies must be [1, 1|T, 1|H, P, 2, 2], got {tuple(frequencies.shape)}")
    if f.shape[0] != 1 or f.shape[1] not in (1, tokens) or f.shape[2] not in (1, heads) or f.shape[3] < pairs:
        raise ValueError(f"frequencies {tuple(frequencies.shape)} do not cover {tokens} tokens x {heads} heads x "
                         f"{pairs} pairs")
    if f.dtype not in _TABLE_DTYPE_CODES:
        raise ValueError(f"frequencies must be float32, float16 or bfloat16, got {f.dtype}")
    if f.stride(5) != 1 or f.stride(4) != 2 or f.stride(3) != 4:
        f = f.contiguous()
    return f, (f.stride(1) if f.shape[1] != 1 else 0), (f.stride(2) if f.shape[2] != 1 else 0)


def qknorm_rope_strided_(q: torch.Tensor, q_weight: torch.Tensor, frequencies: torch.Tensor, eps: float = 1e-6,
                         rot_dim: int = 0, q_out: torch.Tensor | None = None, k: torch.Tensor | None = None,
                         k_weight: torch.Tensor | None = None, k_out: torch.Tensor | None = None):
    """Per-head RMSNorm + partial split-half RoPE on Q (and K when given) over strided
    [T, H, 128] views, writing ``q_out`` / ``k_out`` (default: in place), which may be
    HND-backed views. The reference launcher ``launch_rms_rope_kernel`` with
    ``split_half=True`` and ``has_k`` (backends/cuda/ops/rms_rope.cu:36-229); eager math
    backends/eager/rope.py:67-92. Returns (q_out, k_out)."""
    _need_cuda(q, q_weight, frequencies)
    q3 = _nhd(q, "q")
    t, h, d = q3.shape
    qo3 = _nhd(q if q_out is None else q_out, "q_out")
    if qo3.shape != q3.shape:
        raise ValueError("q_out must have q's [T, H, D] shape")
    rd = d if rot_dim in (0, None) else int(rot_dim)
    f, fst, fsh = _rope_rows(frequencies, t, h, rd // 2)
    wq = q_weight.to(device=q.device, dtype=torch.bfloat16).reshape(-1).contiguous()
    if wq.numel() != d:
        raise ValueError(f"q_weight must have {d} elements")
    k3 = ko3 = wk = None
    if k is not None:
        k3 = _nhd(k, "k")
        ko3 = _nhd(k if k_out is None else k_out, "k_out")
        if k3.shape != q3.shape or ko3.shape != q3.shape:
            raise ValueError("k and k_out must have q's [T, H, D] shape")
        wk = (q_weight if k_weight is None else k_weight).to(device=q.device, dtype=torch.bfloat16).reshape(-1)
        wk = wk.contiguous()
        if wk.numel() != d:
            raise ValueError(f"k_weight must have {d} elements")
    kp = (lambda v, i: 0 if v is None else v.stride(i))  # noqa: E731
    _lib.call("h3b200_qknorm_rope_strided", q3.data_ptr(), q3.stride(0), q3.stride(1), qo3.data_ptr(), qo3.stride(0),
              qo3.stride(1), wq.data_ptr(), _ptr(k3), kp(k3, 0), kp(k3, 1), _ptr(ko3), kp(ko3, 0), kp(ko3, 1), _ptr(wk),
              f.data_ptr(), _TABLE_DTYPE_CODES[f.dtype], fst, fsh, t, h, d, rd, float(eps), _stream(q))
    q_res = q if q_out is None else q_out
    k_res = None if k is None else (k if k_out is None else k_out)
    return q_res, k_res


def single_qknorm_rope_(value: torch.Tensor, *, weight: torch.Tensor, frequencies: torch.Tensor,
                        eps: float) -> torch.Tensor:
    """Single-side QK-norm + split-half RoPE in place on ``value`` [T, H, D]
    (``try_apply_single_qknorm_rope_``, h3serve/native_engine/model/single_qknorm_rope.py:
    190-206): ``rot_dim = 2 * frequencies.shape[-3]``. Raises where the reference returns
    False."""
    qknorm_rope_strided_(value, weight, frequencies, eps, 2 * int(frequencies.shape[-3]))
    return value


def single_qknorm_rope_to_hnd(value: torch.Tensor, output_nhd_view: torch.Tensor, *, weight: torch.Tensor,
                              frequencies: torch.Tensor, eps: float) -> torch.Tensor:
    """Single-side QK-norm + split-half RoPE from logical NHD ``value`` [T, H, D] into an
    HND-backed NHD view (``try_apply_single_qknorm_rope_to_hnd``,
    single_qknorm_rope.py:209-236: strides ``(D, >= T*D, 1)``, a multiple of D)."""
    t, h, d = value.shape
    s = tuple(int(v) for v in output_nhd_view.stride())
    if output_nhd_view.is_contiguous() or s[0] != d or s[1] < t * d or s[1] % d or s[2] != 1:
        raise ValueError(f"output view strides {s} are not an HND-backed [T, H, D] view")
    qknorm_rope_strided_(value, weight, frequencies, eps, 2 * int(frequencies.shape[-3]), q_out=output_nhd_view)
    return output_nhd_view


_QKV_SECTIONS = {"qkv": (0, 3), "qk": (0, 2), "kv": (1, 3), "q": (0, 1), "k": (1, 2), "v": (2, 3)}


def qkv_qknorm_rope(xq: torch.Tensor, x_scale: torch.Tensor, w_qkv: torch.Tensor, w_scale: torch.Tensor,
                    bias: torch.Tensor | None, heads: int, q_norm_weight: torch.Tensor | None,
                    k_norm_weight: torch.Tensor | None, frequencies: torch.Tensor | None, eps: float,
                    sections: str = "qkv", q_out=None, k_out=None, v_out=None, workspace=None):
    """Q/K/V projection of a token chunk with QK-norm + partial split-half RoPE, written into the
    attention layout.

    ``xq``/``x_scale``: the chunk's activation quantized once (``quantize_int8_rowwise_convrot``,
    the reference's ``prepare_output_slices``, h3serve/native_engine/model/quantization.py:
    340-375); ``w_qkv`` int8 [3 H 128, K] with rows Q | K | V and its per-row ``w_scale`` /
    ``bias``. ``sections`` picks the output rows computed, as ``forward_prepared_output_slice``
    does (:377-415): "qkv", "kv" (the K/V build), "q" (a query chunk), ... Q and K get per-head
    RMSNorm with their norm weights and, when ``frequencies`` is given, split-half RoPE over
    ``2 * frequencies.shape[-3]`` dims (layers.py:445-641 with
    ``try_apply_single_qknorm_rope_to_hnd``); V is copied. Outputs default to fresh HND
    buffers [H, m, 128]; any [m, H, 128] view (unit stride on the last dim) is accepted.
    Returns the (q, k, v) [m, H, 128] views (None for sections not computed)."""
    _need_cuda(xq, x_scale, w_qkv, w_scale)
    if sections not in _QKV_SECTIONS:
        raise ValueError(f"sections must be one of {sorted(_QKV_SECTIONS)}, got {sections!r}")
    s0, s1 = _QKV_SECTIONS[sections]
    if xq.dtype != torch.int8 or xq.dim() != 2 or xq.stride(1) != 1 or xq.stride(0) != xq.shape[1]:
        raise ValueError("xq must be a contiguous int8 [m, K] tensor")
    m, k = xq.shape
    inner = int(heads) * 128
    if w_qkv.dtype != torch.int8 or tuple(w_qkv.shape) != (3 * inner, k) or not w_qkv.is_contiguous():
        raise ValueError(f"w_qkv must be a contiguous int8 [{3 * inner}, {k}] tensor")
    xs = x_scale.to(torch.float32).reshape(-1).contiguous()
    ws = w_scale.to(torch.float32).reshape(-1).contiguous()
    if xs.numel() != m or ws.numel() not in (1, 3 * inner):
        raise ValueError("x_scale must have m values and w_scale 1 or 3 * heads * 128")
    b = None
    if bias is not None:
        b = bias.to(torch.bfloat16).reshape(-1).contiguous()
        if b.numel() != 3 * inner:
            raise ValueError(f"bias must have {3 * inner} values")
    f, fst, fsh, fcode, rot = None, 0, 0, 0, 0
    if frequencies is not None:
        rot = 2 * int(frequencies.shape[-3])
        f, fst, fsh = _rope_rows(frequencies, m, int(heads), rot // 2)
        fcode = _TABLE_DTYPE_CODES[f.dtype]
    outs = []
    for sec, view, nw in ((0, q_out, q_norm_weight), (1, k_out, k_norm_weight), (2, v_out, None)):
        if not s0 <= sec < s1:
            outs.append((None, None))
            continue
        if view is None:
            view = torch.empty(int(heads), m, 128, dtype=torch.bfloat16, device=xq.device).permute(1, 0, 2)
        view3 = _nhd(view, ("q_out", "k_out", "v_out")[sec])
        if tuple(view3.shape) != (m, int(heads), 128):
            raise ValueError(f"output view must be [{m}, {heads}, 128], got {tuple(view3.shape)}")
        w = None
        if sec < 2:
            if nw is None:
                raise ValueError("q_norm_weight / k_norm_weight are required for the Q / K sections")
            w = nw.to(device=xq.device, dtype=torch.bfloat16).reshape(-1).contiguous()
            if w.numel() != 128:
                raise ValueError("norm weights must have 128 values")
        outs.append((view3, w))
    nbytes = int(_lib.load().h3b200_qkv_qknorm_rope_workspace_bytes(m, int(heads), 128, s0, s1))
    if workspace is None or workspace.numel() < nbytes:
        workspace = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=xq.device)
    (qv, qw), (kv, kw), (vv, _) = outs
    st = (lambda v, i: 0 if v is None else v.stride(i))  # noqa: E731
    _lib.call("h3b200_qkv_qknorm_rope", xq.data_ptr(), xs.data_ptr(), m, k, w_qkv.data_ptr(), ws.data_ptr(),
              ws.numel(), _ptr(b), int(heads), 128, s0, s1, _ptr(qw), _ptr(kw), _ptr(f), fcode, fst, fsh, rot,
              float(eps), _ptr(qv), st(qv, 0), st(qv, 1), _ptr(kv), st(kv, 0), st(kv, 1), _ptr(vv), st(vv, 0),
              st(vv, 1), workspace.data_ptr(), workspace.numel(), _stream(xq))
    return qv, kv, vv


def _persistent_norm_rope_fits(q, k, freqs_cis) -> bool:
    """The persistent norm-RoPE kernel takes contiguous heads (at most 32 of 128) and an fp32
    table with one row per token; other layouts go to the strided kernel."""
    try:
        q3, k3 = _nhd(q, "q"), _nhd(k, "k")
    except ValueError:
        return False
    return (q3.shape[1] <= 32 and q3.shape[2] == 128 and q3.stride(1) == 128 and k3.stride(1) == 128
            and freqs_cis.dtype == torch.float32 and freqs_cis.numel() // (freqs_cis.shape[-3] * 4) == q3.shape[0])


def rms_rope_split_half_(q, k, freqs_cis, q_scale, k_scale=None, epsilon: float = 1e-6, rot_dim: int = 0):
    """In-place per-head RMSNorm + split-half RoPE (``comfy_kitchen.rms_rope_split_half_``,
    __init__.py:566-580; CUDA backends/cuda/ops/rms_rope.cu:36-229). Up to 32 contiguous
    heads with an fp32 per-token table run on the persistent norm-RoPE kernel; any other
    head count, stride or table dtype (e.g. H3's 56 heads, bf16 table) on the strided one."""
    if _persistent_norm_rope_fits(q, k, freqs_cis):
        return adaln_rms_rope_(q, k, freqs_cis, q_scale, k_scale, None, None, epsilon, "head", rot_dim)
    return qknorm_rope_strided_(q, q_scale, freqs_cis, epsilon, rot_dim, k=k,
                                k_weight=q_scale if k_scale is None else k_scale)


def rms_rope_split_half(q, k, freqs_cis, q_scale, k_scale=None, epsilon: float = 1e-6, rot_dim: int = 0):
    """Out-of-place ``comfy_kitchen.rms_rope_split_half`` (__init__.py:549-563)."""
    if _persistent_norm_rope_fits(q, k, freqs_cis):
        return adaln_rms_rope(q, k, freqs_cis, q_scale, k_scale, None, None, epsilon, "head", rot_dim)
    return qknorm_rope_strided_(q, q_scale, freqs_cis, epsilon, rot_dim, q_out=torch.empty_like(q), k=k,
                                k_weight=q_scale if k_scale is None else k_scale, k_out=torch.empty_like(k))


# ---------------------------------------------------------------------------
# W4A8
# ---------------------------------------------------------------------------


_S_REL_DTYPE_CODES = {torch.float32: 0, torch.float8_e4m3fn: 5}   # eager/quantization.py:34-40 codes


def _s_rel_code(s_rel: torch.Tensor) -> int:
    code = _S_REL_DTYPE_CODES.get(s_rel.dtype)
    if code is None:
        raise ValueError(f"s_rel must be float32 or float8_e4m3fn, got {s_rel.dtype}")
    return code


def _codebook(codebook, device):
    if codebook is None:
        return None
    cb = codebook.to(device=device, dtype=torch.float32).contiguous()
    if tuple(cb.shape) != (16,):
        raise ValueError(f"codebook must have shape (16,), got {tuple(cb.shape)}")
    return cb


def dequant_int4_grouped_to_int8(qdata: torch.Tensor, s_rel: torch.Tensor, group_size: int,
                                 codebook: torch.Tensor | None = None) -> torch.Tensor:
    """Decode packed uint4 to the int8 grid, ``clamp(rne(level(u) * s_rel), -127, 127)`` with
    ``level(u) = u - 8`` or ``codebook[u]``; ``s_rel`` fp32 or float8_e4m3fn
    (eager/w4a8_int8.py:344-363; CUDA w4a8_gemm.cu:36-121)."""
    _need_cuda(qdata, s_rel)
    code = _s_rel_code(s_rel)
    qd = qdata.contiguous()
    n, kh = qd.shape
    k = kh * 2
    sr = s_rel.contiguous()
    if tuple(sr.shape) != (n, k // group_size):
        raise ValueError(f"s_rel must have shape {(n, k // group_size)}, got {tuple(sr.shape)}")
    cb = _codebook(codebook, qd.device)
    out = torch.empty((n, k), dtype=torch.int8, device=qd.device)
    _lib.call("h3b200_dequant_int4_grouped_to_int8_ex", qd.data_ptr(), sr.data_ptr(), code, _ptr(cb), n, k,
              group_size, out.data_ptr(), _stream(qd))
    return out


def quantize_int8_rowwise_convrot(x: torch.Tensor, convrot_groupsize: int = 256, input_act=None):
    """ConvRot-256 rotation + row quantization (``quantize_and_rotate_rowwise``,
    eager/quantization.py:878-895; CUDA int8_linear.cu:256-340)."""
    _need_cuda(x)
    if x.dtype != torch.bfloat16:
        raise ValueError("x must be bf16")
    k = _act_k(x, input_act)
    x2, ldx = _rows(x)
    m = x2.shape[0]
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    s = torch.empty((m, 1), dtype=torch.float32, device=x.device)
    _lib.call("h3b200_quantize_int8_rowwise_convrot", x2.data_ptr(), m, k, ldx, convrot_groupsize,
              input_act_code(input_act), q.data_ptr(), s.data_ptr(), _stream(x))
    return q.reshape(*x.shape[:-1], k), s.reshape(*x.shape[:-1], 1)


_ROW_MAPS: dict = {}
_ROW_MAPS_MAX = 64


def segment_row_map(length: int, segments, device) -> torch.Tensor:
    """int32 [length]: the modulation row of each token, from ``(start, stop, row)`` segments
    that partition ``[0, length)`` in order (``_segment_row_map``,
    h3serve/native_engine/model/fused_mlp.py:34-55, same validation).

    A model calls this with the same few layouts in every block and step, so the device
    maps are cached per (length, segments, device) and must not be written by callers."""
    segs = tuple((int(a), int(b), int(r)) for a, b, r in segments)
    key = (int(length), segs, str(torch.device(device)))
    hit = _ROW_MAPS.get(key)
    if hit is not None:
        return hit
    host = torch.empty(length, dtype=torch.int32)
    previous = 0
    for start, stop, row in segs:
        if start != previous or stop <= start:
            raise ValueError("modulation segments must be an ordered partition")
        if row < 0:
            raise ValueError("modulation rows must be non-negative")
        host[start:stop] = row
        previous = stop
    if previous != length:
        raise ValueError("modulation segments do not cover the packed sequence")
    dev_map = host.to(device)
    if len(_ROW_MAPS) >= _ROW_MAPS_MAX:
        _ROW_MAPS.pop(next(iter(_ROW_MAPS)))
    _ROW_MAPS[key] = dev_map
    return dev_map


def _gate_rows(gate: torch.Tensor, segments, m: int, d: int, device):
    """(gate rows [rows, d] contiguous, int32 row map [m] or None, row stride) of a gated
    residual: one row [d] without segments, else the ``(start, stop, row)`` partition."""
    if segments is None:
        g = gate.reshape(-1).contiguous()
        if g.numel() != d:
            raise ValueError(f"gate must have {d} elements when no segments are given")
        return g, None, d
    g = gate.reshape(-1, d).contiguous()
    row_map = segment_row_map(m, segments, device)
    if m and int(row_map.max()) >= g.shape[0]:
        raise ValueError(f"a segment names gate row {int(row_map.max())}, gate has {g.shape[0]} rows")
    return g, row_map, d


def _mlp_io(residual, hidden, gate, d_w):
    _need_cuda(residual, hidden, gate)
    for name, t in (("residual", residual), ("hidden", hidden), ("gate", gate)):
        if t.dtype != torch.bfloat16:
            raise ValueError(f"{name} must be bf16, got {t.dtype}")
    x2, ldx = _rows(hidden)
    r2, ldr = _rows(residual)
    if x2.shape[1] != d_w or r2.shape != x2.shape:
        raise ValueError(f"hidden/residual [M, {x2.shape[1]}] do not match the weights (d={d_w})")
    return x2, ldx, r2, ldr


def fused_gated_mlp_swiglu(residual: torch.Tensor, hidden: torch.Tensor, weights, gate: torch.Tensor,
                           segments=None, out: torch.Tensor | None = None, chunk_tokens: int = 8192,
                           workspace: torch.Tensor | None = None) -> torch.Tensor:
    """The H3 SwiGLU MLP with the gated residual per modulation segment.

    Drop-in for the INT8 path of ``try_fused_gated_mlp`` (h3serve/native_engine/model/
    fused_mlp.py:269-426): ``raw = fc1(hidden)`` (ConvRot INT8 linear, fc1 bias),
    ``y = int8_linear(raw, W2, s2, b2, convrot=True, input_act="swiglu")``, then
    ``residual[a:b].addcmul_(y[a:b], gate[row])`` for each ``(a, b, row)`` in
    ``segments`` (``gate`` [rows, d]); with ``segments=None`` ``gate`` is one row [d].
    ``weights`` is a :class:`h3b200.SwiGLUMLPWeights`; ``out`` may be ``residual``."""
    x2, ldx, r2, ldr = _mlp_io(residual, hidden, gate, weights.d)
    m, d = x2.shape
    ffn = weights.ffn
    g, row_map, ldg = _gate_rows(gate, segments, m, d, hidden.device)
    if out is None:
        out = torch.empty_like(r2)
    o2, ldo = _rows(out)
    chunk = max(1, min(int(chunk_tokens), m)) if m else 1
    nbytes = int(_lib.load().h3b200_fused_gated_mlp_swiglu_workspace_bytes(chunk, d, ffn))
    if workspace is None or workspace.numel() < nbytes:
        workspace = torch.empty(nbytes, dtype=torch.uint8, device=hidden.device)
    s1 = weights.s1.to(torch.float32).contiguous()
    s2 = weights.s2.to(torch.float32).contiguous()
    _lib.call("h3b200_fused_gated_mlp_swiglu", x2.data_ptr(), ldx, weights.w1q.data_ptr(), s1.data_ptr(),
              s1.numel(), _ptr(weights.b1), weights.w2q.data_ptr(), s2.data_ptr(), s2.numel(), _ptr(weights.b2),
              g.data_ptr(), ldg, _ptr(row_map), r2.data_ptr(), ldr, o2.data_ptr(), ldo, m, d, ffn,
              256 if weights.fc1_convrot else 0, chunk, workspace.data_ptr(), workspace.numel(), _stream(hidden))
    return out


def fused_gated_mlp_swiglu_w4a8(residual: torch.Tensor, hidden: torch.Tensor, weights, gate: torch.Tensor,
                                segments=None, out: torch.Tensor | None = None, chunk_tokens: int = 8192,
                                workspace: torch.Tensor | None = None) -> torch.Tensor:
    """The H3 SwiGLU MLP on W4A8 weights (H3 release format: group 16, fp8-e4m3 ``s_rel``,
    16-level codebook, symmetric, ConvRot-256), gated residual per modulation segment.

    Drop-in for the W4A8 path of ``try_fused_gated_mlp``, ``_chunked_module_gated_mlp``
    (h3serve/native_engine/model/fused_mlp.py:222-266) over ``ConvRotW4A8Linear`` modules
    bound to ``comfy_kitchen.w4a8_int8_linear`` (quantization.py:64-95, 416-600):
    ``raw = fc1(hidden)``, ``y = fc2(silu(raw_gate) * raw_up)``, then the per-segment
    ``addcmul_``. ``weights`` is a :class:`h3b200.W4A8SwiGLUMLPWeights`; both int4 weights
    are decoded once per call into the workspace; ``out`` may be ``residual``."""
    x2, ldx, r2, ldr = _mlp_io(residual, hidden, gate, weights.d)
    m, d = x2.shape
    ffn = weights.ffn
    if weights.s_rel1.dtype != weights.s_rel2.dtype:
        raise ValueError("fc1 and fc2 s_rel must have the same dtype")
    code = _s_rel_code(weights.s_rel1)
    gsz = int(weights.group_size)
    for name, t, shape in (("s_rel1", weights.s_rel1, (2 * ffn, d // gsz)), ("s_rel2", weights.s_rel2, (d, ffn // gsz)),
                           ("s_ch1", weights.s_ch1, (2 * ffn,)), ("s_ch2", weights.s_ch2, (d,)),
                           ("q2", weights.q2, (d, ffn // 2))):
        if tuple(t.shape) != shape:
            raise ValueError(f"{name} must have shape {shape}, got {tuple(t.shape)}")
    g, row_map, ldg = _gate_rows(gate, segments, m, d, hidden.device)
    if out is None:
        out = torch.empty_like(r2)
    o2, ldo = _rows(out)
    chunk = max(1, min(int(chunk_tokens), m)) if m else 1
    nbytes = int(_lib.load().h3b200_fused_gated_mlp_swiglu_w4a8_workspace_bytes(chunk, d, ffn))
    if workspace is None or workspace.numel() < nbytes:
        workspace = torch.empty(nbytes, dtype=torch.uint8, device=hidden.device)
    c = lambda t: t.contiguous()  # noqa: E731
    sc1 = weights.s_ch1.to(torch.float32).contiguous()
    sc2 = weights.s_ch2.to(torch.float32).contiguous()
    cb1 = _codebook(weights.codebook1, hidden.device)
    cb2 = _codebook(weights.codebook2, hidden.device)
    q1, q2, sr1, sr2 = c(weights.q1), c(weights.q2), c(weights.s_rel1), c(weights.s_rel2)
    _lib.call("h3b200_fused_gated_mlp_swiglu_w4a8", x2.data_ptr(), ldx, q1.data_ptr(), sr1.data_ptr(),
              sc1.data_ptr(), _ptr(cb1), _ptr(weights.b1), q2.data_ptr(), sr2.data_ptr(), sc2.data_ptr(), _ptr(cb2),
              _ptr(weights.b2), code, gsz, g.data_ptr(), ldg, _ptr(row_map), r2.data_ptr(), ldr, o2.data_ptr(), ldo,
              m, d, ffn, chunk, workspace.data_ptr(), workspace.numel(), _stream(hidden))
    return out


def w4a8_int8_linear(x: torch.Tensor, qdata: torch.Tensor, s_rel: torch.Tensor, s_channel: torch.Tensor,
                     codebook: torch.Tensor | None = None, correction: torch.Tensor | None = None,
                     bias: torch.Tensor | None = None, group_size: int = 16, convrot_groupsize: int = 256,
                     out_dtype: torch.dtype = torch.bfloat16, grid: torch.Tensor | None = None,
                     input_act=None) -> torch.Tensor:
    """W4A8 linear (``comfy_kitchen`` w4a8_int8_linear, tensor/w4a8_int8.py:89-115; CUDA
    backends/cuda/__init__.py:2139-2298): ConvRot-quantize x, INT8 GEMM against
    the decoded int8 grid, dequant by ``s_channel`` (+ bias, rounded to bf16), then the
    asymmetric group correction (``correction`` given; for symmetric weights the call is
    ``int8_linear(x, grid, s_channel, bias, convrot=True)``, eager/w4a8_int8.py:494-508).
    ``s_rel`` fp32 or float8_e4m3fn; ``codebook`` the 16 levels of the H3 release format.

    ``grid`` is the decoded weight from :func:`dequant_int4_grouped_to_int8`;
    pass it to keep the decode out of the per-call path (weights are static). Without it
    the packed weight goes to ``h3b200_w4a8_int8_linear_packed``: for up to 256 rows the
    GEMM unpacks the int4 weight to int8 in shared memory tile by tile (the weight crosses
    HBM at 4 bits), for more rows it is decoded once into a workspace grid."""
    _need_cuda(x, qdata, s_rel, s_channel)
    if out_dtype != torch.bfloat16 or x.dtype != torch.bfloat16:
        raise NotImplementedError("h3b200 builds bf16 activations and outputs only")
    n, kh = qdata.shape
    k = kh * 2
    if _act_k(x, input_act) != k:
        raise ValueError(f"Input K={_act_k(x, input_act)} (after input_act) does not match qdata K={k}")
    groups = k // group_size
    corr = None
    if correction is not None:
        if tuple(correction.shape) != (groups, n):
            raise ValueError(f"correction must have shape {(groups, n)}, got {tuple(correction.shape)}")
        corr = correction.to(torch.bfloat16).contiguous()
    b = None
    if bias is not None:
        b = bias.to(torch.bfloat16).contiguous().reshape(-1)
        if b.numel() != n:
            raise ValueError(f"bias must have {n} elements, got {b.numel()}")
    sch = s_channel.to(torch.float32).contiguous()
    if tuple(sch.shape) != (n,):
        raise ValueError(f"s_channel must have shape {(n,)}, got {tuple(sch.shape)}")
    x2, ldx = _rows(x)
    m = x2.shape[0]
    out = torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    if grid is None:
        code = _s_rel_code(s_rel)
        sr = s_rel.contiguous()
        if tuple(sr.shape) != (n, groups):
            raise ValueError(f"s_rel must have shape {(n, groups)}, got {tuple(sr.shape)}")
        cb = _codebook(codebook, x.device)
        qd = qdata.contiguous()
        nbytes = int(_lib.load().h3b200_w4a8_linear_packed_workspace_bytes(m, n, k, group_size))
        work = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
        _lib.call("h3b200_w4a8_int8_linear_packed", x2.data_ptr(), ldx, qd.data_ptr(), sr.data_ptr(), code, _ptr(cb),
                  sch.data_ptr(), _ptr(corr), _ptr(b), group_size, convrot_groupsize, input_act_code(input_act),
                  out.data_ptr(), m, n, k, work.data_ptr(), nbytes, _stream(x))
        return out.reshape(*x.shape[:-1], n)
    nbytes = int(_lib.load().h3b200_w4a8_linear_workspace_bytes(m, n, k, group_size))
    work = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    _lib.call("h3b200_w4a8_int8_linear", x2.data_ptr(), ldx, grid.contiguous().data_ptr(), sch.data_ptr(), _ptr(corr),
              _ptr(b), group_size, convrot_groupsize, input_act_code(input_act), out.data_ptr(), m, n, k,
              work.data_ptr(), nbytes, _stream(x))
    return out.reshape(*x.shape[:-1], n)
