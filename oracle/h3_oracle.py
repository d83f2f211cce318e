"""NumPy restatement of X-MinimaxH3's quantized DiT-block hot path.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``). Every function restates
the reference eager algorithm (comfy_kitchen 0.2.28 vendored at
``backends/turbo/vendor/comfy_kitchen``; paths below are relative to that
directory unless they start with ``h3serve/``) with explicit IEEE fp32 and bf16
round-to-nearest-even steps, so the result is a deterministic function of the
inputs and does not depend on the host CPU's vector width.

bf16 tensors are carried as ``uint16`` bit patterns; ``bf16_to_f32`` and
``f32_to_bf16`` convert. Integer work (int8 quantization, int32 accumulators)
is exact. Floating work reproduces the reference operation order; the only
places where the reference itself is not a pure function of IEEE arithmetic are
documented where they occur:

* ``torch.nn.functional.gelu(approximate="tanh")`` on CPU evaluates tanh with
  SLEEF ``tanhf_u10`` (torch 2.11 ATen ``GeluKernel`` vector path), which is
  faithfully rounded and saturates to +-1 above |x| > 8.664339742. The oracle
  uses a double-precision tanh rounded to fp32 plus the same saturation; the
  golden table ``tests/golden/gelu_tanh_bf16_all.npz`` pins it on all 65,536
  bf16 inputs.
* ``torch.nn.functional.silu`` (the gate of ``input_act="swiglu"``) on CPU
  evaluates ``x / (1 + exp(-x))`` in fp32 with SLEEF ``expf_u10``. The oracle
  uses a double-precision exp rounded to fp32; ``tests/golden/silu_bf16_all.npz``
  pins it on all 65,536 bf16 inputs.
* ``torch.nn.functional.rms_norm`` sums x^2 in fp32 in an ISA-dependent order.
  The oracle sums in float64 and rounds the mean to fp32 once (error below the
  reference's own), so rare last-bit differences against the reference remain
  and are checked under the float tolerance.
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "bf16_to_f32",
    "f32_to_bf16",
    "quantize_int8_rowwise",
    "quantize_int8_rowwise_given_absmax",
    "quantize_int8_rowwise_stochastic",
    "quantize_int8_rowwise_f16",
    "dequant_epilogue_f16",
    "int8_linear_f16",
    "stochastic_noise_bf16",
    "gelu_tanh_bf16",
    "silu_bf16",
    "swiglu_bf16",
    "apply_input_act",
    "int8_matmul_accumulate",
    "dequant_epilogue",
    "int8_linear",
    "gated_residual",
    "w8a8_gelu_mlp",
    "swiglu_mlp",
    "rms_norm_row",
    "rms_adaln",
    "rms_adaln_rows",
    "rms_norm_noaffine",
    "rope_split_half",
    "adaln_rms_rope",
    "rms_rope_split_half",
    "rope_axis_inv_freq",
    "rope_grid_table",
    "build_hadamard",
    "rotate_activation",
    "f64_to_bf16",
    "decode_int4_grouped_to_int8",
    "e4m3_to_f32",
    "w4a8_symmetric_linear",
    "w4a8_swiglu_mlp",
    "w4a8_int8_linear_quantized",
    "w4a8_quantize_weight",
    "GELU_TANH_SATURATION",
]

F32 = np.float32

# ---------------------------------------------------------------------------
# bf16 <-> fp32
# ---------------------------------------------------------------------------


def bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    """Widen bf16 bit patterns (uint16) to fp32 exactly."""
    u16 = np.ascontiguousarray(u16, dtype=np.uint16)
    return (u16.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(f: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 (round-to-nearest-even), returning uint16 bit patterns.

    Same rounding as torch's ``c10::BFloat16`` conversion (NaN -> 0x7FC0)."""
    f = np.ascontiguousarray(f, dtype=np.float32)
    u = f.view(np.uint32)
    # uint32 arithmetic: only NaN patterns (patched below) can wrap
    r = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(f)
    if nan.any():
        r[nan] = 0x7FC0
    return r


def _bf16_round(f: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 -> fp32 (the value a bf16 store leaves behind)."""
    return bf16_to_f32(f32_to_bf16(f))


# ---------------------------------------------------------------------------
# (a) per-token absmax INT8 quantizer
# ---------------------------------------------------------------------------


def _quantize_rows(xf: np.ndarray, absmax: np.ndarray):
    # scale = (absmax.float() / 127).clamp(min=1e-30)      eager/quantization.py:872
    scale = np.maximum((absmax.astype(np.float32) / F32(127.0)).astype(np.float32), F32(1e-30))
    scale = scale.astype(np.float32)
    # _int8_scale_for_math: scale.to(x.dtype), 0 -> tiny      eager/quantization.py:815-818
    sb = _bf16_round(scale)
    sb = np.where(sb == 0, np.float32(np.finfo(np.float32).tiny), sb).astype(np.float32)
    # x / scale in bf16 (fp32 divide, bf16 store), then round_() + clamp_()   :821-826, :874
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        quo = _bf16_round((xf / sb).astype(np.float32))
    q = np.clip(np.rint(quo), -128.0, 127.0).astype(np.int8)
    return q, scale


def quantize_int8_rowwise(x_bf16: np.ndarray):
    """Per-row absmax INT8 quantization.

    Follows ``quantize_int8_rowwise`` eager/quantization.py:857-875 (CUDA twin
    backends/cuda/ops/int8_linear.cu:157-200): row absmax in bf16 (exact),
    ``scale = max(absmax/127, 1e-30)`` in fp32, quotient ``x / bf16(scale)``
    stored as bf16, round-half-even, clamp to [-128, 127].

    Returns (int8 [..., K], fp32 scale [..., 1]).
    """
    xf = bf16_to_f32(x_bf16)
    absmax = np.abs(xf).max(axis=-1, keepdims=True) if xf.shape[-1] else np.zeros(xf.shape[:-1] + (1,), np.float32)
    return _quantize_rows(xf, absmax)


def quantize_int8_rowwise_f16(x_f16: np.ndarray):
    """Per-row absmax INT8 quantization of an fp16 activation (numpy float16 array).

    The same eager code (eager/quantization.py:815-826, 857-875) with x in fp16: the
    row absmax in fp16 (exact), ``scale = max(absmax/127, 1e-30)`` in fp32, the divisor
    ``scale.to(fp16)`` with ``finfo(fp16).tiny`` (2^-14) for a zero, the quotient formed
    in fp32 and stored as fp16, round-half-even, clamp to [-128, 127]."""
    xf = np.asarray(x_f16, np.float16).astype(np.float32)
    absmax = np.abs(xf).max(axis=-1, keepdims=True) if xf.shape[-1] else np.zeros(xf.shape[:-1] + (1,), np.float32)
    scale = np.maximum((absmax / F32(127.0)).astype(np.float32), F32(1e-30)).astype(np.float32)
    with np.errstate(over="ignore"):
        sh = scale.astype(np.float16).astype(np.float32)
    sh = np.where(sh == 0, np.float32(np.finfo(np.float16).tiny), sh).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        quo = (xf / sh).astype(np.float32).astype(np.float16).astype(np.float32)
    q = np.clip(np.rint(quo), -128.0, 127.0).astype(np.int8)
    return q, scale


def quantize_int8_rowwise_given_absmax(x_bf16: np.ndarray, absmax: np.ndarray):
    """Quantizer body with a precomputed row absmax (fp32 [..., 1]).

    Same arithmetic as ``quantize_int8_rowwise``; the fused MLP computes the
    absmax inside the fc1 epilogue and quantizes fc2's input with it."""
    return _quantize_rows(bf16_to_f32(x_bf16), np.asarray(absmax, np.float32))


def _pcg_hash_u32(x: np.ndarray) -> np.ndarray:
    """PCG-based integer hash (Jarzynski & Olano, JCGT 2020) on uint32 arrays, the
    ``pcg_hash`` of backends/cuda/ops/int8_linear.cu:78-82."""
    x = np.asarray(x, dtype=np.uint32)
    state = x * np.uint32(747796405) + np.uint32(2891336453)
    word = ((state >> ((state >> np.uint32(28)) + np.uint32(4))) ^ state) * np.uint32(277803737)
    return (word >> np.uint32(22)) ^ word


def stochastic_noise_bf16(idx: np.ndarray, seed: int) -> np.ndarray:
    """Noise of element ``idx`` for stochastic rounding (fp32 value of a bf16 in [0, 1]):
    ``bf16(float(pcg_hash(lo32(idx + seed) ^ hi32(idx + seed)) >> 8) * 2^-24)``,
    ``stochastic_rng_value`` backends/cuda/ops/int8_linear.cu:84-90."""
    key = np.asarray(idx, dtype=np.uint64) + np.uint64(seed)
    folded = ((key & np.uint64(0xFFFFFFFF)) ^ (key >> np.uint64(32))).astype(np.uint32)
    u = (_pcg_hash_u32(folded) >> np.uint32(8)).astype(np.float32) * np.float32(2.0 ** -24)
    return _bf16_round(u.astype(np.float32))


def quantize_int8_rowwise_stochastic(x_bf16: np.ndarray, seed: int):
    """``quantize_int8_rowwise(x, stochastic_rounding=seed)`` for seed > 0 on [M, K] bf16.

    Row scale as ``quantize_int8_rowwise`` (eager/quantization.py:870-873); then the
    rounding of the reference's CUDA kernel (backends/cuda/ops/int8_linear.cu:186-193,
    noise :84-90): ``q = clamp(floor(bf16(bf16(x / bf16(scale)) + u)), -128, 127)`` with
    ``u`` the counter-based noise of element ``row * K + col``. (The eager branch,
    eager/quantization.py:821-826, adds ``torch.rand`` noise from a seeded generator,
    which is device-specific; the CUDA kernel's noise is a function of the index.)
    Parity unpinned: the reference's CUDA kernel cannot be built or run here.
    Returns (int8 [M, K], fp32 scale [M, 1])."""
    xf = bf16_to_f32(x_bf16)
    m, k = xf.shape
    absmax = np.abs(xf).max(axis=-1, keepdims=True) if k else np.zeros((m, 1), np.float32)
    scale = np.maximum((absmax.astype(np.float32) / F32(127.0)).astype(np.float32), F32(1e-30)).astype(np.float32)
    sb = _bf16_round(scale)
    sb = np.where(sb == 0, np.float32(np.finfo(np.float32).tiny), sb).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        quo = _bf16_round((xf / sb).astype(np.float32))
        u = stochastic_noise_bf16(np.arange(m * k, dtype=np.uint64).reshape(m, k), seed)
        v = np.floor(_bf16_round((quo + u).astype(np.float32)))
    # fminf(127, fmaxf(-128, v)): a NaN becomes -128, as in the CUDA kernel
    q = np.fmin(np.fmax(v, np.float32(-128.0)), np.float32(127.0)).astype(np.int8)
    return q, scale


# ---------------------------------------------------------------------------
# tanh-GELU on bf16 (input_act="gelu_tanh")
# ---------------------------------------------------------------------------

GELU_TANH_SATURATION = F32(8.664339742)
_GELU_BETA = F32(np.sqrt(2.0) * (2.0 / np.sqrt(np.pi)) * 0.5)
_GELU_KAPPA = F32(0.044715)


def gelu_tanh_bf16(x_bf16: np.ndarray) -> np.ndarray:
    """tanh-GELU of bf16 values, returned as bf16 bits.

    ``apply_input_act(x, "gelu_tanh")`` backends/_activations.py:40-53 calls
    ``torch.nn.functional.gelu(x, approximate="tanh")``. On a bf16 CPU tensor
    torch 2.11 (ATen ``GeluKernel``, tanh branch, reduced-float path) computes in
    fp32, left to right, without fused multiply-add::

        cube  = (x * x) * x
        inner = beta * (x + kappa * cube)        beta = f32(sqrt(2)*2/sqrt(pi)*0.5)
        out   = (0.5 * x) * (1 + tanh(inner))    kappa = f32(0.044715)

    and stores bf16. tanh is SLEEF ``tanhf_u10``: faithfully rounded, exactly
    +-1 for |inner| > 8.664339742. Restated with a double tanh rounded to fp32.
    """
    x = bf16_to_f32(x_bf16)
    with np.errstate(all="ignore"):
        cube = ((x * x).astype(np.float32) * x).astype(np.float32)
        inner = (_GELU_BETA * (x + (_GELU_KAPPA * cube).astype(np.float32)).astype(np.float32)).astype(np.float32)
        t = np.tanh(inner.astype(np.float64)).astype(np.float32)
        t = np.where(np.abs(inner) > GELU_TANH_SATURATION, np.copysign(F32(1.0), inner), t).astype(np.float32)
        out = ((F32(0.5) * x).astype(np.float32) * (F32(1.0) + t).astype(np.float32)).astype(np.float32)
    return f32_to_bf16(out)


def silu_bf16(x_bf16: np.ndarray) -> np.ndarray:
    """SiLU of bf16 values, returned as bf16 bits.

    ``apply_input_act(x, "swiglu")`` backends/_activations.py:50-52 calls
    ``torch.nn.functional.silu(gate)``; on a bf16 CPU tensor torch 2.11 (ATen silu
    kernel, reduced-float path) computes ``x / (1 + exp(-x))`` in fp32 and stores
    bf16. Restated with a double exp rounded to fp32."""
    x = bf16_to_f32(x_bf16)
    with np.errstate(all="ignore"):
        e = np.exp(-x.astype(np.float64)).astype(np.float32)
        d = (F32(1.0) + e).astype(np.float32)
        r = (x / d).astype(np.float32)
    return f32_to_bf16(r)


def swiglu_bf16(x_bf16: np.ndarray) -> np.ndarray:
    """``silu(gate).mul_(up)`` on the ``[gate | up]`` halves of the last dim
    (backends/_activations.py:50-52): bf16 silu, then the bf16 product (exact in
    fp32, rounded once). Returns bf16 bits, half as wide."""
    x = np.asarray(x_bf16, np.uint16)
    k = x.shape[-1] // 2
    s = bf16_to_f32(silu_bf16(x[..., :k]))
    u = bf16_to_f32(x[..., k:2 * k])
    return f32_to_bf16((s * u).astype(np.float32))


def apply_input_act(x_bf16: np.ndarray, input_act) -> np.ndarray:
    """``apply_input_act`` backends/_activations.py:40-53 on bf16 bits."""
    x = np.asarray(x_bf16, np.uint16)
    if input_act in (None, "none"):
        return x
    if input_act == "gelu_tanh":
        return gelu_tanh_bf16(x)
    if input_act == "swiglu":
        return swiglu_bf16(x)
    raise ValueError(f"unsupported input_act {input_act!r}")


# ---------------------------------------------------------------------------
# INT8 GEMM + dequant epilogue
# ---------------------------------------------------------------------------


def int8_matmul_accumulate(a_i8: np.ndarray, w_i8: np.ndarray, row_chunk: int = 4096) -> np.ndarray:
    """int32 accumulators ``A[M,K] @ W[N,K]^T``.

    ``_int8_matmul_accumulate`` eager/quantization.py:749-783 (``torch._int_mm``).
    Evaluated as a float64 GEMM: every partial sum is an integer below 2^53
    (|acc| <= 2^14 * K), so the result is exact whatever the summation order.
    """
    a = np.asarray(a_i8)
    w = np.asarray(w_i8)
    m, k = a.shape
    n = w.shape[0]
    if w.shape[1] != k:
        raise ValueError(f"K mismatch: {k} vs {w.shape[1]}")
    if k > (1 << 24):
        raise ValueError("K too large for the exact float64 accumulation")
    wt = w.astype(np.float64).T.copy()
    out = np.empty((m, n), dtype=np.int32)
    for s in range(0, m, row_chunk):
        out[s:s + row_chunk] = (a[s:s + row_chunk].astype(np.float64) @ wt).astype(np.int32)
    return out


def dequant_epilogue(acc: np.ndarray, x_scale: np.ndarray, w_scale: np.ndarray, bias_bf16=None) -> np.ndarray:
    """``bf16(float(acc) * (x_scale[m] * w_scale[n]))`` (+ bf16 bias).

    eager/quantization.py:1034-1053: the row and channel scales are multiplied
    first (fp32), then the int32 accumulator is converted to fp32 and scaled,
    then stored as bf16; bias is added to the bf16 result in bf16."""
    xs = np.asarray(x_scale, np.float32).reshape(-1, 1)
    ws = np.asarray(w_scale, np.float32).reshape(1, -1)
    s = (xs * ws).astype(np.float32)
    out = _bf16_round((acc.astype(np.float32) * s).astype(np.float32))
    if bias_bf16 is not None:
        out = _bf16_round((out + bf16_to_f32(bias_bf16).reshape(1, -1)).astype(np.float32))
    return f32_to_bf16(out)


def dequant_epilogue_f16(acc: np.ndarray, x_scale: np.ndarray, w_scale: np.ndarray, bias_f16=None) -> np.ndarray:
    """``fp16(float(acc) * (x_scale[m] * w_scale[n]))`` (+ fp16 bias): ``dequant_epilogue``
    with ``out_dtype=float16`` (eager/quantization.py:1034-1053; the bias is converted
    to the output dtype and added in it). Returns numpy float16."""
    xs = np.asarray(x_scale, np.float32).reshape(-1, 1)
    ws = np.asarray(w_scale, np.float32).reshape(1, -1)
    s = (xs * ws).astype(np.float32)
    with np.errstate(over="ignore"):
        out = (acc.astype(np.float32) * s).astype(np.float32).astype(np.float16)
        if bias_f16 is not None:
            b = np.asarray(bias_f16, np.float16).astype(np.float32).reshape(1, -1)
            out = (out.astype(np.float32) + b).astype(np.float32).astype(np.float16)
    return out


def int8_linear_f16(x, w_i8, w_scale, bias=None, out_dtype="float16"):
    """``int8_linear(x, weight, weight_scale, bias, out_dtype)`` with an fp16 activation
    (numpy float16) or a bf16 one (uint16 bits), and an fp16 or bf16 output: the
    quantizer of x's dtype, the int32 GEMM, the epilogue of the output dtype (bias
    converted to it: numpy float16 for fp16, bf16 bits for bf16)."""
    if np.asarray(x).dtype == np.float16:
        q, s = quantize_int8_rowwise_f16(x)
    else:
        q, s = quantize_int8_rowwise(x)
    acc = int8_matmul_accumulate(q, w_i8)
    if out_dtype == "float16":
        return dequant_epilogue_f16(acc, s, w_scale, bias)
    return dequant_epilogue(acc, s, w_scale, bias)


def int8_linear(x_bf16, w_i8, w_scale, bias_bf16=None, input_act=None):
    """``int8_linear(x, weight, weight_scale, bias, bf16, convrot=False, input_act)``.

    eager/quantization.py:971-1056: optional activation on the bf16 input,
    per-row quantization, int32 GEMM, dequant epilogue. Returns bf16 bits."""
    x = apply_input_act(x_bf16, input_act)
    q, s = quantize_int8_rowwise(x)
    acc = int8_matmul_accumulate(q, w_i8)
    return dequant_epilogue(acc, s, w_scale, bias_bf16)


def gated_residual(residual_bf16, y_bf16, gate_bf16):
    """``residual.clone().addcmul_(y, gate)`` in bf16.

    h3serve/native_engine/model/fused_mlp.py:414-425 (``addcmul_`` per segment).
    torch's reduced-float CPU addcmul evaluates ``self + (1*y)*gate`` in fp32
    with separate multiply and add, then stores bf16."""
    r = bf16_to_f32(residual_bf16)
    y = bf16_to_f32(y_bf16)
    g = bf16_to_f32(gate_bf16).reshape(1, -1)
    p = (y * g).astype(np.float32)
    return f32_to_bf16((r + p).astype(np.float32))


def w8a8_gelu_mlp(x_bf16, w1_i8, s1, w2_i8, s2, gate_bf16, residual_bf16, return_intermediates=False):
    """Gated tanh-GELU W8A8 MLP: fc1 -> GELU -> per-token requant -> fc2 -> gated residual.

    Composition of reference operators (``int8_linear`` twice, the second with
    ``input_act="gelu_tanh"``, then ``addcmul_``), as in
    h3serve/native_engine/model/fused_mlp.py:393-425 with the activation
    replaced by tanh-GELU (backends/_activations.py:19-24)."""
    h = int8_linear(x_bf16, w1_i8, s1)
    a = gelu_tanh_bf16(h)
    q2, xs2 = quantize_int8_rowwise(a)
    acc2 = int8_matmul_accumulate(q2, w2_i8)
    y = dequant_epilogue(acc2, xs2, s2)
    out = gated_residual(residual_bf16, y, gate_bf16)
    if return_intermediates:
        return out, {"h": h, "a": a, "q2": q2, "xs2": xs2, "acc2": acc2, "y": y}
    return out


# ---------------------------------------------------------------------------
# (c) AdaLN-modulate + RMSNorm + split-half RoPE
# ---------------------------------------------------------------------------


def swiglu_mlp(x_bf16, w1q, s1, b1_bf16, w2q, s2, b2_bf16, gate_rows_bf16, row_map, residual_bf16,
               fc1_convrot=True, return_intermediates=False):
    """H3 SwiGLU MLP, the INT8 path of ``try_fused_gated_mlp``
    (h3serve/native_engine/model/fused_mlp.py:366-424): ``raw = int8_linear(x, W1, s1, b1,
    convrot=fc1_convrot)``; ``y = int8_linear(raw, W2, s2, b2, convrot=True,
    input_act="swiglu")``; ``out[t] = residual[t] + y[t] * gate[row_map[t]]`` (the
    per-segment ``addcmul_``). ConvRot uses the exact rotation (``rotate_activation``).
    Returns bf16 bits."""
    xr = rotate_activation(x_bf16, 256) if fc1_convrot else np.asarray(x_bf16, np.uint16)
    q1, xs1 = quantize_int8_rowwise(xr)
    raw = dequant_epilogue(int8_matmul_accumulate(q1, w1q), xs1, s1, b1_bf16)
    a = rotate_activation(swiglu_bf16(raw), 256)
    q2, xs2 = quantize_int8_rowwise(a)
    y = dequant_epilogue(int8_matmul_accumulate(q2, w2q), xs2, s2, b2_bf16)
    g = bf16_to_f32(np.asarray(gate_rows_bf16, np.uint16).reshape(-1, y.shape[-1])[np.asarray(row_map)])
    out = f32_to_bf16((bf16_to_f32(residual_bf16) + (bf16_to_f32(y) * g).astype(np.float32)).astype(np.float32))
    if return_intermediates:
        return out, {"raw": raw, "y": y}
    return out


def _rms_rstd(xf: np.ndarray, eps: float) -> np.ndarray:
    ms = (np.square(xf.astype(np.float64)).sum(axis=-1, keepdims=True) / xf.shape[-1]).astype(np.float32)
    v = (ms + F32(eps)).astype(np.float32)
    return (F32(1.0) / np.sqrt(v).astype(np.float32)).astype(np.float32)


def rms_norm_row(x_bf16, weight_bf16, eps=1e-6):
    """``F.rms_norm(x, (D,), weight, eps)`` on bf16.

    torch 2.11 CPU: mean(x^2) in fp32, ``rstd = 1/sqrt(mean + eps)``, result
    ``(x * rstd) * weight`` in fp32, one bf16 store (h3serve/native_engine/model/
    layers.py:43-48; kernels.py:7623). The oracle sums x^2 in float64."""
    xf = bf16_to_f32(x_bf16)
    rstd = _rms_rstd(xf, eps)
    w = bf16_to_f32(weight_bf16)
    return f32_to_bf16(((xf * rstd).astype(np.float32) * w).astype(np.float32))


def rms_norm_noaffine(x_bf16, eps=1e-6):
    """``F.rms_norm(x, (D,), eps=eps)`` without a weight on bf16: ``bf16(x * rstd)``
    (comfy_kitchen backends/eager/adaln.py:17-20)."""
    xf = bf16_to_f32(x_bf16)
    return f32_to_bf16((xf * _rms_rstd(xf, eps)).astype(np.float32))


def rms_adaln_rows(x_bf16, weight_bf16, scale_rows_bf16, shift_rows_bf16, row_map, eps=1e-6):
    """RMS-AdaLN with a modulation row per token.

    H3 ``rms_adaln(value, norm, shift, scale, segments)`` eager branch
    (h3serve/native_engine/model/kernels.py:7623-7634): ``hidden = norm(value)``
    (``F.rms_norm`` with the module weight, layers.py:39-48), then for each segment
    ``hidden[start:stop].mul_(1.0 + scale[row].to(bf16)).add_(shift[row].to(bf16))``.
    ``weight_bf16=None`` is comfy_kitchen's weightless ``rms_adaln``
    (backends/eager/adaln.py:17-20). x: bf16 [M, D]; scale/shift rows: bf16 [R, D];
    row_map: int [M] (the segment row of each token). Returns bf16 bits."""
    if weight_bf16 is None:
        h = bf16_to_f32(rms_norm_noaffine(x_bf16, eps))
    else:
        h = bf16_to_f32(rms_norm_row(x_bf16, weight_bf16, eps))
    rm = np.asarray(row_map, np.int64)
    sc = bf16_to_f32(np.asarray(scale_rows_bf16, np.uint16).reshape(-1, h.shape[-1]))[rm]
    sh = bf16_to_f32(np.asarray(shift_rows_bf16, np.uint16).reshape(-1, h.shape[-1]))[rm]
    one_plus = _bf16_round((F32(1.0) + sc).astype(np.float32))
    h = _bf16_round((h * one_plus).astype(np.float32))
    h = _bf16_round((h + sh).astype(np.float32))
    return f32_to_bf16(h)


def rms_adaln(x_bf16, weight_bf16, scale_bf16, shift_bf16, eps=1e-6):
    """RMSNorm with weight, then ``mul_(1 + scale)``, then ``add_(shift)``, bf16 after each.

    h3serve/native_engine/model/kernels.py:7623-7631 (eager order of ``rms_adaln``):
    ``hidden = norm(value); hidden.mul_(1.0 + scale.to(bf16)).add_(shift.to(bf16))``."""
    h = bf16_to_f32(rms_norm_row(x_bf16, weight_bf16, eps))
    one_plus = _bf16_round((F32(1.0) + bf16_to_f32(scale_bf16)).astype(np.float32))
    h = _bf16_round((h * one_plus).astype(np.float32))
    h = _bf16_round((h + bf16_to_f32(shift_bf16)).astype(np.float32))
    return f32_to_bf16(h)


def rope_split_half(x_bf16, table_f32, rot_dim=0):
    """Split-half RoPE per head.

    ``apply_rope_split_half1`` eager/rope.py:39-42 with the partial-rotary rule
    of ``_rms_rope1`` eager/rope.py:67-92. x: bf16 [M, H, D]; table: fp32
    [M, rot_dim/2, 2, 2] packed ``[[cos, -sin], [sin, cos]]``
    (h3serve/native_engine/model/layers.py:61-69). Pair i couples element i and
    i + rot_dim/2: ``y0 = t00*x0 + t01*x1``, ``y1 = t10*x0 + t11*x1`` in fp32
    (two products, one add), then bf16."""
    x = bf16_to_f32(x_bf16)
    m, h, d = x.shape
    rd = d if rot_dim in (0, d) else rot_dim
    half = rd // 2
    t = np.asarray(table_f32, np.float32).reshape(m, 1, half, 2, 2)
    x0 = x[..., :half]
    x1 = x[..., half:rd]
    y0 = ((t[..., 0, 0] * x0).astype(np.float32) + (t[..., 0, 1] * x1).astype(np.float32)).astype(np.float32)
    y1 = ((t[..., 1, 0] * x0).astype(np.float32) + (t[..., 1, 1] * x1).astype(np.float32)).astype(np.float32)
    out = np.concatenate([y0, y1, x[..., rd:]], axis=-1).astype(np.float32)
    return f32_to_bf16(out)


def adaln_rms_rope(q_bf16, k_bf16, table_f32, q_weight, k_weight, scale, shift, eps=1e-6, norm_span="row", rot_dim=0):
    """Fused AdaLN-modulate + RMSNorm + split-half RoPE on Q and K ([M, H, D] bf16).

    ``norm_span="row"``: ``rms_adaln`` over the H*D row (kernels.py:7586-7634 eager
    order), then per-head RoPE. ``norm_span="head"``: per-head RMSNorm with a
    [D] weight (``rms_rope_split_half``, eager/rope.py:129-143) and the same
    modulation applied per row afterwards when ``scale``/``shift`` are given.
    Returns (q_out, k_out) bf16 bits."""
    outs = []
    for x, w in ((q_bf16, q_weight), (k_bf16, k_weight)):
        m, h, d = x.shape
        if norm_span == "row":
            y = rms_adaln(x.reshape(m, h * d), w, scale, shift, eps).reshape(m, h, d)
        elif norm_span == "head":
            y = rms_norm_row(x, w, eps)
            if scale is not None:
                yf = bf16_to_f32(y).reshape(m, h * d)
                one_plus = _bf16_round((F32(1.0) + bf16_to_f32(scale)).astype(np.float32))
                yf = _bf16_round((yf * one_plus).astype(np.float32))
                yf = _bf16_round((yf + bf16_to_f32(shift)).astype(np.float32))
                y = f32_to_bf16(yf).reshape(m, h, d)
        else:
            raise ValueError(f"norm_span must be 'row' or 'head', got {norm_span!r}")
        outs.append(rope_split_half(y, table_f32, rot_dim))
    return outs[0], outs[1]


def rms_rope_split_half(q_bf16, k_bf16, table_f32, q_weight, k_weight=None, eps=1e-6, rot_dim=0):
    """``rms_rope_split_half(q, k, freqs, q_scale, k_scale, eps, rot_dim)`` eager/rope.py:129-143."""
    if k_weight is None:
        k_weight = q_weight
    return adaln_rms_rope(q_bf16, k_bf16, table_f32, q_weight, k_weight, None, None, eps, "head", rot_dim)


def rope_axis_inv_freq(dim: int, base: float = 10000.0) -> np.ndarray:
    """``1 / base^(arange(0, dim, 2) / dim)`` for one RoPE axis of width ``dim`` (float64, rounded to fp32)."""
    return (1.0 / (base ** (np.arange(0, dim, 2, dtype=np.float64) / dim))).astype(np.float32)


def rope_grid_table(grid, dims=(44, 42, 42), base=10000.0, token_slice=None) -> np.ndarray:
    """Packed split-half rotation table for a (t, h, w) token grid, fp32 [M, sum(dims)/2, 2, 2].

    Positions are the row-major (t, h, w) meshgrid; each axis contributes
    ``pos * inv_freq`` angles (h3serve/native_engine/model/layers.py:51-58, with a
    per-axis frequency width), and the table packs ``[[cos, -sin], [sin, cos]]``
    (layers.py:61-69). ``token_slice`` restricts to a contiguous token range.
    The table is an input to the kernels, not part of their measured work."""
    t, h, w = grid
    m = t * h * w
    lo, hi = (0, m) if token_slice is None else token_slice
    idx = np.arange(lo, hi, dtype=np.int64)
    pos = np.stack([idx // (h * w), (idx // w) % h, idx % w], axis=1).astype(np.float32)
    angs = [pos[:, a:a + 1] * rope_axis_inv_freq(d, base)[None, :] for a, d in enumerate(dims)]
    ang = np.concatenate(angs, axis=1).astype(np.float32)
    c = np.cos(ang.astype(np.float64)).astype(np.float32)
    s = np.sin(ang.astype(np.float64)).astype(np.float32)
    return np.stack([c, -s, s, c], axis=-1).reshape(hi - lo, ang.shape[1], 2, 2).astype(np.float32)


# ---------------------------------------------------------------------------
# W4A8 (asymmetric grouped int4 weights, ConvRot-256 activations)
# ---------------------------------------------------------------------------


def build_hadamard(size: int = 256) -> np.ndarray:
    """Normalized regular Hadamard matrix H4^(x)n / sqrt(size) (tensor/int8_utils.py:11-38)."""
    if size < 4 or size & (size - 1) or (size.bit_length() - 1) % 2:
        raise ValueError(f"Regular Hadamard size must be a power of 4, got {size}")
    h4 = np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=np.float64)
    h = h4
    while h.shape[0] < size:
        h = np.kron(h, h4)
    return h / np.sqrt(size)


def f64_to_bf16(y) -> np.ndarray:
    """Round float64 values to bf16 (round-to-nearest-even, one rounding), uint16 patterns.

    In the fp32 normal range the value is first rounded to fp32 with round-to-odd (the
    dropped bits OR-ed into the last kept bit; 24 bits > 8 + 1, so the following
    nearest-even rounding to bf16 is the correctly rounded one); other values take
    exact integer arithmetic on the binary64 fields: 8 significant bits in the bf16
    normal range, units of 2^-133 below it, inf on overflow, 0x7FC0 for NaN."""
    y = np.ascontiguousarray(y, dtype=np.float64)
    w = y.view(np.uint32).reshape(y.shape + (2,))       # little-endian halves: [..., 0] low, [..., 1] high
    lo, hi = w[..., 0], w[..., 1]
    ef = (hi >> np.uint32(20)) & np.uint32(0x7FF)
    f32 = (hi & np.uint32(0x80000000)) | ((ef - np.uint32(896)) << np.uint32(23)) | \
        ((hi & np.uint32(0xFFFFF)) << np.uint32(3)) | (lo >> np.uint32(29))
    f32 |= ((lo & np.uint32((1 << 29) - 1)) != 0).astype(np.uint32)
    out = f32_to_bf16(f32.view(np.float32))
    slow = np.nonzero((ef < np.uint32(1023 - 126)) | (ef > np.uint32(1023 + 127)))
    if slow[0].size:
        out[slow] = _f64_to_bf16_general(y[slow])
    return out


def _f64_to_bf16_general(y) -> np.ndarray:
    y = np.ascontiguousarray(y, dtype=np.float64)
    u = y.view(np.uint64)
    sign = ((u >> np.uint64(63)) << np.uint64(15)).astype(np.uint64)
    ef = ((u >> np.uint64(52)) & np.uint64(0x7FF)).astype(np.int64)
    frac = (u & np.uint64((1 << 52) - 1)).astype(np.uint64)
    mfull = np.where(ef > 0, frac | np.uint64(1 << 52), frac)        # value = mfull * 2^(max(ef,1) - 1075)
    e_unb = np.maximum(ef, 1) - 1075                                 # weight exponent of mfull's bit 0
    top = np.frexp(mfull.astype(np.float64))[1].astype(np.int64) - 1   # exact: mfull < 2^53
    top = np.where(mfull > 0, top, 0)
    e_top = top + e_unb                                              # weight exponent of the leading bit
    # bf16 keeps bits down to weight 2^(e_top - 7) (normal) or 2^-133 (subnormal)
    keep_w = np.where(e_top >= -126, e_top - 7, -133)
    shift = keep_w - e_unb                                           # bits of mfull dropped (can be <= 0)
    # mfull < 2^53, so a drop of 54 or more bits leaves less than half a unit: zero
    sh = np.clip(shift, 0, 54).astype(np.uint64)
    q = np.where(shift >= 54, np.uint64(0), mfull >> sh)
    rem = mfull & ((np.uint64(1) << sh) - np.uint64(1))
    half = np.where(shift > 0, np.uint64(1) << np.clip(shift - 1, 0, 53).astype(np.uint64), np.uint64(0))
    up = (shift > 0) & (shift < 54) & ((rem > half) | ((rem == half) & ((q & np.uint64(1)) == 1)))
    q = np.where(shift < 0, mfull << np.clip(-shift, 0, 63).astype(np.uint64), q) + up.astype(np.uint64)
    normal = e_top >= -126
    e_out = np.where(normal & (q == 256), e_top + 1, e_top)
    q = np.where(normal & (q == 256), np.uint64(128), q)
    bits = np.where(normal, ((e_out + 127).astype(np.uint64) << np.uint64(7)) | (q & np.uint64(0x7F)), q)
    bits = np.where(normal & (e_out + 127 >= 255), np.uint64(0x7F80), bits)
    bits = np.where(mfull == 0, np.uint64(0), bits)
    bits = np.where(ef == 0x7FF, np.uint64(0x7F80), bits)
    r = (bits | sign).astype(np.uint16)
    nan = np.isnan(y)
    if nan.any():
        r[nan] = 0x7FC0
    return r


def _bf16_from_fraction(v) -> int:
    """Correctly rounded bf16 (RNE) of an exact rational value, as a bit pattern."""
    from fractions import Fraction

    if v == 0:
        return 0
    sign = 0x8000 if v < 0 else 0
    a = -v if v < 0 else v
    e = a.numerator.bit_length() - a.denominator.bit_length()
    while Fraction(2) ** e > a:
        e -= 1
    while Fraction(2) ** (e + 1) <= a:
        e += 1
    lsb = e - 7 if e >= -126 else -133
    scaled = a / Fraction(2) ** lsb
    q, r = divmod(scaled.numerator, scaled.denominator)
    r2 = 2 * r
    if r2 > scaled.denominator or (r2 == scaled.denominator and q & 1):
        q += 1
    if e >= -126:
        if q == 256:
            q, e = 128, e + 1
        if e + 127 >= 255:
            return sign | 0x7F80
        return sign | ((e + 127) << 7) | (q & 0x7F)
    return sign | q


def _rotate_group_exact(xg: np.ndarray) -> np.ndarray:
    """Exact rotation of one 256-group (bf16 bit patterns) with IEEE rules for inf / NaN."""
    from fractions import Fraction

    f = bf16_to_f32(xg).astype(np.float64)
    n = f.shape[0]
    h = np.sign(build_hadamard(n)).astype(np.int64)
    out = np.zeros(n, np.uint16)
    if np.isnan(f).any():
        out[:] = 0x7FC0
        return out
    fin = np.isfinite(f)
    vals = [Fraction(float(v)) for v in np.where(fin, f, 0.0)]
    for j in range(n):
        col = h[:, j]
        pinf = bool(((f == np.inf) & (col > 0)).any() or ((f == -np.inf) & (col < 0)).any())
        ninf = bool(((f == np.inf) & (col < 0)).any() or ((f == -np.inf) & (col > 0)).any())
        if pinf or ninf:
            out[j] = 0x7FC0 if (pinf and ninf) else (0x7F80 if pinf else 0xFF80)
            continue
        tot = sum((vals[i] if col[i] > 0 else -vals[i]) for i in range(n) if fin[i] and f[i] != 0)
        out[j] = _bf16_from_fraction(Fraction(tot) / int(round(n ** 0.5)))   # H = H4^(x)k / sqrt(n), n a power of 4
    return out


def rotate_activation(x_bf16, group_size: int = 256) -> np.ndarray:
    """ConvRot online rotation ``x_grouped @ H`` per group, bf16 out (tensor/int8_utils.py:58-74).

    The reference runs a bf16 matmul with fp32 accumulation in its BLAS order; the
    oracle defines the rotation as the correctly rounded bf16 of the exact sum
    ``sum_i x_i H[i][j]`` (H = H4^(x)4 / 16), which is what the reference's fp32 sums
    approximate. Groups whose float64 sums are exact (exponent spread of the nonzero
    inputs at most 37 bits, |x| < 2^124, finite) are summed in float64 and rounded once;
    the rest are summed exactly with rationals."""
    xb = np.ascontiguousarray(np.asarray(x_bf16, np.uint16))
    k = xb.shape[-1]
    if k % group_size:
        raise ValueError(f"features {k} not divisible by group_size {group_size}")
    g = xb.reshape(-1, group_size)
    x = bf16_to_f32(g).astype(np.float64)
    hm = build_hadamard(group_size)
    y = f64_to_bf16(x @ hm)
    a = (g & 0x7FFF).astype(np.int64)
    fld = a >> 7
    fmax = fld.max(axis=1)
    nz = a != 0
    fmin = np.where(nz, np.maximum(fld, 1), 1 << 20).min(axis=1)
    fmin = np.where(nz.any(axis=1), fmin, fmax)
    exact = (a.max(axis=1) < 0x7D80) & (fmax - np.maximum(fmin, 1) <= 37)
    exact |= ~nz.any(axis=1)
    for r in np.nonzero(~exact)[0]:
        y[r] = _rotate_group_exact(g[r])
    return y.reshape(xb.shape)


def e4m3_to_f32(bits_u8) -> np.ndarray:
    """Widen OCP FP8 E4M3 (``torch.float8_e4m3fn``) bit patterns to fp32 exactly.

    Format definition: sign bit, 4-bit exponent with bias 7, 3-bit mantissa,
    subnormals ``m * 2^-9`` at exponent 0, no infinities, ``S.1111.111`` is NaN."""
    b = np.asarray(bits_u8, np.uint8).astype(np.int64)
    e = (b >> 3) & 0xF
    m = (b & 7).astype(np.float64)
    mag = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.exp2(e - 7.0))
    mag = np.where((b & 0x7F) == 0x7F, np.nan, mag)
    return np.where(b & 0x80, -mag, mag).astype(np.float32)


def decode_int4_grouped_to_int8(qdata_i8, s_rel, group_size: int, codebook=None) -> np.ndarray:
    """Decode packed uint4 to the int8 grid: ``clamp(rne(level(u) * s_rel), -127, 127)``,
    ``level(u) = u - 8`` or ``codebook[u]``.

    ``_dequant_int4_grouped_to_int8`` eager/w4a8_int8.py:344-363 (even column =
    low nibble; ``s_rel`` per (row, group) as fp32, or as fp8-e4m3 given here as its
    uint8 bit patterns and widened exactly); CUDA twin backends/cuda/ops/w4a8_gemm.cu:36-121."""
    p = np.asarray(qdata_i8).view(np.uint8).astype(np.int32)
    n, kh = p.shape
    k = kh * 2
    u = np.empty((n, k), dtype=np.int32)
    u[:, 0::2] = p & 0xF
    u[:, 1::2] = (p >> 4) & 0xF
    s = np.asarray(s_rel)
    s = e4m3_to_f32(s) if s.dtype == np.uint8 else s.astype(np.float32)
    if codebook is None:
        lv = u.astype(np.float32) - F32(8.0)
    else:
        lv = np.asarray(codebook, np.float32)[u]
    vals = (lv.reshape(n, k // group_size, group_size) * s[..., None]).astype(np.float32)
    return np.clip(np.rint(vals), -127, 127).astype(np.int8).reshape(n, k)


def w4a8_symmetric_linear(x_bf16, qdata_i8, s_rel, s_channel, codebook=None, bias_bf16=None, group_size=16,
                          input_act=None):
    """Symmetric W4A8 linear (no correction): the H3 release format.

    ``w4a8_int8_linear`` eager/w4a8_int8.py:494-508: decode the int4 weight to the
    int8 grid, then ``int8_linear(x, grid, s_channel, bias, convrot=True)`` (ConvRot-256
    rotation of the activation, exact here, then row quantization, int32 GEMM,
    dequant, bias). Returns bf16 bits."""
    grid = decode_int4_grouped_to_int8(qdata_i8, s_rel, group_size, codebook)
    xr = rotate_activation(apply_input_act(x_bf16, input_act), 256)
    q, xs = quantize_int8_rowwise(xr)
    return dequant_epilogue(int8_matmul_accumulate(q, grid), xs, s_channel, bias_bf16)


def w4a8_swiglu_mlp(x_bf16, w4, gate_rows_bf16, row_map, residual_bf16, return_intermediates=False):
    """H3 SwiGLU MLP on W4A8 weights: ``_chunked_module_gated_mlp``
    (h3serve/native_engine/model/fused_mlp.py:222-266) with the W4A8 kernel
    binding: ``raw = fc1(x)``, ``y = fc2(silu(gate).mul_(up))``,
    ``out[t] = residual[t] + y[t] * gate[row_map[t]]``. ``w4`` maps ``q1, s_rel1,
    s_ch1, codebook1, b1, q2, ...`` and ``group_size``; per token the result equals
    ``swiglu_mlp`` on the decoded grids."""
    gs = int(w4["group_size"])
    g1 = decode_int4_grouped_to_int8(w4["q1"], w4["s_rel1"], gs, w4.get("codebook1"))
    g2 = decode_int4_grouped_to_int8(w4["q2"], w4["s_rel2"], gs, w4.get("codebook2"))
    return swiglu_mlp(x_bf16, g1, w4["s_ch1"], w4.get("b1"), g2, w4["s_ch2"], w4.get("b2"), gate_rows_bf16,
                      row_map, residual_bf16, fc1_convrot=True, return_intermediates=return_intermediates)


def w4a8_int8_linear_quantized(x_bf16, qdata_i8, s_rel, s_channel, correction_bf16, group_size=128,
                               convrot_groupsize=256, return_intermediates=False, bias_bf16=None):
    """W4A8 linear with quantized activations (the reference's CUDA route).

    backends/cuda/__init__.py:2139-2298 for asymmetric weights: ConvRot-rotate and
    row-quantize x, decode the int4 weight to the int8 grid, int32 GEMM, dequant
    ``bf16(acc * (xs * s_channel))``, then the asymmetric correction
    ``out + bf16(bf16(sum_g xq) * bf16(xs)) @ correction`` (:2294-2297) accumulated
    in fp32 and rounded once. The eager reference (eager/w4a8_int8.py:481-492)
    instead dequantizes the weight to bf16 and runs a bf16 ``F.linear`` on the
    unquantized input; the two agree within the float tolerance. A bias joins the
    dequantized value before the correction (the CUDA route's order: bias in the
    dequant epilogue, then ``out.addmm_``), rounded to bf16 as the linear's bias is."""
    xr = rotate_activation(x_bf16, convrot_groupsize)
    xq, xs = quantize_int8_rowwise(xr)
    wgrid = decode_int4_grouped_to_int8(qdata_i8, s_rel, group_size)
    acc = int8_matmul_accumulate(xq, wgrid)
    out = bf16_to_f32(dequant_epilogue(acc, xs, s_channel, bias_bf16))
    if correction_bf16 is not None:
        m, k = xq.shape
        gs = xq.astype(np.int32).reshape(m, k // group_size, group_size).sum(-1)
        sx = _bf16_round(_bf16_round(gs.astype(np.float32)) * _bf16_round(xs.astype(np.float32)))
        corr = bf16_to_f32(correction_bf16).astype(np.float64)
        out = (out.astype(np.float64) + sx.astype(np.float64) @ corr).astype(np.float32)
    res = f32_to_bf16(out)
    if return_intermediates:
        return res, {"xr": xr, "xq": xq, "xs": xs, "wgrid": wgrid, "acc": acc}
    return res


def w4a8_quantize_weight(w_bf16, group_size=128, convrot_groupsize=256):
    """Asymmetric W4A8 weight preparation (offline), float32 ``s_rel``, no codebook.

    ``quantize_w4a8_int8_weight(symmetric=False, codebook=False,
    scale_dtype=float32)`` eager/w4a8_int8.py:315-341 -> :122-209 (asymmetric
    branch :175-186, ``s_channel``/``s_rel`` :188-191, packing :200-202), after the
    offline ConvRot rotation ``W @ H^T`` per 256-group (tensor/int8_utils.py:41-55,
    a bf16 matmul in the reference; float64 here). Returns
    (qdata int8 [N, K/2], s_rel fp32 [N, K/g], s_channel fp32 [N], correction bf16 [K/g, N])."""
    w = bf16_to_f32(w_bf16).astype(np.float64)
    n, k = w.shape
    hm = build_hadamard(convrot_groupsize)
    wr = bf16_to_f32(f32_to_bf16((w.reshape(n, k // convrot_groupsize, convrot_groupsize) @ hm.T)
                                 .reshape(n, k).astype(np.float32)))
    g = wr.astype(np.float32).reshape(n, k // group_size, group_size)
    mn = g.min(-1, keepdims=True)
    gsc = np.maximum(((g.max(-1, keepdims=True) - mn) / F32(15.0)).astype(np.float32), F32(1e-8))
    u = np.clip(np.rint(((g - mn) / gsc).astype(np.float32)), 0, 15).astype(np.int32)
    shifted = ((u - 8).astype(np.float32) * gsc).astype(np.float32)
    corr = f32_to_bf16((F32(8.0) * gsc + mn).astype(np.float32).squeeze(-1).T.copy())
    s_ch = np.maximum((np.abs(shifted).max(axis=(1, 2)) / F32(127.0)).astype(np.float32), F32(1e-8))
    s_rel = (gsc.squeeze(-1) / s_ch[:, None]).astype(np.float32)
    u = u.reshape(n, k)
    packed = ((u[:, 0::2] & 0xF) | ((u[:, 1::2] & 0xF) << 4)).astype(np.uint8).view(np.int8)
    return packed, s_rel, s_ch.astype(np.float32), corr
