"""ctypes binding of ``libh3b200.so`` (the C ABI declared in ``include/h3b200.h``).

The library is loaded from this directory. There is no fallback: if the library
is missing or a call returns a non-zero status, a ``RuntimeError`` (or
``ValueError`` for contract violations) is raised with the library's message.
"""

from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libh3b200.so")

OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_LAUNCH, ERR_DEVICE = 0, 1, 2, 3, 4
STATUS_SELFTEST = 0x7E57
ACT_NONE, ACT_GELU_TANH, ACT_SWIGLU = 0, 1, 2
DTYPE_F32, DTYPE_F16, DTYPE_BF16, DTYPE_I32 = 0, 1, 2, 3

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float

# name -> (restype, argtypes); mirrors include/h3b200.h
SIGNATURES = {
    "h3b200_version": (ctypes.c_char_p, []),
    "h3b200_last_error": (ctypes.c_char_p, []),
    "h3b200_device_status": (_i32, [_i32, ctypes.POINTER(ctypes.c_uint), _i32]),
    "h3b200_device_status_nowait": (_i32, [_i32, ctypes.POINTER(ctypes.c_uint)]),
    "h3b200_selftest_expire_wait": (_i32, [_i64, _p]),
    "h3b200_apply_input_act": (_i32, [_p, _p, _i64, _i32, _p]),
    "h3b200_swiglu": (_i32, [_p, _i64, _p, _i64, _i64, _i64, _p]),
    "h3b200_quantize_int8_rowwise": (_i32, [_p, _i64, _i64, _i64, _i32, _p, _p, _p]),
    "h3b200_quantize_int8_rowwise_stochastic": (_i32, [_p, _i64, _i64, _i64, _i32, _i64, _p, _p, _p]),
    "h3b200_quantize_int8_rowwise_f16": (_i32, [_p, _i64, _i64, _i64, _p, _p, _p]),
    "h3b200_quantize_int8_rowwise_absmax": (_i32, [_p, _p, _i64, _i64, _i64, _p, _p, _p]),
    "h3b200_int8_mm": (_i32, [_p, _p, _i64, _i64, _i64, _p, _p]),
    "h3b200_int8_linear_prequantized": (_i32, [_p, _p, _p, _p, _i64, _p, _i32, _p, _i64, _i64, _i64, _p]),
    "h3b200_int8_gemm_fused": (_i32, [_p, _i64, _p, _i64, _i64, _i64, _i64, _i32, _p, _p, _i64, _p, _p, _p, _i64, _p,
                                      _i64, _p, _p]),
    "h3b200_requant_gemm_workspace_bytes": (_i64, [_i64, _i64]),
    "h3b200_requant_gemm_gated_residual": (_i32, [_p, _i64, _p, _p, _p, _i64, _p, _p, _i64, _p, _p, _i64, _p, _i64,
                                                  _i64, _i64, _i64, _p, _i64, _p]),
    "h3b200_dequant_gated_residual": (_i32, [_p, _p, _p, _p, _p, _i64, _p, _i64, _i64, _i64, _p]),
    "h3b200_int8_linear_workspace_bytes": (_i64, [_i64, _i64]),
    "h3b200_int8_linear": (_i32, [_p, _i64, _p, _p, _i64, _p, _i32, _p, _i64, _i64, _i64, _p, _i64, _p]),
    "h3b200_int8_linear_noalloc_max_scratch_bytes": (_i64, []),
    "h3b200_int8_linear_noalloc": (_i32, [_p, _i64, _p, _p, _i64, _p, _i32, _p, _i64, _i64, _i64, _p]),
    "h3b200_fused_gated_mlp_workspace_bytes": (_i64, [_i64, _i64, _i64]),
    "h3b200_fused_gated_mlp": (_i32, [_p, _i64, _p, _p, _p, _p, _p, _p, _i64, _p, _i64, _i64, _i64, _i64, _i32,
                                      _p, _i64, _p]),
    "h3b200_fused_gated_mlp_segmented": (_i32, [_p, _i64, _p, _p, _p, _p, _p, _i64, _p, _p, _i64, _p, _i64, _i64,
                                                _i64, _i64, _i32, _p, _i64, _p]),
    "h3b200_rms_adaln": (_i32, [_p, _i64, _p, _p, _i64, _p, _i64, _i64, _p, _i64, _f32, _p, _i64, _i64, _i64, _p]),
    "h3b200_adaln_rms_rope_segmented": (_i32, [_p, _i64, _p, _i64, _p, _i64, _p, _i64, _p, _p, _p, _p, _i64, _p,
                                               _i64, _i64, _p, _i64, _i64, _i64, _i64, _i64, _f32, _p]),
    "h3b200_adaln_rms_rope": (_i32, [_p, _i64, _p, _i64, _p, _i64, _p, _i64, _p, _p, _p, _p, _p, _i64, _i64, _i64,
                                     _i64, _i32, _f32, _p]),
    "h3b200_dequant_int4_grouped_to_int8": (_i32, [_p, _p, _i64, _i64, _i64, _p, _p]),
    "h3b200_qkv_qknorm_rope_workspace_bytes": (_i64, [_i64, _i64, _i64, _i32, _i32]),
    "h3b200_qkv_qknorm_rope": (_i32, [_p, _p, _i64, _i64, _p, _p, _i64, _p, _i64, _i64, _i32, _i32, _p, _p, _p, _i32,
                                      _i64, _i64, _i64, _f32, _p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _p,
                                      _i64, _p]),
    "h3b200_qknorm_rope_strided": (_i32, [_p, _i64, _i64, _p, _i64, _i64, _p, _p, _i64, _i64, _p, _i64, _i64, _p, _p,
                                          _i32, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _p]),
    "h3b200_quantize_int8_rowwise_convrot": (_i32, [_p, _i64, _i64, _i64, _i64, _i32, _p, _p, _p]),
    "h3b200_w4a8_linear_workspace_bytes": (_i64, [_i64, _i64, _i64, _i64]),
    "h3b200_dequant_int4_grouped_to_int8_ex": (_i32, [_p, _p, _i32, _p, _i64, _i64, _i64, _p, _p]),
    "h3b200_w4a8_int8_linear": (_i32, [_p, _i64, _p, _p, _p, _p, _i64, _i64, _i32, _p, _i64, _i64, _i64, _p, _i64,
                                       _p]),
    "h3b200_w4a8_linear_packed_workspace_bytes": (_i64, [_i64, _i64, _i64, _i64]),
    "h3b200_w4a8_int8_linear_packed": (_i32, [_p, _i64, _p, _p, _i32, _p, _p, _p, _p, _i64, _i64, _i32, _p, _i64,
                                              _i64, _i64, _p, _i64, _p]),
    "h3b200_fused_gated_mlp_w4a8_workspace_bytes": (_i64, [_i64, _i64, _i64, _i64]),
    "h3b200_fused_gated_mlp_swiglu_workspace_bytes": (_i64, [_i64, _i64, _i64]),
    "h3b200_fused_gated_mlp_swiglu": (_i32, [_p, _i64, _p, _p, _i64, _p, _p, _p, _i64, _p, _p, _i64, _p, _p, _i64, _p,
                                             _i64, _i64, _i64, _i64, _i64, _i64, _p, _i64, _p]),
    "h3b200_fused_gated_mlp_w4a8": (_i32, [_p, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _p, _i64, _i64,
                                           _i64, _i64, _i64, _i32, _p, _i64, _p]),
    "h3b200_fused_gated_mlp_swiglu_w4a8_workspace_bytes": (_i64, [_i64, _i64, _i64]),
    "h3b200_fused_gated_mlp_swiglu_w4a8": (_i32, [_p, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i32, _i64, _p,
                                                  _i64, _p, _p, _i64, _p, _i64, _i64, _i64, _i64, _i64, _p, _i64,
                                                  _p]),
    "h3b200_tp_comm_create": (_i32, [_i32, _i32, _i64, _i64, _i64, _i64, ctypes.POINTER(_p), _p]),
    "h3b200_tp_comm_open": (_i32, [_p, _p]),
    "h3b200_tp_comm_link_local": (_i32, [ctypes.POINTER(_p), _i32]),
    "h3b200_tp_comm_destroy": (_i32, [_p]),
    "h3b200_tp_barrier": (_i32, [_p, _p]),
    "h3b200_tp_stage": (_i32, [_p, _i32, _i64, _p, _i64, _p, _i64, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _p]),
    "h3b200_tp_gated_mlp": (_i32, [_p, _p, _i64, _p, _i64, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _p]),
}

TP_HANDLE_BYTES = 192
STATUS_TP_BARRIER = 0x201

_lock = threading.Lock()
_lib = None


def load(path: str | None = None) -> ctypes.CDLL:
    """Load the shared library (once). Raises if it is missing."""
    global _lib
    with _lock:
        if _lib is None:
            p = path or LIB_PATH
            if not os.path.exists(p):
                raise RuntimeError(
                    f"h3b200: {p} is missing; build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                    "(there is no CPU fallback)")
            lib = ctypes.CDLL(p)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    if status == OK:
        return
    msg = load().h3b200_last_error().decode(errors="replace")
    if status == ERR_INVALID:
        raise ValueError(f"{what}: {msg}")
    if status == ERR_UNSUPPORTED:
        raise NotImplementedError(f"{what}: {msg}")
    raise RuntimeError(f"{what}: status {status}: {msg}")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


def device_status(device: int, clear: bool = False) -> int:
    v = ctypes.c_uint(0)
    check(load().h3b200_device_status(device, ctypes.byref(v), 1 if clear else 0), "h3b200_device_status")
    return int(v.value)


def device_status_nowait(device: int) -> int:
    """Status word as last written to its mapped host copy (no synchronisation)."""
    v = ctypes.c_uint(0)
    check(load().h3b200_device_status_nowait(device, ctypes.byref(v)), "h3b200_device_status_nowait")
    return int(v.value)


def check_device(device: int, what: str) -> None:
    """Raise if a bounded wait on ``device`` has expired. Reads the mapped host copy
    of the status word, so call it after synchronising with the work to check.

    Called at the sync points of the host pipeline and the bench, so a failure
    inside a kernel is never reported as a result."""
    code = device_status_nowait(device)
    if code:
        raise RuntimeError(f"{what}: a bounded device wait expired on device {device} (status {code:#x}); "
                           "outputs since then are not valid")
