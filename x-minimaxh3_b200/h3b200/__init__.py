"""h3b200: B200-native (sm_100a) quantized DiT-block hot path for X-MinimaxH3.

Public operators mirror the comfy_kitchen backend surface that
``h3serve/native_engine`` and ``backends/turbo`` call (``int8_linear``,
``quantize_int8_rowwise``, ``int8_linear_prequantized``, ``mm_int8``,
``w4a8_int8_linear``, ``rms_rope_split_half(_)``) plus the fused entry points
``fused_gated_mlp`` and ``adaln_rms_rope(_)``, and ``fused_gated_mlp_host`` for
token buffers in host memory (copies overlapped with the MLP). All of them run hand-written CUDA
from ``libh3b200.so`` through its C ABI; there is no other backend.
"""

from . import _lib
from .ops import (  # noqa: F401
    adaln_rms_rope,
    apply_input_act,
    adaln_rms_rope_,
    dequant_int4_grouped_to_int8,
    fused_gated_mlp,
    fused_gated_mlp_swiglu,
    fused_gated_mlp_swiglu_w4a8,
    fused_gated_mlp_w4a8,
    input_act_code,
    input_act_width,
    int8_gemm_fused,
    requant_gemm_gated_residual,
    int8_linear,
    int8_linear_prequantized,
    mm_int8,
    quantize_int8_rowwise,
    quantize_int8_rowwise_absmax,
    quantize_int8_rowwise_convrot,
    rms_adaln,
    rms_adaln_segmented,
    rms_rope_split_half,
    rms_rope_split_half_,
    qknorm_rope_strided_,
    single_qknorm_rope_,
    single_qknorm_rope_to_hnd,
    qkv_qknorm_rope,
    segment_row_map,
    w4a8_int8_linear,
)
from .pipeline import fused_gated_mlp_host  # noqa: F401
from .rope import rope_grid_table  # noqa: F401
from .weights import (  # noqa: F401
    SwiGLUMLPWeights,
    W4A8SwiGLUMLPWeights,
    W4A8MLPWeights,
    W8A8MLPWeights,
    quantize_int8_convrot_weight,
    quantize_int8_weight,
    quantize_w4a8_int8_weight,
    quantize_w4a8_weight,
    rotate_weight,
)

__version__ = "0.1.0"


def library():
    """Load and return the ctypes handle of libh3b200.so (raises if it is missing)."""
    return _lib.load()


def device_status(device: int = 0, clear: bool = False) -> int:
    """Device status word (0 = healthy; non-zero = a bounded wait expired). Synchronises."""
    return _lib.device_status(device, clear)
