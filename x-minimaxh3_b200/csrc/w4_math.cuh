// int4 -> int8 weight decode arithmetic of the W4A8 formats, shared by the
// standalone decode kernel (w4a8.cu) and the small-M W4A8 GEMM that unpacks in
// shared memory (gemm_w4.cu).
//
// q = clamp(rne(level(u) * s), -127, 127), level(u) = u - 8 or a 16-entry fp32
// codebook, s the row's group scale (fp32, or fp8-e4m3 bytes); the reference's
// _dequant_int4_grouped_to_int8 (backends/eager/w4a8_int8.py:344-363) and its CUDA
// kernel (backends/cuda/ops/w4a8_gemm.cu:36-90).
#pragma once

#include "common.cuh"

namespace h3 {

// OCP FP8 E4M3 (float8_e4m3fn) -> fp32, exact: exponent bias 7 -> 127 is a
// shift of the 7 magnitude bits by 20 plus 120 << 23; exponent 0 is m * 2^-9;
// S.1111.111 is NaN.
__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {
  const uint32_t mag = b & 0x7Fu;
  float v = mag >= 8u ? __uint_as_float((mag << 20) + (120u << 23)) : (float)mag * 0.001953125f;
  if (mag == 0x7Fu) v = __uint_as_float(0x7FC00000u);
  return (b & 0x80u) ? -v : v;
}

// The exact per-element decode: one fp32 multiply, cvt.rni (NaN -> 0), integer clamp.
__device__ __forceinline__ uint32_t decode_one(float level, float s) {
  const int v = __float2int_rn(__fmul_rn(level, s));
  return (uint32_t)(uint8_t)(int8_t)max(-127, min(127, v));
}

// The decoded byte with |level| <= 8 and |s| <= 2048 (|level * s| <= 16384): the rounded
// product plus 1.5 * 2^23 holds rne(level * s) in its low bits (offset 0x4B400000); an
// integer clamp of those bits to 0x4B400000 +- 127 clamps it. Equal to decode_one there.
// (Scalar intrinsics: the product must round before the add, not fuse into it.)
__device__ __forceinline__ uint32_t decode_fast_bits(float level, float s) {
  const int r = __float_as_int(__fadd_rn(__fmul_rn(level, s), 12582912.0f));
  return (uint32_t)max(0x4B3FFF81, min(0x4B40007F, r));
}

}  // namespace h3
