// RMSNorm / AdaLN arithmetic shared by the norm kernels (norm_rope.cu, adaln.cu).
//
// RMSNorm: rstd = 1 / sqrt(mean(x^2) + eps) in fp32, with the sum of squares
// accumulated in double so that the fp32 mean is the correctly rounded one (the
// reference, torch's CPU rms_norm, sums in fp32 in an ISA-dependent order).
// |x| becomes a double through two integer operations on its bf16 bits (exact
// for normal values; zero and subnormals become a value below 2^-126 whose
// square cannot change the fp32 mean); a row whose mean is not finite is
// re-summed with exact conversions, so inf and NaN behave as in the reference.
//
// Modulation steps on bf16 operands are single correctly rounded bf16x2
// operations: the fp32 product of two bf16 values is exact, and the fp32 sum of
// two bf16 values rounds to the same bf16 value as their exact sum, so both
// equal the reference's fp32 operation followed by a bf16 rounding.
#pragma once

#include "common.cuh"

namespace h3 {

__device__ __forceinline__ uint32_t bf2_mul(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bf2_add(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// |bf16| of the low / high half of w as a double: exponent rebiased by
// 1023 - 127 = 896, mantissa moved to the top of the double's fraction.
__device__ __forceinline__ double abs_lo_as_double(uint32_t w) {
  return __hiloint2double((int)(((w & 0x7FFFu) << 13) + 0x38000000u), 0);
}
__device__ __forceinline__ double abs_hi_as_double(uint32_t w) {
  return __hiloint2double((int)(((w >> 3) & 0x0FFFE000u) + 0x38000000u), 0);
}

// sum of squares of the 8 bf16 values of v (fast: integer-built doubles)
__device__ __forceinline__ void sumsq8_fast(const uint4& v, double (&acc)[4]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const double a = abs_lo_as_double(w[e]);
    const double b = abs_hi_as_double(w[e]);
    acc[e] = fma(a, a, acc[e]);
    acc[e] = fma(b, b, acc[e]);
  }
}
// the same with exact conversions (inf / NaN aware)
__device__ __forceinline__ void sumsq8_exact(const uint4& v, double (&acc)[4]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const double a = (double)bf16_lo(w[e]);
    const double b = (double)bf16_hi(w[e]);
    acc[e] = fma(a, a, acc[e]);
    acc[e] = fma(b, b, acc[e]);
  }
}

// 1 / sqrt(mean + eps), each step rounded in fp32 as torch's CPU rms_norm does
__device__ __forceinline__ float rms_rstd(float mean_sq, float eps) {
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean_sq, eps)));
}

}  // namespace h3
