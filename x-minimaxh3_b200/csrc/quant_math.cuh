// Row-quantization arithmetic shared by the quantizer kernels (plain and
// ConvRot): the reference's q = clamp(rne(bf16(x / bf16(scale))), -128, 127)
// (backends/eager/quantization.py:815-826, 857-875) evaluated with a
// correctly rounded reciprocal (which rounds like the division on every bf16
// operand pair; the argument is in quantize.cu), on packed f32x2 / bf16x2
// operations.
#pragma once

#include "common.cuh"

namespace h3 {

// The stored per-row scale: max(absmax / 127, 1e-30) in fp32
__device__ __forceinline__ float row_scale(float rowmax) { return fmaxf(__fdiv_rn(rowmax, 127.0f), 1e-30f); }

// bf16(scale) as the divisor, with torch.finfo(bf16).tiny for a zero
__device__ __forceinline__ float quant_divisor(float scale) {
  float sb = bf16_round(scale);
  return sb == 0.0f ? 1.17549435e-38f : sb;
}

// ---- packed helpers (sm_100: f32x2 and bf16x2 arithmetic) ----
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_dup(float v) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %1};" : "=l"(r) : "f"(v));
  return r;
}
__device__ __forceinline__ uint64_t bf16x2_to_f2(uint32_t w) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(w << 16), "r"(w & 0xFFFF0000u));
  return r;
}
__device__ __forceinline__ void f2_bits(uint64_t v, uint32_t& lo, uint32_t& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=r"(lo), "=r"(hi) : "l"(v));
}
__device__ __forceinline__ uint32_t bf16x2_from_bits(uint32_t lo, uint32_t hi) {  // round to nearest even
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "r"(hi), "r"(lo));
  return r;
}
__device__ __forceinline__ uint32_t bf16x2_clamp_i8(uint32_t b) {  // clamp both halves to [-128, 127]
  uint32_t r;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(b), "r"(0xC300C300u));
  asm("min.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(r), "r"(0x42FE42FEu));
  return r;
}

// 8 bf16 (one 16-byte vector) -> 8 int8 packed in a uint2, for r = rcp_rn(sb).
// Per pair: packed product, bf16x2 rounding and clamp, then round-to-nearest-
// even to an integer by adding 1.5 * 2^23 (the integer lands in the low byte
// of the sum).
__device__ __forceinline__ uint2 quant_vec8(const uint4& v, float r) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  const uint64_t r2 = f2_dup(r);
  const uint64_t magic = f2_dup(12582912.0f);  // 1.5 * 2^23
  uint32_t q[8];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    uint32_t t0, t1;
    f2_bits(f2_mul(bf16x2_to_f2(w[e]), r2), t0, t1);
    const uint32_t b = bf16x2_clamp_i8(bf16x2_from_bits(t0, t1));
    f2_bits(f2_add(bf16x2_to_f2(b), magic), q[2 * e], q[2 * e + 1]);
  }
  const uint32_t lo = __byte_perm(__byte_perm(q[0], q[1], 0x0040), __byte_perm(q[2], q[3], 0x0040), 0x5410);
  const uint32_t hi = __byte_perm(__byte_perm(q[4], q[5], 0x0040), __byte_perm(q[6], q[7], 0x0040), 0x5410);
  return make_uint2(lo, hi);
}

}  // namespace h3
