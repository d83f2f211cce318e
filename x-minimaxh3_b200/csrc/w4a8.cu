// W4A8 pieces: int4 -> int8 grid decode and the transposed, zero-padded
// correction matrix (the ConvRot-256 activation quantizer, which also emits the
// asymmetric-correction operand sx[m, g] = bf16(bf16(sum_{k in g} q) * bf16(xs)),
// is in convrot.cu). The correction itself, out += sx . corr, is
// accumulated on the tensor cores inside the INT8 GEMM's epilogue (gemm_i8.cu,
// kEpi*Corr).
//
// Reference: comfy_kitchen W4A8 (backends/eager/w4a8_int8.py:344-363 decode;
// backends/cuda/ops/w4a8_gemm.cu:36-90; ConvRot quantizer
// backends/cuda/ops/int8_linear.cu:256-340 / eager quantize_and_rotate_rowwise
// backends/eager/quantization.py:878-895; correction
// backends/cuda/__init__.py:2294-2297).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "quant_math.cuh"
#include "w4_math.cuh"

namespace h3 {
namespace {

// ---------------------------------------------------------------------------
// Decode: q = clamp(rne(level(u) * s), -127, 127) with level(u) = u - 8 or a
// 16-entry fp32 codebook, s the row's group scale (fp32, or fp8-e4m3 bytes),
// even column in the low nibble. The product is one fp32 multiply and the
// rounding is cvt.rni (NaN -> 0), then an integer clamp.
// ---------------------------------------------------------------------------

template <bool E4M3>
__device__ __forceinline__ float group_scale(const void* s_rel, int64_t i) {
  if constexpr (E4M3) return e4m3_to_f32(static_cast<const uint8_t*>(s_rel)[i]);
  else return static_cast<const float*>(s_rel)[i];
}



// Unsigned 32-bit division by a launch constant d >= 1 (round-up method of
// Granlund and Montgomery, "Division by invariant integers using
// multiplication", 1994): l = ceil(log2 d), m = floor(2^32 (2^l - d) / d) + 1,
// q = (t + ((n - t) >> 1)) >> (l - 1) with t = umulhi(m, n); d = 1 is q = n.
struct FastDivU32 {
  uint32_t m = 0;
  int l = 0;
  explicit FastDivU32(uint32_t d = 1) {
    while ((1ull << l) < d) ++l;
    m = l == 0 ? 0u : (uint32_t)(((1ull << 32) * ((1ull << l) - d)) / d + 1);
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    if (l == 0) return n;
    const uint32_t t = __umulhi(m, n);
    return (t + ((n - t) >> 1)) >> (l - 1);
  }
};

// 16 outputs per thread (8 packed bytes, one 16-byte store). Group sizes 4, 8
// or a multiple of 16, so the 16 columns use 4, 2 or 1 group scales (an
// adjacent column pair always shares one). Index arithmetic is 32-bit (the
// launcher guarantees n * k / 16 < 2^31); byte offsets are formed in 64 bits.
//
// Fast path (every scale of the thread and every level within |s| <= 2048,
// |level| <= 8, so |level * s| <= 16384): the codes are spread into bytes
// (even columns = low nibbles, odd = high), each level comes from a byte
// permute (codebook: an index into the shared-memory table; uniform: 2^23 + u
// under exponent byte 0x4B, minus 2^23 + 8), the rounded product with the
// scale plus 1.5 * 2^23 leaves rne(level * s) as 0x4B400000 + n in its bits,
// an integer clamp of those bits to 0x4B400000 +- 127 clamps n, and byte
// permutes pack the low bytes into the output. This
// equals clamp(cvt.rni(level * s)) exactly and keeps the conversions off the
// quarter-rate pipe. Other threads take the exact per-element path
// (NaN -> 0, +-inf -> +-127), so every input decodes as the reference does.
template <bool E4M3, bool CODEBOOK, int PER_SCALE>
__global__ void __launch_bounds__(256) dequant_int4_kernel(const uint8_t* __restrict__ qd,
                                                           const void* __restrict__ s_rel,
                                                           const float* __restrict__ codebook, int n, int k,
                                                           int group, const FastDivU32 div_row,
                                                           const FastDivU32 div_group, int8_t* __restrict__ out) {
  __shared__ float lv_s[16];
  bool levels_ok = true;
  if constexpr (CODEBOOK) {
    float l = 0.0f;
    if (threadIdx.x < 16) {
      l = codebook[threadIdx.x];
      lv_s[threadIdx.x] = l;
    }
    levels_ok = __syncthreads_and(fabsf(l) <= 8.0f) != 0;  // false for NaN too
  }
  const uint32_t per_row = (uint32_t)k >> 4;
  const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (uint32_t)n * per_row) return;
  const uint32_t row = div_row.div(idx);   // idx / per_row
  const uint32_t c16 = (idx - row * per_row) << 4;
  const int64_t sbase = (int64_t)row * (uint32_t)(k / group) + div_group.div(c16);
  constexpr int per_scale = PER_SCALE;   // columns sharing one scale: 16 (group >= 16), 8 or 4
  float s[4];
  s[0] = group_scale<E4M3>(s_rel, sbase);
  s[1] = s[2] = s[3] = s[0];
  if constexpr (per_scale < 16) {
    s[1] = group_scale<E4M3>(s_rel, sbase + 1);
    if constexpr (per_scale < 8) {
      s[2] = group_scale<E4M3>(s_rel, sbase + 2);
      s[3] = group_scale<E4M3>(s_rel, sbase + 3);
    }
  }
  const uint2 pk = __ldg(reinterpret_cast<const uint2*>(qd + (int64_t)row * (k >> 1) + (c16 >> 1)));
  const uint32_t w[2] = {pk.x, pk.y};
  uint32_t o[4];
  const bool fast = levels_ok && fabsf(s[0]) <= 2048.0f && fabsf(s[1]) <= 2048.0f && fabsf(s[2]) <= 2048.0f &&
                    fabsf(s[3]) <= 2048.0f;
  if (fast) {
    uint32_t c[8];  // bytes 0, 1: the int8 of columns 2j and 2j + 1
    const uint8_t* const lv_b = reinterpret_cast<const uint8_t*>(lv_s);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t ev = w[h] & 0x0F0F0F0Fu;          // codes of columns 8h + 2b in byte b
      const uint32_t od = (w[h] >> 4) & 0x0F0F0F0Fu;   // codes of columns 8h + 2b + 1
      const uint32_t ev4 = (w[h] << 2) & 0x3C3C3C3Cu;  // the same codes times 4: byte offsets
      const uint32_t od4 = (w[h] >> 2) & 0x3C3C3C3Cu;  //   into the level table
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int j = 4 * h + b;                       // column pair index
        const float sc = per_scale == 16 ? s[0] : (per_scale == 8 ? s[j >> 2] : s[j >> 1]);
        float l0, l1;
        if constexpr (CODEBOOK) {
          l0 = *reinterpret_cast<const float*>(lv_b + __byte_perm(ev4, 0u, 0x4440u | b));
          l1 = *reinterpret_cast<const float*>(lv_b + __byte_perm(od4, 0u, 0x4440u | b));
        } else {
          // 2^23 + u as a float (code byte into bits 0..7 under exponent byte 0x4B), minus 2^23 + 8
          l0 = __fsub_rn(__uint_as_float(__byte_perm(ev, 0x4B000000u, 0x7540u | b)), 8388616.0f);
          l1 = __fsub_rn(__uint_as_float(__byte_perm(od, 0x4B000000u, 0x7540u | b)), 8388616.0f);
        }
        // scalar intrinsics: the product must round before the magic add (a packed
        // multiply and add may be contracted into a fused multiply-add)
        // bits of rne(v) + 1.5 * 2^23, clamped to 0x4B400000 +- 127 (the low byte is the int8)
        const int r0 = __float_as_int(__fadd_rn(__fmul_rn(l0, sc), 12582912.0f));
        const int r1 = __float_as_int(__fadd_rn(__fmul_rn(l1, sc), 12582912.0f));
        c[j] = __byte_perm((uint32_t)max(0x4B3FFF81, min(0x4B40007F, r0)),
                           (uint32_t)max(0x4B3FFF81, min(0x4B40007F, r1)), 0x0040u);
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) o[q] = __byte_perm(c[2 * q], c[2 * q + 1], 0x5410u);
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) o[q] = 0u;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const uint32_t u = (w[e >> 3] >> (4 * (e & 7))) & 0xFu;
      const float level = CODEBOOK ? lv_s[u] : (float)u - 8.0f;
      const float sc = per_scale == 16 ? s[0] : (per_scale == 8 ? s[e >> 3] : s[e >> 2]);
      o[e >> 2] |= decode_one(level, sc) << (8 * (e & 3));
    }
  }
  *reinterpret_cast<uint4*>(out + (int64_t)row * k + c16) = make_uint4(o[0], o[1], o[2], o[3]);
}

// One output per thread, for buffers without the 8/16-byte alignment above.
template <bool E4M3, bool CODEBOOK>
__global__ void dequant_int4_scalar_kernel(const uint8_t* __restrict__ qd, const void* __restrict__ s_rel,
                                           const float* __restrict__ codebook, int64_t n, int64_t k, int64_t group,
                                           int8_t* __restrict__ out) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * k) return;
  const int64_t row = idx / k, col = idx - row * k;
  const uint32_t u = (qd[row * (k / 2) + col / 2] >> (4 * (col & 1))) & 0xFu;
  const float level = CODEBOOK ? codebook[u] : (float)u - 8.0f;
  out[idx] = (int8_t)decode_one(level, group_scale<E4M3>(s_rel, row * (k / group) + col / group));
}

// corrT[n, kp] = correction[g, n] for g < groups, 0 for groups <= g < kp
__global__ void correction_transpose_kernel(const __nv_bfloat16* __restrict__ corr, int64_t groups, int64_t n,
                                            int64_t kp, __nv_bfloat16* __restrict__ corr_t) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n * kp) return;
  const int64_t col = i / kp, g = i - col * kp;
  corr_t[i] = g < groups ? corr[g * n + col] : __float2bfloat16_rn(0.0f);
}

}  // namespace

cudaError_t launch_dequant_int4(const int8_t* qdata, const void* s_rel, bool s_rel_e4m3, const float* codebook,
                                int64_t n, int64_t k, int64_t group, int8_t* out, cudaStream_t stream) {
  if (n == 0 || k == 0) return cudaSuccess;
  if (k % 16 || group < 4 || k % group || (16 % group && group % 16)) return cudaErrorNotSupported;
  const uint8_t* qd = reinterpret_cast<const uint8_t*>(qdata);
  const bool vec = !(reinterpret_cast<uintptr_t>(qdata) & 7) && !(reinterpret_cast<uintptr_t>(out) & 15) &&
                   n * (k / 16) < (int64_t(1) << 31) && k < (int64_t(1) << 31);
  const int64_t total = vec ? n * (k / 16) : n * k;
  const FastDivU32 drow(vec ? (uint32_t)(k / 16) : 1u), dgrp(vec ? (uint32_t)group : 1u);
  const unsigned grid = (unsigned)((total + 255) / 256);
#define H3_DEQ_V(E, C, P) \
  dequant_int4_kernel<E, C, P><<<grid, 256, 0, stream>>>(qd, s_rel, codebook, (int)n, (int)k, (int)group, drow, dgrp, out)
#define H3_DEQ(E, C)                                                                                    \
  (vec ? (group >= 16 ? H3_DEQ_V(E, C, 16) : (group == 8 ? H3_DEQ_V(E, C, 8) : H3_DEQ_V(E, C, 4)))    \
       : dequant_int4_scalar_kernel<E, C><<<grid, 256, 0, stream>>>(qd, s_rel, codebook, n, k, group, out))
  if (s_rel_e4m3) {
    if (codebook) H3_DEQ(true, true); else H3_DEQ(true, false);
  } else {
    if (codebook) H3_DEQ(false, true); else H3_DEQ(false, false);
  }
#undef H3_DEQ
#undef H3_DEQ_V
  return cudaGetLastError();
}

cudaError_t launch_correction_transpose(const void* corr, int64_t groups, int64_t n, int64_t kp, void* corr_t,
                                        cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  if (groups <= 0 || kp < groups) return cudaErrorNotSupported;
  const int64_t total = n * kp;
  correction_transpose_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(corr), groups, n, kp, static_cast<__nv_bfloat16*>(corr_t));
  return cudaGetLastError();
}

}  // namespace h3
