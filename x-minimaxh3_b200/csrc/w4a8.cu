// W4A8 pieces: int4 -> int8 grid decode, ConvRot-256 rotation + row
// quantization (emitting the asymmetric-correction operand
// sx[m, g] = bf16(bf16(sum_{k in g} q) * bf16(xs))), and the transposed,
// zero-padded correction matrix. The correction itself, out += sx . corr, is
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

namespace h3 {
namespace {

// ---------------------------------------------------------------------------
// Decode: q = clamp(rne(level(u) * s), -127, 127) with level(u) = u - 8 or a
// 16-entry fp32 codebook, s the row's group scale (fp32, or fp8-e4m3 bytes),
// even column in the low nibble. The product is one fp32 multiply and the
// rounding is cvt.rni (NaN -> 0), then an integer clamp.
// ---------------------------------------------------------------------------

// OCP FP8 E4M3 (float8_e4m3fn) -> fp32, exact: exponent bias 7 -> 127 is a
// shift of the 7 magnitude bits by 20 plus 120 << 23; exponent 0 is m * 2^-9;
// S.1111.111 is NaN.
__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {
  const uint32_t mag = b & 0x7Fu;
  float v = mag >= 8u ? __uint_as_float((mag << 20) + (120u << 23)) : (float)mag * 0.001953125f;
  if (mag == 0x7Fu) v = __uint_as_float(0x7FC00000u);
  return (b & 0x80u) ? -v : v;
}

template <bool E4M3>
__device__ __forceinline__ float group_scale(const void* s_rel, int64_t i) {
  if constexpr (E4M3) return e4m3_to_f32(static_cast<const uint8_t*>(s_rel)[i]);
  else return static_cast<const float*>(s_rel)[i];
}

__device__ __forceinline__ uint32_t decode_one(float level, float s) {
  const int v = __float2int_rn(__fmul_rn(level, s));
  return (uint32_t)(uint8_t)(int8_t)max(-127, min(127, v));
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

// ---------------------------------------------------------------------------
// ConvRot-256 + row quantization. One CTA per row; each half-warp rotates one
// 256-group, lane li holding elements 16 li .. 16 li + 15. The regular Hadamard
// H4^(x)4 acts on the four base-4 digits of the in-group index independently
// (y_j = S - 2 v_(3-j), S the sum of the four values on that digit's axis;
// S - 2 v is one fused multiply-add, exact in its product since 2 v is):
// digits 0-1 are lane-local; a transpose through shared memory (each lane then
// holds indices li + 16 e) makes digits 2-3 lane-local. The sums are formed in
// the fixed order (v0 + v1) + (v2 + v3); the 1/16 normalisation is exact. The
// rotated value is rounded to bf16 (the reference's bf16 rotation matmul
// output); once the row absmax is known a second transpose restores the
// contiguous order and the row is quantized exactly like quantize_int8_rowwise,
// with 16-byte stores. The optional correction operand is
// sx[row, g] = bf16(bf16(sum of the int8 over group g) * bf16(xs)).
// Shared memory per warp: 16 rows x 32 floats; half h's 16 values of row r sit
// in 16-byte chunk (4 h + c) ^ (r & 7) of the row, so row-wise 16-byte accesses
// and column-wise 4-byte accesses are both free of bank conflicts.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void h4_digit_lo(float (&v)[16]) {  // digit over index bits 0-1
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const float s = __fadd_rn(__fadd_rn(v[4 * a], v[4 * a + 1]), __fadd_rn(v[4 * a + 2], v[4 * a + 3]));
    const float t0 = __fmaf_rn(-2.0f, v[4 * a + 3], s), t1 = __fmaf_rn(-2.0f, v[4 * a + 2], s);
    const float t2 = __fmaf_rn(-2.0f, v[4 * a + 1], s), t3 = __fmaf_rn(-2.0f, v[4 * a], s);
    v[4 * a] = t0; v[4 * a + 1] = t1; v[4 * a + 2] = t2; v[4 * a + 3] = t3;
  }
}
__device__ __forceinline__ void h4_digit_hi(float (&v)[16]) {  // digit over index bits 2-3
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const float s = __fadd_rn(__fadd_rn(v[b], v[4 + b]), __fadd_rn(v[8 + b], v[12 + b]));
    const float t0 = __fmaf_rn(-2.0f, v[12 + b], s), t1 = __fmaf_rn(-2.0f, v[8 + b], s);
    const float t2 = __fmaf_rn(-2.0f, v[4 + b], s), t3 = __fmaf_rn(-2.0f, v[b], s);
    v[b] = t0; v[4 + b] = t1; v[8 + b] = t2; v[12 + b] = t3;
  }
}
// word address (floats) of (row r, value c) of half h in a warp's transpose tile
__device__ __forceinline__ int tr_addr(int r, int h, int c) {
  return r * 32 + ((((h << 2) + (c >> 2)) ^ (r & 7)) << 2) + (c & 3);
}

constexpr int kCvThreadsMax = 256;

template <int PPW>
__global__ void __launch_bounds__(kCvThreadsMax) quantize_convrot_kernel(const __nv_bfloat16* __restrict__ x,
                                                                         int64_t ldx, int64_t m, int64_t k, int act,
                                                                         int8_t* __restrict__ q,
                                                                         float* __restrict__ scale,
                                                                         __nv_bfloat16* __restrict__ sx,
                                                                         int64_t sum_group, int64_t kp) {
  __shared__ __align__(16) float tile[kCvThreadsMax / 32][16 * 32];
  __shared__ float red[kCvThreadsMax / 32];
  const int64_t row = blockIdx.x;
  if (row >= m) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int h = lane >> 4, li = lane & 15;
  const int ngroups = (int)(k / 256);
  float* tw = tile[warp];
  uint32_t vals[PPW][8];  // rotated bf16 pairs, transposed order: lane holds indices li + 16 e
  uint32_t amax_bits = 0u;
#pragma unroll
  for (int t = 0; t < PPW; ++t) {
    const int g = 2 * (warp + nwarps * t) + h;
    const bool ok = g < ngroups;
    float v[16];
    uint4 raw[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
    if (ok) {
      const __nv_bfloat16* src = x + row * ldx + (int64_t)g * 256 + 16 * li;
      raw[0] = ldg_nc_v4(src);
      raw[1] = ldg_nc_v4(src + 8);
      if (act == H3B200_ACT_SWIGLU) {  // [gate | up] raw row: silu(gate) * up, exact bf16
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const uint4 u = ldg_nc_v4(src + k + 8 * hh);
          raw[hh] = make_uint4(swiglu_bf16x2(raw[hh].x, u.x), swiglu_bf16x2(raw[hh].y, u.y),
                               swiglu_bf16x2(raw[hh].z, u.z), swiglu_bf16x2(raw[hh].w, u.w));
        }
      }
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      uint32_t w[4] = {raw[hh].x, raw[hh].y, raw[hh].z, raw[hh].w};
      if (act == H3B200_ACT_GELU_TANH) {  // exact bf16 GELU from the device table
#pragma unroll
        for (int e = 0; e < 4; ++e) w[e] = gelu_bf16_bits(w[e]) | (gelu_bf16_bits(w[e] >> 16) << 16);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        v[8 * hh + 2 * e] = bf16_lo(w[e]);
        v[8 * hh + 2 * e + 1] = bf16_hi(w[e]);
      }
    }
    h4_digit_lo(v);
    h4_digit_hi(v);
    // transpose: write row li (16-byte chunks), read column li
#pragma unroll
    for (int c = 0; c < 4; ++c)
      *reinterpret_cast<float4*>(tw + tr_addr(li, h, 4 * c)) = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
    __syncwarp();
#pragma unroll
    for (int e = 0; e < 16; ++e) v[e] = tw[tr_addr(e, h, li)];
    __syncwarp();
    h4_digit_lo(v);
    h4_digit_hi(v);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t pb = pack_bf16(v[2 * e] * 0.0625f, v[2 * e + 1] * 0.0625f);
      vals[t][e] = pb;
      if (ok) amax_bits = __vmaxu2(amax_bits, pb & 0x7FFF7FFFu);  // per-half running max of |bf16|
    }
  }
  amax_bits = max(amax_bits & 0xFFFFu, amax_bits >> 16);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax_bits = max(amax_bits, __shfl_xor_sync(0xffffffffu, amax_bits, o));
  if (lane == 0) red[warp] = __uint_as_float(amax_bits << 16);
  __syncthreads();
  float rowmax = red[0];
  for (int i = 1; i < nwarps; ++i) rowmax = fmaxf(rowmax, red[i]);
  const float s = fmaxf(__fdiv_rn(rowmax, 127.0f), 1e-30f);
  const float sb = quant_divisor(s);
  const float rcp = __frcp_rn(sb);
  const int lanes_per_sum = (int)(sum_group / 16);
#pragma unroll
  for (int t = 0; t < PPW; ++t) {
    const int g = 2 * (warp + nwarps * t) + h;
    // back to contiguous order: write column li, read row li
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      tw[tr_addr(2 * e, h, li)] = bf16_lo(vals[t][e]);
      tw[tr_addr(2 * e + 1, h, li)] = bf16_hi(vals[t][e]);
    }
    __syncwarp();
    uint32_t pw[8];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float4 f = *reinterpret_cast<const float4*>(tw + tr_addr(li, h, 4 * c));
      pw[2 * c] = pack_bf16(f.x, f.y);
      pw[2 * c + 1] = pack_bf16(f.z, f.w);
    }
    __syncwarp();
    const bool ok = g < ngroups;  // the same for the 16 lanes of a half-warp
    const uint2 q0 = quant_vec8(make_uint4(pw[0], pw[1], pw[2], pw[3]), rcp);
    const uint2 q1 = quant_vec8(make_uint4(pw[4], pw[5], pw[6], pw[7]), rcp);
    if (ok) *reinterpret_cast<uint4*>(q + row * k + (int64_t)g * 256 + 16 * li) = make_uint4(q0.x, q0.y, q1.x, q1.y);
    if (sx != nullptr) {  // all lanes shuffle; partners stay inside the half-warp (offsets < 16)
      int isum = __dp4a((int)q0.x, 0x01010101, __dp4a((int)q0.y, 0x01010101,
                        __dp4a((int)q1.x, 0x01010101, __dp4a((int)q1.y, 0x01010101, 0))));
      for (int o = 1; o < lanes_per_sum; o <<= 1) isum += __shfl_xor_sync(0xffffffffu, isum, o);
      if (ok && (li % lanes_per_sum) == 0)
        sx[row * kp + ((int64_t)g * 256 + 16 * li) / sum_group] =
            __float2bfloat16_rn(__fmul_rn(bf16_round((float)isum), bf16_round(s)));
    }
  }
  if (sx != nullptr) {  // zero the K padding of the correction operand
    for (int64_t i = k / sum_group + threadIdx.x; i < kp; i += blockDim.x) sx[row * kp + i] = __float2bfloat16_rn(0.0f);
  }
  if (threadIdx.x == 0) scale[row] = s;
}

// corrT[n, kp] = correction[g, n] for g < groups, 0 for groups <= g < kp
__global__ void correction_transpose_kernel(const __nv_bfloat16* __restrict__ corr, int64_t groups, int64_t n,
                                            int64_t kp, __nv_bfloat16* __restrict__ corr_t) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n * kp) return;
  const int64_t col = i / kp, g = i - col * kp;
  corr_t[i] = g < groups ? corr[g * n + col] : __float2bfloat16_rn(0.0f);
}

// ---------------------------------------------------------------------------
// ConvRot-256 + row quantization, persistent, for rows of ng 256-groups (K = 256 ng,
// ng <= 12 NP; NP = 1..4 covers K up to 12288). One CTA per SM: a producer warp streams rows into a
// ring of one-row stages (cp.async.bulk, completion counted on mbarriers);
// 12 consumer warps form 4 teams of 3, each team taking every 4th row of the
// CTA, so that 4 rows are in flight at different points of their work. The
// team's 6 half-warps take 2 NP group slots each (slots past ng hold zeros and are
// never stored) and rotate them two at a time in
// lock step (group a in the low, group b in the high half of packed f32x2
// registers) with the butterflies, transposes and summation order of
// quantize_convrot_kernel; the 1/16 normalisation is folded exactly into the
// last butterfly ((s - 2 v) / 16 = fma(-1/8, v, s / 16), both scalings
// exact). The rotated bf16 pairs wait (in registers for a single pair, else in
// the lane's own slots of the stage) until the team's row absmax (met on an
// mbarrier, bounded wait) is known. The
// int8 values are then formed in the transposed order, stored byte by byte
// into shared memory in natural order and written to HBM with 16-byte stores;
// the correction operand sx is summed from those bytes as in
// quantize_convrot_kernel.
// ---------------------------------------------------------------------------
constexpr int kCrConsumers = 12;
constexpr int kCrTeamWarps = 3;
constexpr int kCrTeams = kCrConsumers / kCrTeamWarps;
constexpr int kCrMaxStages = 24;
constexpr int kCrTileBytes = 2048;  // per consumer warp: float transpose tile / byte tile
constexpr int kCrOffRed = 512;      // after the mbarriers
constexpr int kCrOffTiles = 1024;
constexpr int kCrOffRing = kCrOffTiles + kCrConsumers * kCrTileBytes;
constexpr int kCrSmemLimit = 232448;
constexpr unsigned kErrCrProducer = 0x301, kErrCrFull = 0x302, kErrCrTeam = 0x303, kErrCrDrain = 0x304;

__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_make(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_split(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void sts_u8(void* p, uint32_t v) {
  asm volatile("st.shared.u8 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}

// The H4 butterflies of h4_digit_lo / h4_digit_hi on two groups at once. LAST:
// the output is scaled by 1/16 (exact).
template <bool LAST>
__device__ __forceinline__ void h4x2_lo(uint64_t (&P)[16]) {
  const uint64_t m2 = f2_dup(LAST ? -0.125f : -2.0f);
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    uint64_t s = f2_add(f2_add(P[4 * a], P[4 * a + 1]), f2_add(P[4 * a + 2], P[4 * a + 3]));
    if (LAST) s = f2_mul(s, f2_dup(0.0625f));
    const uint64_t t0 = f2_fma(m2, P[4 * a + 3], s), t1 = f2_fma(m2, P[4 * a + 2], s);
    const uint64_t t2 = f2_fma(m2, P[4 * a + 1], s), t3 = f2_fma(m2, P[4 * a], s);
    P[4 * a] = t0; P[4 * a + 1] = t1; P[4 * a + 2] = t2; P[4 * a + 3] = t3;
  }
}
template <bool LAST>
__device__ __forceinline__ void h4x2_hi(uint64_t (&P)[16]) {
  const uint64_t m2 = f2_dup(LAST ? -0.125f : -2.0f);
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    uint64_t s = f2_add(f2_add(P[b], P[4 + b]), f2_add(P[8 + b], P[12 + b]));
    if (LAST) s = f2_mul(s, f2_dup(0.0625f));
    const uint64_t t0 = f2_fma(m2, P[12 + b], s), t1 = f2_fma(m2, P[8 + b], s);
    const uint64_t t2 = f2_fma(m2, P[4 + b], s), t3 = f2_fma(m2, P[b], s);
    P[b] = t0; P[4 + b] = t1; P[8 + b] = t2; P[12 + b] = t3;
  }
}

// Consumer teams of a CTA (12 consumer warps); 4 rows in flight.
template <int NP>
__global__ void __launch_bounds__(32 * (1 + kCrTeamWarps * kCrTeams), 1)
    convrot_ring_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int64_t m, int act,
                        int8_t* __restrict__ q, float* __restrict__ scale, __nv_bfloat16* __restrict__ sx,
                        int sum_group, int64_t kp, int stages, int ng) {
  const int K = 256 * ng;
  const int ROW_BYTES = 2 * K;
  constexpr int HALF_GROUPS = 2 * kCrTeamWarps;  // half-warps of a team
  constexpr int TEAMS = kCrTeams;                // NP: group pairs per half-warp
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty_bar = full_bar + kCrMaxStages;
  uint64_t* team_bar = empty_bar + kCrMaxStages;  // [TEAMS]
  uint32_t* red = reinterpret_cast<uint32_t*>(smem + kCrOffRed);  // [TEAMS][2][kCrTeamWarps] row-max bits
  uint8_t* ring = smem + kCrOffRing;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t G = gridDim.x;
  const int64_t cnt = m > (int64_t)blockIdx.x ? (m - blockIdx.x + G - 1) / G : 0;  // rows of this CTA
  const int S = stages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kCrTeamWarps);
    }
    for (int t = 0; t < TEAMS; ++t) mbar_init(&team_bar[t], kCrTeamWarps);
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer ----------------
      int64_t j = 0;
      for (; j < cnt; ++j) {
        const int s = (int)(j % S);
        const uint32_t use = (uint32_t)(j / S);
        if (!mbar_wait(&empty_bar[s], (use & 1u) ^ 1u, kErrCrProducer)) break;
        mbar_arrive_expect_tx(&full_bar[s], (uint32_t)ROW_BYTES);
        bulk_g2s(ring + (size_t)s * ROW_BYTES, x + (blockIdx.x + j * G) * ldx, (uint32_t)ROW_BYTES, &full_bar[s]);
      }
      // every copy issued lands before the CTA may exit
      for (int64_t i = (j > S ? j - S : 0); i < j; ++i)
        mbar_wait(&full_bar[i % S], (uint32_t)(i / S) & 1u, kErrCrDrain, 200000000ull);
    }
    return;
  }

  // ---------------- consumers ----------------
  const int cw = warp - 1;
  const int team = cw / kCrTeamWarps, tw = cw - team * kCrTeamWarps;
  const int h = lane >> 4, li = lane & 15;
  const int hw = 2 * tw + h;  // half-warp within the team: groups hw + 6 i
  // The lane's 32 bytes of a group are read as two 16-byte halves, the upper
  // one first in lanes with bit 2 set, so that the 8 lanes of a quarter-warp
  // hit distinct banks. Registers 0-7 then hold indices 8 c1 .. 8 c1 + 7: the
  // H4 butterflies commute with that relabelling (flipping index bit 3 maps a
  // digit d to d ^ 2 on inputs and outputs alike), so only the transpose
  // write addresses depend on it.
  const int c1 = (li >> 2) & 1;
  uint8_t* tile = smem + kCrOffTiles + cw * kCrTileBytes;
  float* tf = reinterpret_cast<float*>(tile);
  uint8_t* bt = tile + h * 528;  // byte tile: group a [0, 256), group b [256, 512)
  uint32_t* rteam = red + team * (2 * kCrTeamWarps);
  const int lanes_per_sum = sum_group / 16;
  const uint64_t magic = f2_dup(12582912.0f);  // 1.5 * 2^23
  uint32_t team_phase = 0;
  for (int64_t j = team; j < cnt; j += TEAMS) {
    const int s = (int)(j % S);
    const int64_t row = blockIdx.x + j * G;
    if (!mbar_wait(&full_bar[s], (uint32_t)(j / S) & 1u, kErrCrFull)) break;
    const uint8_t* st = ring + (size_t)s * ROW_BYTES;
    uint32_t amax = 0u;
    // per pair: bf16 (group a, group b) of index li + 16 e. One pair stays in
    // registers; with more, each waits in this lane's own 32-byte slots of the
    // stage (only this lane reads them back) until the row absmax is known.
    uint32_t wab[16];
#pragma unroll 1
    for (int pr = 0; pr < NP; ++pr) {
      const int ga = hw + HALF_GROUPS * pr, gb = ga + HALF_GROUPS * NP;
      const bool oka = ga < ng, okb = gb < ng;  // slots past the row hold zeros
      uint8_t* sa = const_cast<uint8_t*>(st) + (oka ? ga : 0) * 512 + li * 32;
      uint8_t* sb = const_cast<uint8_t*>(st) + (okb ? gb : 0) * 512 + li * 32;
      uint32_t wa[8], wb[8];
      {
        const uint4 z = make_uint4(0, 0, 0, 0);
        const uint4 a0 = oka ? *reinterpret_cast<const uint4*>(sa + 16 * c1) : z;
        const uint4 a1 = oka ? *reinterpret_cast<const uint4*>(sa + 16 - 16 * c1) : z;
        const uint4 b0 = okb ? *reinterpret_cast<const uint4*>(sb + 16 * c1) : z;
        const uint4 b1 = okb ? *reinterpret_cast<const uint4*>(sb + 16 - 16 * c1) : z;
        wa[0] = a0.x; wa[1] = a0.y; wa[2] = a0.z; wa[3] = a0.w; wa[4] = a1.x; wa[5] = a1.y; wa[6] = a1.z; wa[7] = a1.w;
        wb[0] = b0.x; wb[1] = b0.y; wb[2] = b0.z; wb[3] = b0.w; wb[4] = b1.x; wb[5] = b1.y; wb[6] = b1.z; wb[7] = b1.w;
      }
      if (act == H3B200_ACT_GELU_TANH) {  // exact bf16 GELU from the device table
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          wa[e] = gelu_bf16_bits(wa[e]) | (gelu_bf16_bits(wa[e] >> 16) << 16);
          wb[e] = gelu_bf16_bits(wb[e]) | (gelu_bf16_bits(wb[e] >> 16) << 16);
        }
      }
      uint64_t P[16];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        P[2 * e] = f2_make(bf16_lo(wa[e]), bf16_lo(wb[e]));
        P[2 * e + 1] = f2_make(bf16_hi(wa[e]), bf16_hi(wb[e]));
      }
      h4x2_lo<false>(P);
      h4x2_hi<false>(P);
      // transpose each group: write row li, read column li (lane then holds indices li + 16 e)
      float va[16], vb[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) f2_split(P[e], va[e], vb[e]);
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<float4*>(tf + tr_addr(li, h, 4 * (c ^ (2 * c1)))) =
            make_float4(va[4 * c], va[4 * c + 1], va[4 * c + 2], va[4 * c + 3]);
      __syncwarp();
#pragma unroll
      for (int e = 0; e < 16; ++e) va[e] = tf[tr_addr(e, h, li)];
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<float4*>(tf + tr_addr(li, h, 4 * (c ^ (2 * c1)))) =
            make_float4(vb[4 * c], vb[4 * c + 1], vb[4 * c + 2], vb[4 * c + 3]);
      __syncwarp();
#pragma unroll
      for (int e = 0; e < 16; ++e) vb[e] = tf[tr_addr(e, h, li)];
      __syncwarp();
#pragma unroll
      for (int e = 0; e < 16; ++e) P[e] = f2_make(va[e], vb[e]);
      h4x2_lo<false>(P);
      h4x2_hi<true>(P);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        float a, b;
        f2_split(P[e], a, b);
        wab[e] = pack_bf16(a, b);
        amax = __vmaxu2(amax, wab[e] & 0x7FFF7FFFu);  // per-half running max of |bf16|
      }
      if (NP > 1) {  // park the pair in this lane's own slots of the groups it read
        if (okb) {     // the 16 (a, b) words span both 32-byte slots
          *reinterpret_cast<uint4*>(sa) = make_uint4(wab[0], wab[1], wab[2], wab[3]);
          *reinterpret_cast<uint4*>(sa + 16) = make_uint4(wab[4], wab[5], wab[6], wab[7]);
          *reinterpret_cast<uint4*>(sb) = make_uint4(wab[8], wab[9], wab[10], wab[11]);
          *reinterpret_cast<uint4*>(sb + 16) = make_uint4(wab[12], wab[13], wab[14], wab[15]);
        } else if (oka) {  // empty b slot: group a's 16 values (the low halves) fit its own slot
          uint32_t w[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) w[i] = __byte_perm(wab[2 * i], wab[2 * i + 1], 0x5410);
          *reinterpret_cast<uint4*>(sa) = make_uint4(w[0], w[1], w[2], w[3]);
          *reinterpret_cast<uint4*>(sa + 16) = make_uint4(w[4], w[5], w[6], w[7]);
        }
      }
    }
    // row absmax over the team
    amax = max(amax & 0xFFFFu, amax >> 16);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    uint32_t* rr = rteam + (team_phase & 1u) * kCrTeamWarps;
    if (lane == 0) {
      rr[tw] = amax;
      mbar_arrive(&team_bar[team]);
    }
    if (!mbar_wait(&team_bar[team], team_phase & 1u, kErrCrTeam)) break;
    ++team_phase;
    uint32_t rowbits = rr[0];
#pragma unroll
    for (int i = 1; i < kCrTeamWarps; ++i) rowbits = max(rowbits, rr[i]);
    const float s_row = fmaxf(__fdiv_rn(__uint_as_float(rowbits << 16), 127.0f), 1e-30f);
    const uint64_t r2 = f2_dup(__frcp_rn(quant_divisor(s_row)));
#pragma unroll 1
    for (int pr = 0; pr < NP; ++pr) {
      const int ga = hw + HALF_GROUPS * pr, gb = ga + HALF_GROUPS * NP;
      const bool oka = ga < ng, okb = gb < ng;
      if (NP > 1) {
        const uint8_t* sa = st + (oka ? ga : 0) * 512 + li * 32;
        const uint8_t* sb = st + (okb ? gb : 0) * 512 + li * 32;
        const uint4 z = make_uint4(0, 0, 0, 0);
        const uint4 a0 = oka ? *reinterpret_cast<const uint4*>(sa) : z, a1 = oka ? *reinterpret_cast<const uint4*>(sa + 16) : z;
        if (okb) {
          const uint4 b0 = *reinterpret_cast<const uint4*>(sb), b1 = *reinterpret_cast<const uint4*>(sb + 16);
          wab[0] = a0.x; wab[1] = a0.y; wab[2] = a0.z; wab[3] = a0.w; wab[4] = a1.x; wab[5] = a1.y; wab[6] = a1.z;
          wab[7] = a1.w; wab[8] = b0.x; wab[9] = b0.y; wab[10] = b0.z; wab[11] = b0.w; wab[12] = b1.x; wab[13] = b1.y;
          wab[14] = b1.z; wab[15] = b1.w;
        } else {  // group a's values only (b is an empty slot: zeros in the high halves)
          const uint32_t w[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            wab[2 * i] = w[i] & 0xFFFFu;
            wab[2 * i + 1] = w[i] >> 16;
          }
        }
      }
      // quantize in the transposed order; bytes land in natural order in the byte tile
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        uint32_t t0, t1;
        f2_bits(f2_mul(bf16x2_to_f2(wab[e]), r2), t0, t1);
        const uint32_t b = bf16x2_clamp_i8(bf16x2_from_bits(t0, t1));
        uint32_t qa, qb;
        f2_bits(f2_add(bf16x2_to_f2(b), magic), qa, qb);  // the integers sit in the low bytes
        sts_u8(bt + li + 16 * e, qa);
        sts_u8(bt + 256 + li + 16 * e, qb);
      }
      __syncwarp();
#pragma unroll
      for (int pg = 0; pg < 2; ++pg) {
        const int g = pg ? gb : ga;
        const bool live = g < ng;  // an empty slot stores nothing (its lanes still take part in the shuffles)
        const uint4 v = *reinterpret_cast<const uint4*>(bt + pg * 256 + 16 * li);
        if (live) stg_v4(q + row * K + g * 256 + 16 * li, v);
        if (sx != nullptr) {  // all lanes shuffle; partners stay inside the half-warp (offsets < 16)
          int isum = __dp4a((int)v.x, 0x01010101, __dp4a((int)v.y, 0x01010101,
                            __dp4a((int)v.z, 0x01010101, __dp4a((int)v.w, 0x01010101, 0))));
          for (int o = 1; o < lanes_per_sum; o <<= 1) isum += __shfl_xor_sync(0xffffffffu, isum, o);
          if (live && (li % lanes_per_sum) == 0)
            sx[row * kp + (g * 256 + 16 * li) / sum_group] =
                __float2bfloat16_rn(__fmul_rn(bf16_round((float)isum), bf16_round(s_row)));
        }
      }
      __syncwarp();  // the byte tile is reused
    }
    // the stage was written here (parked pairs) and is refilled by the async proxy next
    fence_proxy_async_shared();
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[s]);  // this warp is done with the stage
    if (tw == 0) {
      if (lane == 0) scale[row] = s_row;
      if (sx != nullptr)  // zero the K padding of the correction operand
        for (int64_t i = K / sum_group + lane; i < kp; i += 32) sx[row * kp + i] = __float2bfloat16_rn(0.0f);
    }
  }
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

cudaError_t launch_quantize_convrot(const void* x, int64_t ldx, int64_t m, int64_t k, int act, int8_t* q,
                                    float* scale, void* sx, int64_t sum_group, int64_t kp, cudaStream_t stream) {
  if (m == 0) return cudaSuccess;
  if (k % 256 || ldx % 8 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(q) & 15))
    return cudaErrorNotSupported;
  if (sx != nullptr && (sum_group < 16 || sum_group > 256 || 256 % sum_group || kp < k / sum_group))
    return cudaErrorNotSupported;
  {
    const cudaError_t e = ensure_act_table(act, stream);
    if (e != cudaSuccess) return e;
  }
  const int64_t ngroups = k / 256;
  const int64_t np = (ngroups + 2 * 6 - 1) / (2 * 6);  // group pairs per half-warp of a 6-half-warp team
  // the persistent kernel's stages hold one activated-width row, so SwiGLU rows
  // ([gate | up], twice as wide) take the per-row kernel
  if (np >= 1 && np <= 5 && act != H3B200_ACT_SWIGLU) {
    int dev = 0;
    cudaGetDevice(&dev);
    static bool attr_set[64][9] = {};
    const int64_t row_bytes = 2 * k;
    const int stages = (int)std::min<int64_t>(kCrMaxStages, (kCrSmemLimit - 1024 - kCrOffRing) / row_bytes);
    const int smem = 1024 + kCrOffRing + stages * (int)row_bytes;
    const unsigned grid = (unsigned)std::min<int64_t>(m, (int64_t)num_sms(dev));
    const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
    __nv_bfloat16* sxb = static_cast<__nv_bfloat16*>(sx);
    const int sg = sx != nullptr ? (int)sum_group : 16;
    auto go = [&](auto kern) -> cudaError_t {
      if (dev >= 0 && dev < 64 && !attr_set[dev][np]) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kCrSmemLimit);
        if (e != cudaSuccess) return e;
        attr_set[dev][np] = true;
      }
      const int threads = 32 * (1 + kCrConsumers);
      kern<<<grid, threads, smem, stream>>>(xb, ldx, m, act, q, scale, sxb, sg, kp, stages, (int)ngroups);
      return cudaGetLastError();
    };
    // A team waits for row j after consuming its row j - teams; the producer fills in
    // order, so with stages >= teams the stage's previous row (j - stages) has landed
    // and the parity wait cannot pass on the phase before it. Rows of up to 48
    // groups get 8 or more stages; 49-60 groups (H3's 56-group fc2 input) 7 or 8.
    if (stages >= kCrTeams) {
      switch (np) {
        case 1: return go(convrot_ring_kernel<1>);
        case 2: return go(convrot_ring_kernel<2>);
        case 3: return go(convrot_ring_kernel<3>);
        case 4: return go(convrot_ring_kernel<4>);
        case 5: return go(convrot_ring_kernel<5>);
        default: break;
      }
    }
  }
  const int64_t pairs = (k / 256 + 1) / 2;
  const int64_t nwarps = pairs < 8 ? pairs : 8;
  const int64_t ppw = (pairs + nwarps - 1) / nwarps;
  const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
  __nv_bfloat16* sxb = static_cast<__nv_bfloat16*>(sx);
  dim3 grid((unsigned)m), block((unsigned)(32 * nwarps));
  switch (ppw) {
    case 1: quantize_convrot_kernel<1><<<grid, block, 0, stream>>>(xb, ldx, m, k, act, q, scale, sxb, sum_group, kp); break;
    case 2: quantize_convrot_kernel<2><<<grid, block, 0, stream>>>(xb, ldx, m, k, act, q, scale, sxb, sum_group, kp); break;
    case 3: quantize_convrot_kernel<3><<<grid, block, 0, stream>>>(xb, ldx, m, k, act, q, scale, sxb, sum_group, kp); break;
    case 4: quantize_convrot_kernel<4><<<grid, block, 0, stream>>>(xb, ldx, m, k, act, q, scale, sxb, sum_group, kp); break;
    default: return cudaErrorNotSupported;  // k > 32768
  }
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
