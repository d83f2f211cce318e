// W4A8 pieces: int4 -> int8 grid decode, ConvRot-256 rotation + row
// quantization (with int8 group sums for the asymmetric correction), and the
// asymmetric group-correction epilogue.
//
// Reference: comfy_kitchen W4A8 (backends/eager/w4a8_int8.py:344-363 decode;
// backends/cuda/ops/w4a8_gemm.cu:36-90; ConvRot quantizer
// backends/cuda/ops/int8_linear.cu:256-340 / eager quantize_and_rotate_rowwise
// backends/eager/quantization.py:878-895; correction
// backends/cuda/__init__.py:2294-2297).
#include "common.cuh"
#include "kernels.h"
#include "quant_math.cuh"

namespace h3 {
namespace {

// ---------------------------------------------------------------------------
// Decode: 16 outputs per thread (8 packed bytes), group_size % 16 == 0.
// q = clamp(rne((u - 8) * s_rel), -127, 127); even column = low nibble.
// ---------------------------------------------------------------------------
__global__ void dequant_int4_kernel(const uint8_t* __restrict__ qd, const float* __restrict__ s_rel, int64_t n,
                                    int64_t k, int64_t group, int8_t* __restrict__ out) {
  const int64_t per_row = k / 16;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * per_row) return;
  const int64_t row = idx / per_row;
  const int64_t c16 = (idx - row * per_row) * 16;
  const float s = s_rel[row * (k / group) + c16 / group];
  const uint2 pk = *reinterpret_cast<const uint2*>(qd + row * (k / 2) + c16 / 2);
  const uint32_t w[2] = {pk.x, pk.y};
  uint32_t o[4] = {0, 0, 0, 0};
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    const uint32_t byte = (w[b >> 2] >> (8 * (b & 3))) & 0xFFu;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float u = (float)((byte >> (4 * h)) & 0xFu) - 8.0f;
      float v = rintf(__fmul_rn(u, s));
      v = fminf(fmaxf(v, -127.0f), 127.0f);
      const int e = 2 * b + h;
      o[e >> 2] |= (uint32_t)(uint8_t)(int8_t)(int)v << (8 * (e & 3));
    }
  }
  *reinterpret_cast<uint4*>(out + row * k + c16) = make_uint4(o[0], o[1], o[2], o[3]);
}

// Generic decode (any group size dividing k).
__global__ void dequant_int4_scalar_kernel(const uint8_t* __restrict__ qd, const float* __restrict__ s_rel,
                                           int64_t n, int64_t k, int64_t group, int8_t* __restrict__ out) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * k) return;
  const int64_t row = idx / k, col = idx - row * k;
  const uint32_t byte = qd[row * (k / 2) + col / 2];
  const float u = (float)((byte >> (4 * (col & 1))) & 0xFu) - 8.0f;
  float v = rintf(__fmul_rn(u, s_rel[row * (k / group) + col / group]));
  out[idx] = (int8_t)(int)fminf(fmaxf(v, -127.0f), 127.0f);
}

// ---------------------------------------------------------------------------
// ConvRot-256 + row quantization. One CTA (8 warps) per row; warp w rotates
// groups w, w+8, ...; lane l holds elements 8l..8l+7 of a 256-group. The
// regular Hadamard H4^(x)4 is applied one base-4 digit at a time:
// y_j = S - 2 v_(3-j) with S the sum of the four values on that digit axis.
// Digit 0 is lane-local, digit 1 pairs lanes l^1, digits 2/3 use lanes l^{2,4,6}
// and l^{8,16,24}. The 1/16 normalisation is exact. The rotated value is
// rounded to bf16 (the reference's bf16 rotation matmul output), then the row
// is quantized exactly like quantize_int8_rowwise.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float h4_lane_digit(float v, int mask_lo, int mask_hi, int mask_pair) {
  const float s1 = v + __shfl_xor_sync(0xffffffffu, v, mask_lo);
  const float s = s1 + __shfl_xor_sync(0xffffffffu, s1, mask_hi);
  const float p = __shfl_xor_sync(0xffffffffu, v, mask_pair);
  return s - 2.0f * p;
}

template <int GPW>
__global__ void __launch_bounds__(256) quantize_convrot_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                               int64_t m, int64_t k, int act, int8_t* __restrict__ q,
                                                               float* __restrict__ scale,
                                                               int32_t* __restrict__ gsum, int64_t sum_group) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  if (row >= m) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t ngroups = k / 256;
  float vals[GPW][8];
  float amax = 0.0f;
#pragma unroll
  for (int gi = 0; gi < GPW; ++gi) {
    const int64_t g = warp + 8 * gi;
    if (g < ngroups) {  // warp-uniform
      const uint4 raw = ldg_nc_v4(x + row * ldx + g * 256 + lane * 8);
      uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
      if (act == H3B200_ACT_GELU_TANH) {  // exact bf16 GELU from the device table
#pragma unroll
        for (int e = 0; e < 4; ++e) w[e] = gelu_bf16_bits(w[e]) | (gelu_bf16_bits(w[e] >> 16) << 16);
      }
      float v[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        v[2 * e] = bf16_lo(w[e]);
        v[2 * e + 1] = bf16_hi(w[e]);
      }
      // digit 0 (lane-local, elements 4a + b)
#pragma unroll
      for (int a = 0; a < 2; ++a) {
        const float s = v[4 * a] + v[4 * a + 1] + v[4 * a + 2] + v[4 * a + 3];
        const float t0 = s - 2.0f * v[4 * a + 3], t1 = s - 2.0f * v[4 * a + 2];
        const float t2 = s - 2.0f * v[4 * a + 1], t3 = s - 2.0f * v[4 * a];
        v[4 * a] = t0; v[4 * a + 1] = t1; v[4 * a + 2] = t2; v[4 * a + 3] = t3;
      }
      // digit 1: (e >> 2) | ((lane & 1) << 1)
#pragma unroll
      for (int d0 = 0; d0 < 4; ++d0) {
        const float p0 = __shfl_xor_sync(0xffffffffu, v[d0], 1);
        const float p1 = __shfl_xor_sync(0xffffffffu, v[4 + d0], 1);
        const float s = v[d0] + v[4 + d0] + p0 + p1;
        const float y0 = s - 2.0f * p1;   // own a=0 pairs with partner a=1
        const float y1 = s - 2.0f * p0;
        v[d0] = y0;
        v[4 + d0] = y1;
      }
      // digit 2: lane bits 1-2; digit 3: lane bits 3-4
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = h4_lane_digit(v[e], 2, 4, 6);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = h4_lane_digit(v[e], 8, 16, 24);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        vals[gi][e] = bf16_round(v[e] * 0.0625f);
        amax = fmaxf(amax, fabsf(vals[gi][e]));
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (lane == 0) red[warp] = amax;
  __syncthreads();
  float rowmax = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) rowmax = fmaxf(rowmax, red[i]);
  const float s = fmaxf(__fdiv_rn(rowmax, 127.0f), 1e-30f);
  const float sb = quant_divisor(s);
  const float rcp = __frcp_rn(sb);
  const int lanes_per_sum = (int)(sum_group / 8);
#pragma unroll
  for (int gi = 0; gi < GPW; ++gi) {
    const int64_t g = warp + 8 * gi;
    if (g < ngroups) {
      // the rotated values are bf16-exact: pack them and quantize like quantize_int8_rowwise
      const uint4 pv = make_uint4(pack_bf16(vals[gi][0], vals[gi][1]), pack_bf16(vals[gi][2], vals[gi][3]),
                                  pack_bf16(vals[gi][4], vals[gi][5]), pack_bf16(vals[gi][6], vals[gi][7]));
      const uint2 qq = quant_vec8(pv, sb, rcp);
      int isum = __dp4a((int)qq.x, 0x01010101, __dp4a((int)qq.y, 0x01010101, 0));  // sum of the 8 int8
      *reinterpret_cast<uint2*>(q + row * k + g * 256 + lane * 8) = qq;
      if (gsum != nullptr) {
        for (int o = 1; o < lanes_per_sum; o <<= 1) isum += __shfl_xor_sync(0xffffffffu, isum, o);
        if ((lane % lanes_per_sum) == 0) gsum[row * (k / sum_group) + (g * 256 + lane * 8) / sum_group] = isum;
      }
    }
  }
  if (threadIdx.x == 0) scale[row] = s;
}

// ---------------------------------------------------------------------------
// Asymmetric correction: out = bf16(out + sum_g sx[m, g] * corr[g, n]) with
// sx = bf16(bf16(gsum) * bf16(xs)). CTA tile 64 rows x 128 columns, operands
// staged in shared memory, fp32 accumulation.
// ---------------------------------------------------------------------------
constexpr int kCorrRows = 64, kCorrCols = 128, kCorrMaxG = 128;

__global__ void __launch_bounds__(256) w4a8_correction_kernel(const int32_t* __restrict__ gsum,
                                                              const float* __restrict__ xs,
                                                              const __nv_bfloat16* __restrict__ corr, int64_t m,
                                                              int64_t n, int groups, __nv_bfloat16* __restrict__ out,
                                                              int64_t ldo) {
  extern __shared__ float sm[];
  float* sx = sm;                                   // [kCorrRows][groups + 1]
  float* cr = sm + kCorrRows * (groups + 1);        // [groups][kCorrCols]
  const int64_t r0 = (int64_t)blockIdx.y * kCorrRows;
  const int64_t c0 = (int64_t)blockIdx.x * kCorrCols;
  for (int i = threadIdx.x; i < kCorrRows * groups; i += blockDim.x) {
    const int r = i / groups, g = i - r * groups;
    float v = 0.0f;
    if (r0 + r < m) {
      const float gs = bf16_round((float)gsum[(r0 + r) * groups + g]);
      v = bf16_round(__fmul_rn(gs, bf16_round(xs[r0 + r])));
    }
    sx[r * (groups + 1) + g] = v;
  }
  for (int i = threadIdx.x; i < groups * kCorrCols; i += blockDim.x) {
    const int g = i / kCorrCols, c = i - g * kCorrCols;
    cr[i] = (c0 + c < n) ? __bfloat162float(corr[(int64_t)g * n + c0 + c]) : 0.0f;
  }
  __syncthreads();
  // thread -> 4 rows x 8 columns
  const int tc = threadIdx.x & 15, tr = threadIdx.x >> 4;
  float acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
  for (int g = 0; g < groups; ++g) {
    float a[4], b[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) a[i] = sx[(tr * 4 + i) * (groups + 1) + g];
#pragma unroll
    for (int j = 0; j < 8; ++j) b[j] = cr[g * kCorrCols + tc * 8 + j];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = r0 + tr * 4 + i;
    const int64_t c = c0 + tc * 8;
    if (r < m && c < n) {
      __nv_bfloat16* op = out + r * ldo + c;
      const uint4 ov = *reinterpret_cast<const uint4*>(op);
      const uint32_t w[4] = {ov.x, ov.y, ov.z, ov.w};
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        o[e] = pack_bf16(__fadd_rn(bf16_lo(w[e]), acc[i][2 * e]), __fadd_rn(bf16_hi(w[e]), acc[i][2 * e + 1]));
      *reinterpret_cast<uint4*>(op) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

}  // namespace

cudaError_t launch_dequant_int4(const int8_t* qdata, const float* s_rel, int64_t n, int64_t k, int64_t group,
                                int8_t* out, cudaStream_t stream) {
  if (n == 0 || k == 0) return cudaSuccess;
  const uint8_t* qd = reinterpret_cast<const uint8_t*>(qdata);
  if (group % 16 == 0 && k % 16 == 0 && !(reinterpret_cast<uintptr_t>(qdata) & 7) &&
      !(reinterpret_cast<uintptr_t>(out) & 15)) {
    const int64_t total = n * (k / 16);
    dequant_int4_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(qd, s_rel, n, k, group, out);
  } else {
    const int64_t total = n * k;
    dequant_int4_scalar_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(qd, s_rel, n, k, group, out);
  }
  return cudaGetLastError();
}

cudaError_t launch_quantize_convrot(const void* x, int64_t ldx, int64_t m, int64_t k, int act, int8_t* q,
                                    float* scale, int32_t* group_sums, int64_t sum_group, cudaStream_t stream) {
  if (m == 0) return cudaSuccess;
  if (k % 256 || ldx % 8 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(q) & 7))
    return cudaErrorNotSupported;
  if (group_sums != nullptr && (sum_group < 8 || sum_group > 256 || 256 % sum_group)) return cudaErrorNotSupported;
  if (act == H3B200_ACT_GELU_TANH) {
    const cudaError_t e = ensure_gelu_table(stream);
    if (e != cudaSuccess) return e;
  }
  const int64_t ng = k / 256;
  const int64_t gpw = (ng + 7) / 8;
  const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
  dim3 grid((unsigned)m);
  if (gpw <= 1) quantize_convrot_kernel<1><<<grid, 256, 0, stream>>>(xb, ldx, m, k, act, q, scale, group_sums, sum_group);
  else if (gpw <= 2) quantize_convrot_kernel<2><<<grid, 256, 0, stream>>>(xb, ldx, m, k, act, q, scale, group_sums, sum_group);
  else if (gpw <= 4) quantize_convrot_kernel<4><<<grid, 256, 0, stream>>>(xb, ldx, m, k, act, q, scale, group_sums, sum_group);
  else if (gpw <= 6) quantize_convrot_kernel<6><<<grid, 256, 0, stream>>>(xb, ldx, m, k, act, q, scale, group_sums, sum_group);
  else if (gpw <= 8) quantize_convrot_kernel<8><<<grid, 256, 0, stream>>>(xb, ldx, m, k, act, q, scale, group_sums, sum_group);
  else return cudaErrorNotSupported;
  return cudaGetLastError();
}

cudaError_t launch_w4a8_correction(const int32_t* gsum, const float* xs, const void* corr, int64_t m, int64_t n,
                                   int64_t groups, void* out, int64_t ldo, cudaStream_t stream) {
  if (m == 0 || n == 0) return cudaSuccess;
  if (groups <= 0 || groups > kCorrMaxG || n % 8 || ldo % 8 || (reinterpret_cast<uintptr_t>(out) & 15))
    return cudaErrorNotSupported;
  const size_t smem = sizeof(float) * ((size_t)kCorrRows * (groups + 1) + (size_t)groups * kCorrCols);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(w4a8_correction_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
    attr = true;
  }
  dim3 grid((unsigned)((n + kCorrCols - 1) / kCorrCols), (unsigned)((m + kCorrRows - 1) / kCorrRows));
  w4a8_correction_kernel<<<grid, 256, smem, stream>>>(gsum, xs, static_cast<const __nv_bfloat16*>(corr), m, n,
                                                       (int)groups, static_cast<__nv_bfloat16*>(out), ldo);
  return cudaGetLastError();
}

}  // namespace h3
