// W4A8 pieces: int4 -> int8 grid decode, ConvRot-256 rotation + row
// quantization (emitting the asymmetric-correction operand
// sx[m, g] = bf16(bf16(sum_{k in g} q) * bf16(xs))), and the correction itself,
// out += sx . corr, run as a tcgen05 bf16 GEMM (gemm_i8.cu, kEpiAddBF16) against
// the transposed, zero-padded correction matrix.
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
                                                               __nv_bfloat16* __restrict__ sx, int64_t sum_group,
                                                               int64_t kp) {
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
      if (sx != nullptr) {
        for (int o = 1; o < lanes_per_sum; o <<= 1) isum += __shfl_xor_sync(0xffffffffu, isum, o);
        if ((lane % lanes_per_sum) == 0)
          sx[row * kp + (g * 256 + lane * 8) / sum_group] =
              __float2bfloat16_rn(__fmul_rn(bf16_round((float)isum), bf16_round(s)));
      }
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
                                    float* scale, void* sx, int64_t sum_group, int64_t kp, cudaStream_t stream) {
  if (m == 0) return cudaSuccess;
  if (k % 256 || ldx % 8 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(q) & 7))
    return cudaErrorNotSupported;
  if (sx != nullptr && (sum_group < 8 || sum_group > 256 || 256 % sum_group || kp < k / sum_group))
    return cudaErrorNotSupported;
  if (act == H3B200_ACT_GELU_TANH) {
    const cudaError_t e = ensure_gelu_table(stream);
    if (e != cudaSuccess) return e;
  }
  const int64_t ng = k / 256;
  const int64_t gpw = (ng + 7) / 8;
  const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
  __nv_bfloat16* sxb = static_cast<__nv_bfloat16*>(sx);
  dim3 grid((unsigned)m);
  if (gpw <= 1) quantize_convrot_kernel<1><<<grid, 256, 0, stream>>>(xb, ldx, m, k, act, q, scale, sxb, sum_group, kp);
  else if (gpw <= 2) quantize_convrot_kernel<2><<<grid, 256, 0, stream>>>(xb, ldx, m, k, act, q, scale, sxb, sum_group, kp);
  else if (gpw <= 4) quantize_convrot_kernel<4><<<grid, 256, 0, stream>>>(xb, ldx, m, k, act, q, scale, sxb, sum_group, kp);
  else if (gpw <= 6) quantize_convrot_kernel<6><<<grid, 256, 0, stream>>>(xb, ldx, m, k, act, q, scale, sxb, sum_group, kp);
  else if (gpw <= 8) quantize_convrot_kernel<8><<<grid, 256, 0, stream>>>(xb, ldx, m, k, act, q, scale, sxb, sum_group, kp);
  else return cudaErrorNotSupported;
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

cudaError_t launch_w4a8_correction(const void* sx, const void* corr_t, int64_t kp, int64_t m, int64_t n, void* out,
                                   int64_t ldo, cudaStream_t stream) {
  GemmArgs g;
  g.a = static_cast<const int8_t*>(sx);
  g.w = static_cast<const int8_t*>(corr_t);
  g.m = m; g.n = n; g.k = kp; g.lda = kp; g.ldw = kp;
  g.epilogue = kEpiAddBF16;
  g.out = out; g.ldo = ldo;
  return launch_gemm_i8(g, stream);
}

}  // namespace h3
