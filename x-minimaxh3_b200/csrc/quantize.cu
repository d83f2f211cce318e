// Per-token absmax INT8 quantizer (HBM-bound).
//
// Reference algorithm: comfy_kitchen quantize_int8_rowwise
// (backends/eager/quantization.py:857-875, rounding helpers :815-826; CUDA
// kernel backends/cuda/ops/int8_linear.cu:157-200):
//   absmax = max |x| over the row (exact on bf16)
//   scale  = max(absmax / 127, 1e-30)            fp32, stored
//   sb     = bf16(scale)                          scale as the bf16 operand
//   q      = clamp(rne(bf16(x / sb)), -128, 127)
//
// Division. Only the bf16 rounding of the quotient x / sb matters, and
// t = x * rcp(sb) (rcp correctly rounded, sb >= bf16(1e-30) so rcp is finite)
// lies within 2 ulp of the exact quotient. That never moves it across a bf16
// rounding midpoint: with x = a 2^i and sb = b 2^j for integer mantissas
// 1 <= a, b <= 255, the ratio a / b is more than 128 fp32 ulp away from every
// bf16 midpoint of its binade (checked for all 255 x 255 mantissa pairs: the
// midpoints have 9 significant bits, and no ratio of two 8-bit integers comes
// that close to one). The product therefore rounds to the same bf16 as the division, as
// an exhaustive sweep over all finite bf16 x and all normal bf16 divisors
// confirms (2.1e9 pairs, no exception).
//
// B200 layout: rows of up to 4096 elements go one warp per row (the row stays
// in registers between the absmax and the quantize pass; no block barrier);
// longer rows one 256-thread CTA per row. HBM sees one read of x (2 B/elem),
// one write of q (1 B/elem) and 4 B of scale per row; 128-bit loads, 64-bit
// stores.
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "quant_math.cuh"

namespace h3 {

namespace {

constexpr int kQThreads = 256;

__device__ __forceinline__ int8_t quant_one(float x, float sb) {
  float v = rintf(bf16_round(__fdiv_rn(x, sb)));
  v = fminf(fmaxf(v, -128.0f), 127.0f);
  return (int8_t)(int)v;
}

__device__ __forceinline__ uint32_t absmax_bits8(const uint4& v) {
  // |x| of bf16 values orders like their magnitude bits (a NaN wins, as in torch's amax)
  const uint32_t a = __vmaxu2(v.x & 0x7FFF7FFFu, v.y & 0x7FFF7FFFu);
  const uint32_t b = __vmaxu2(v.z & 0x7FFF7FFFu, v.w & 0x7FFF7FFFu);
  const uint32_t c = __vmaxu2(a, b);
  return max(c & 0xFFFFu, c >> 16);
}

// x is a bf16 value (as fp32); the activation result is bf16 too
__device__ __forceinline__ float act_apply(float x, int act) {
  return act == H3B200_ACT_GELU_TANH ? __uint_as_float(gelu_bf16_bits(__float_as_uint(x) >> 16) << 16) : x;
}

__device__ __forceinline__ void apply_act_vec(uint4& v, int act) {
  if (act != H3B200_ACT_GELU_TANH) return;
  uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
  for (int e = 0; e < 4; ++e) w[e] = gelu_bf16_bits(w[e]) | (gelu_bf16_bits(w[e] >> 16) << 16);
}

// The 8 activated values at vector index vi of an activated row of width k:
// the row itself for elementwise activations; for SwiGLU the raw row is
// [gate | up], 2 k wide, and the value is silu(gate) * up.
__device__ __forceinline__ uint4 load_act_vec(const __nv_bfloat16* xr, int64_t k, int64_t vi, int act) {
  uint4 v = ldg_nc_v4(xr + vi * 8);
  if (act == H3B200_ACT_SWIGLU) {
    const uint4 u = ldg_nc_v4(xr + k + vi * 8);
    v = make_uint4(swiglu_bf16x2(v.x, u.x), swiglu_bf16x2(v.y, u.y), swiglu_bf16x2(v.z, u.z), swiglu_bf16x2(v.w, u.w));
  } else {
    apply_act_vec(v, act);
  }
  return v;
}

// One activated value (scalar paths).
__device__ __forceinline__ float act_value(const __nv_bfloat16* xr, int64_t k, int64_t i, int act) {
  if (act == H3B200_ACT_SWIGLU) {
    const float s = __uint_as_float(silu_bf16_fast(__bfloat16_as_ushort(xr[i])) << 16);
    return bf16_round(__fmul_rn(s, __bfloat162float(xr[k + i])));
  }
  return act_apply(__bfloat162float(xr[i]), act);
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int i = 1; i < kQThreads / 32; ++i) r = fmaxf(r, red[i]);
  return r;
}

// One warp per row: k % 8 == 0, 16-byte aligned rows, k <= 32 * 8 * VPL.
template <int VPL, bool GIVEN_ABSMAX>
__global__ void __launch_bounds__(kQThreads) quantize_rows_warp_kernel(const __nv_bfloat16* __restrict__ x,
                                                                       int64_t ldx, int64_t m, int64_t k, int act,
                                                                       const float* __restrict__ absmax_in,
                                                                       int8_t* __restrict__ q,
                                                                       float* __restrict__ scale) {
  const int lane = threadIdx.x & 31;
  const int64_t row = ((int64_t)blockIdx.x * kQThreads + threadIdx.x) >> 5;
  if (row >= m) return;
  const int nvec = (int)(k >> 3);
  const __nv_bfloat16* xr = x + row * ldx;
  uint4 v[VPL];
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int vi = lane + 32 * j;
    v[j] = vi < nvec ? load_act_vec(xr, k, vi, act) : make_uint4(0, 0, 0, 0);
  }
  float rowmax;
  if (GIVEN_ABSMAX) {
    rowmax = absmax_in[row];
  } else {
    uint32_t mb = 0;
#pragma unroll
    for (int j = 0; j < VPL; ++j) mb = max(mb, absmax_bits8(v[j]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, o));
    rowmax = __uint_as_float(mb << 16);
  }
  const float s = row_scale(rowmax);
  const float sb = quant_divisor(s);
  const float r = __frcp_rn(sb);
  int8_t* qr = q + row * k;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int vi = lane + 32 * j;
    if (vi < nvec) *reinterpret_cast<uint2*>(qr + vi * 8) = quant_vec8(v[j], r);
  }
  if (lane == 0) scale[row] = s;
}

// One 256-thread CTA per row: k % 8 == 0, 16-byte aligned rows, k <= kQThreads * 8 * VPT.
template <int VPT, bool GIVEN_ABSMAX>
__global__ void __launch_bounds__(kQThreads) quantize_rows_vec_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                                      int64_t m, int64_t k, int act,
                                                                      const float* __restrict__ absmax_in,
                                                                      int8_t* __restrict__ q,
                                                                      float* __restrict__ scale) {
  __shared__ float red[kQThreads / 32];
  const int64_t row = blockIdx.x;
  if (row >= m) return;
  const int64_t nvec = k >> 3;
  const __nv_bfloat16* xr = x + row * ldx;
  uint4 v[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t vi = threadIdx.x + (int64_t)j * kQThreads;
    v[j] = vi < nvec ? load_act_vec(xr, k, vi, act) : make_uint4(0, 0, 0, 0);
  }
  float rowmax;
  if (GIVEN_ABSMAX) {
    rowmax = absmax_in[row];
  } else {
    uint32_t mb = 0;
#pragma unroll
    for (int j = 0; j < VPT; ++j) mb = max(mb, absmax_bits8(v[j]));
    rowmax = block_max(__uint_as_float(mb << 16), red);
  }
  const float s = row_scale(rowmax);
  const float sb = quant_divisor(s);
  const float r = __frcp_rn(sb);
  int8_t* qr = q + row * k;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t vi = threadIdx.x + (int64_t)j * kQThreads;
    if (vi < nvec) *reinterpret_cast<uint2*>(qr + vi * 8) = quant_vec8(v[j], r);
  }
  if (threadIdx.x == 0) scale[row] = s;
}

// Generic path (any k / alignment): two passes over the row in global memory.
__global__ void __launch_bounds__(kQThreads) quantize_rows_scalar_kernel(const __nv_bfloat16* __restrict__ x,
                                                                         int64_t ldx, int64_t m, int64_t k, int act,
                                                                         const float* __restrict__ absmax_in,
                                                                         int8_t* __restrict__ q,
                                                                         float* __restrict__ scale) {
  __shared__ float red[kQThreads / 32];
  const int64_t row = blockIdx.x;
  if (row >= m) return;
  const __nv_bfloat16* xr = x + row * ldx;
  float rowmax;
  if (absmax_in != nullptr) {
    rowmax = absmax_in[row];
  } else {
    float amax = 0.0f;
    for (int64_t i = threadIdx.x; i < k; i += kQThreads) amax = fmaxf(amax, fabsf(act_value(xr, k, i, act)));
    rowmax = block_max(amax, red);
  }
  const float s = row_scale(rowmax);
  const float sb = quant_divisor(s);
  for (int64_t i = threadIdx.x; i < k; i += kQThreads) q[row * k + i] = quant_one(act_value(xr, k, i, act), sb);
  if (threadIdx.x == 0) scale[row] = s;
}

// ---- fp16 activations ----
// The reference's quantizer on an fp16 x (backends/eager/quantization.py:815-826,
// 857-875): the row absmax in fp16 (exact), scale = max(absmax / 127, 1e-30) in fp32,
// the divisor fp16(scale) (torch.finfo(fp16).tiny = 2^-14 when that rounds to zero)
// and q = clamp(rne(fp16(x / divisor)), -128, 127), the quotient formed in fp32 and
// rounded once to fp16 as torch's fp16 division does. One CTA per row, two passes.
__device__ __forceinline__ float quant_divisor_f16(float scale) {
  const float sh = __half2float(__float2half_rn(scale));
  return sh == 0.0f ? 6.103515625e-05f : sh;
}

__global__ void __launch_bounds__(kQThreads) quantize_rows_f16_kernel(const __half* __restrict__ x, int64_t ldx,
                                                                      int64_t m, int64_t k, int8_t* __restrict__ q,
                                                                      float* __restrict__ scale) {
  __shared__ float red[kQThreads / 32];
  const int64_t row = blockIdx.x;
  if (row >= m) return;
  const uint16_t* xr = reinterpret_cast<const uint16_t*>(x + row * ldx);
  uint32_t amax_bits = 0u;  // |x| of fp16 values orders like their magnitude bits (a NaN wins)
  for (int64_t i = threadIdx.x; i < k; i += kQThreads) amax_bits = max(amax_bits, (uint32_t)(xr[i] & 0x7FFFu));
  const float rowmax = block_max(__half2float(__ushort_as_half((unsigned short)amax_bits)), red);
  const float s = row_scale(rowmax);
  const float d = quant_divisor_f16(s);
  for (int64_t i = threadIdx.x; i < k; i += kQThreads) {
    const float xv = __half2float(__ushort_as_half(xr[i]));
    float v = rintf(__half2float(__float2half_rn(__fdiv_rn(xv, d))));
    v = fminf(fmaxf(v, -128.0f), 127.0f);
    q[row * k + i] = (int8_t)(int)v;
  }
  if (threadIdx.x == 0) scale[row] = s;
}

// ---- stochastic rounding ----
// The reference's CUDA kernel (backends/cuda/ops/int8_linear.cu:78-90 noise, :186-193
// rounding): element idx = row * k + col of the contiguous [m, k] activation gets the
// counter-based noise u = bf16(float(pcg_hash(lo32(idx + seed) ^ hi32(idx + seed)) >> 8)
// * 2^-24) in [0, 1), and q = clamp(floor(bf16(bf16(x / bf16(scale)) + u)), -128, 127).
// pcg_hash is the PCG-based integer hash of Jarzynski and Olano ("Hash Functions for GPU
// Rendering", JCGT 2020): one LCG step, a data-dependent xorshift, a multiply and a
// final xorshift. The row scale is the deterministic quantizer's.
__device__ __forceinline__ uint32_t pcg_hash32(uint32_t x) {
  const uint32_t state = x * 747796405u + 2891336453u;
  const uint32_t word = ((state >> ((state >> 28u) + 4u)) ^ state) * 277803737u;
  return (word >> 22u) ^ word;
}
__device__ __forceinline__ float sr_noise_bf16(uint64_t idx, uint64_t seed) {
  const uint64_t key = idx + seed;
  const uint32_t folded = (uint32_t)key ^ (uint32_t)(key >> 32);
  return bf16_round((float)(pcg_hash32(folded) >> 8) * 0x1.0p-24f);
}

__global__ void __launch_bounds__(kQThreads) quantize_rows_stochastic_kernel(const __nv_bfloat16* __restrict__ x,
                                                                             int64_t ldx, int64_t m, int64_t k,
                                                                             int act, uint64_t seed,
                                                                             int8_t* __restrict__ q,
                                                                             float* __restrict__ scale) {
  __shared__ float red[kQThreads / 32];
  const int64_t row = blockIdx.x;
  if (row >= m) return;
  const __nv_bfloat16* xr = x + row * ldx;
  float amax = 0.0f;
  for (int64_t i = threadIdx.x; i < k; i += kQThreads) amax = fmaxf(amax, fabsf(act_value(xr, k, i, act)));
  const float s = row_scale(block_max(amax, red));
  const float sb = quant_divisor(s);
  for (int64_t i = threadIdx.x; i < k; i += kQThreads) {
    const float t = bf16_round(__fdiv_rn(act_value(xr, k, i, act), sb));
    float v = floorf(bf16_round(__fadd_rn(t, sr_noise_bf16((uint64_t)(row * k + i), seed))));
    v = fminf(fmaxf(v, -128.0f), 127.0f);
    q[row * k + i] = (int8_t)(int)v;
  }
  if (threadIdx.x == 0) scale[row] = s;
}

template <bool GIVEN>
cudaError_t launch_warp(int vpl, const __nv_bfloat16* x, int64_t ldx, int64_t m, int64_t k, int act, const float* am,
                        int8_t* q, float* s, cudaStream_t st) {
  const int64_t rows_per_block = kQThreads / 32;
  dim3 grid((unsigned)((m + rows_per_block - 1) / rows_per_block)), block(kQThreads);
  switch (vpl) {
    case 2: quantize_rows_warp_kernel<2, GIVEN><<<grid, block, 0, st>>>(x, ldx, m, k, act, am, q, s); break;
    case 4: quantize_rows_warp_kernel<4, GIVEN><<<grid, block, 0, st>>>(x, ldx, m, k, act, am, q, s); break;
    case 8: quantize_rows_warp_kernel<8, GIVEN><<<grid, block, 0, st>>>(x, ldx, m, k, act, am, q, s); break;
    case 12: quantize_rows_warp_kernel<12, GIVEN><<<grid, block, 0, st>>>(x, ldx, m, k, act, am, q, s); break;
    default: quantize_rows_warp_kernel<16, GIVEN><<<grid, block, 0, st>>>(x, ldx, m, k, act, am, q, s); break;
  }
  return cudaGetLastError();
}

template <bool GIVEN>
cudaError_t launch_vec(int vpt, const __nv_bfloat16* x, int64_t ldx, int64_t m, int64_t k, int act, const float* am,
                       int8_t* q, float* s, cudaStream_t st) {
  dim3 grid((unsigned)m), block(kQThreads);
  switch (vpt) {
    case 1: quantize_rows_vec_kernel<1, GIVEN><<<grid, block, 0, st>>>(x, ldx, m, k, act, am, q, s); break;
    case 2: quantize_rows_vec_kernel<2, GIVEN><<<grid, block, 0, st>>>(x, ldx, m, k, act, am, q, s); break;
    case 4: quantize_rows_vec_kernel<4, GIVEN><<<grid, block, 0, st>>>(x, ldx, m, k, act, am, q, s); break;
    case 6: quantize_rows_vec_kernel<6, GIVEN><<<grid, block, 0, st>>>(x, ldx, m, k, act, am, q, s); break;
    default: quantize_rows_vec_kernel<8, GIVEN><<<grid, block, 0, st>>>(x, ldx, m, k, act, am, q, s); break;
  }
  return cudaGetLastError();
}

__global__ void apply_act_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y, int64_t n,
                                 int act) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = __float2bfloat16_rn(act_apply(__bfloat162float(x[i]), act));
}

// y[m, k] = silu(x[:, :k]) * x[:, k:2k] (bf16, the reference's two roundings)
__global__ void swiglu_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, __nv_bfloat16* __restrict__ y,
                                   int64_t ldy, int64_t m, int64_t k) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= m * k) return;
  const int64_t row = i / k, col = i - row * k;
  y[row * ldy + col] = __float2bfloat16_rn(act_value(x + row * ldx, k, col, H3B200_ACT_SWIGLU));
}

// out = bf16(residual + bf16(float(acc) * (xs[row] * ws[col])) * gate[col]); 8 columns per thread.
__global__ void dequant_gated_residual_kernel(const int32_t* __restrict__ acc, const float* __restrict__ xs,
                                              const float* __restrict__ ws, const __nv_bfloat16* __restrict__ gate,
                                              const __nv_bfloat16* residual, int64_t ldr, __nv_bfloat16* out,
                                              int64_t ldo, int64_t m, int64_t n) {
  const int64_t per_row = n / 8;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= m * per_row) return;
  const int64_t row = idx / per_row;
  const int64_t c = (idx - row * per_row) * 8;
  const float x = xs[row];
  const uint4 a0 = *reinterpret_cast<const uint4*>(acc + row * n + c);
  const uint4 a1 = *reinterpret_cast<const uint4*>(acc + row * n + c + 4);
  const uint32_t av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
  const uint4 rv = ldg_v4(residual + row * ldr + c);
  const uint4 gv = ldg_nc_v4(gate + c);
  const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
  const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float y0 = bf16_round(__fmul_rn(__int2float_rn((int)av[2 * e]), __fmul_rn(x, ws[c + 2 * e])));
    float y1 = bf16_round(__fmul_rn(__int2float_rn((int)av[2 * e + 1]), __fmul_rn(x, ws[c + 2 * e + 1])));
    o[e] = pack_bf16(__fadd_rn(bf16_lo(rw[e]), __fmul_rn(y0, bf16_lo(gw[e]))),
                     __fadd_rn(bf16_hi(rw[e]), __fmul_rn(y1, bf16_hi(gw[e]))));
  }
  stg_v4(out + row * ldo + c, make_uint4(o[0], o[1], o[2], o[3]));
}

__global__ void act_table_init_kernel(int act) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 65536u) return;
  const float x = __uint_as_float(i << 16);
  if (act == H3B200_ACT_SWIGLU)
    g_silu_bf16[i] = bf16_bits(silu_exact(x));
  else
    g_gelu_bf16[i] = bf16_bits(gelu_tanh_exact(x));
}

}  // namespace

__device__ uint16_t g_gelu_bf16[65536];
__device__ uint16_t g_silu_bf16[65536];

cudaError_t ensure_act_table(int act, cudaStream_t stream) {
  if (act != H3B200_ACT_GELU_TANH && act != H3B200_ACT_SWIGLU) return cudaSuccess;
  static std::mutex mu;
  static bool ready[64][3] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (ready[dev][act]) return cudaSuccess;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if ((e = cudaStreamIsCapturing(stream, &cap)) != cudaSuccess) return e;
  if (cap != cudaStreamCaptureStatusNone) return cudaErrorStreamCaptureUnsupported;
  act_table_init_kernel<<<256, 256, 0, stream>>>(act);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  if ((e = cudaStreamSynchronize(stream)) != cudaSuccess) return e;
  ready[dev][act] = true;
  return cudaSuccess;
}

cudaError_t ensure_gelu_table(cudaStream_t stream) { return ensure_act_table(H3B200_ACT_GELU_TANH, stream); }

cudaError_t launch_dequant_gated_residual(const int32_t* acc, const float* xs, const float* ws, const void* gate,
                                          const void* residual, int64_t ldr, void* out, int64_t ldo, int64_t m,
                                          int64_t n, cudaStream_t stream) {
  if (m == 0 || n == 0) return cudaSuccess;
  if (n % 8 || ldr % 8 || ldo % 8 || (reinterpret_cast<uintptr_t>(acc) & 15) ||
      (reinterpret_cast<uintptr_t>(residual) & 15) || (reinterpret_cast<uintptr_t>(out) & 15) ||
      (reinterpret_cast<uintptr_t>(gate) & 15))
    return cudaErrorNotSupported;
  const int64_t total = m * (n / 8);
  dequant_gated_residual_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(
      acc, xs, ws, static_cast<const __nv_bfloat16*>(gate), static_cast<const __nv_bfloat16*>(residual), ldr,
      static_cast<__nv_bfloat16*>(out), ldo, m, n);
  return cudaGetLastError();
}

cudaError_t launch_swiglu_rows(const void* x, int64_t ldx, void* y, int64_t ldy, int64_t m, int64_t k,
                               cudaStream_t stream) {
  if (m == 0 || k == 0) return cudaSuccess;
  const cudaError_t e = ensure_act_table(H3B200_ACT_SWIGLU, stream);
  if (e != cudaSuccess) return e;
  const int64_t n = m * k;
  swiglu_rows_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), ldx,
                                                                     static_cast<__nv_bfloat16*>(y), ldy, m, k);
  return cudaGetLastError();
}

cudaError_t launch_apply_act(const void* x, void* y, int64_t n, int act, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  if (act == H3B200_ACT_SWIGLU) return cudaErrorNotSupported;  // row-structured: launch_swiglu_rows
  if (act == H3B200_ACT_GELU_TANH) {
    const cudaError_t e = ensure_gelu_table(stream);
    if (e != cudaSuccess) return e;
  }
  apply_act_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x),
                                                                   static_cast<__nv_bfloat16*>(y), n, act);
  return cudaGetLastError();
}

cudaError_t launch_quantize_rows(const void* x, int64_t ldx, int64_t m, int64_t k, int act, const float* absmax_in,
                                 int8_t* q, float* scale, cudaStream_t stream) {
  if (m == 0) return cudaSuccess;
  {
    const cudaError_t e = ensure_act_table(act, stream);
    if (e != cudaSuccess) return e;
  }
  const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
  const bool aligned = (k % 8 == 0) && (ldx % 8 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0) &&
                       ((reinterpret_cast<uintptr_t>(q) & 7) == 0);
  const int64_t nvec = k / 8;
  if (aligned && k > 0 && nvec <= 32 * 16) {
    const int64_t per_lane = (nvec + 31) / 32;
    const int vpl = per_lane <= 2 ? 2 : per_lane <= 4 ? 4 : per_lane <= 8 ? 8 : per_lane <= 12 ? 12 : 16;
    if (absmax_in != nullptr) return launch_warp<true>(vpl, xb, ldx, m, k, act, absmax_in, q, scale, stream);
    return launch_warp<false>(vpl, xb, ldx, m, k, act, nullptr, q, scale, stream);
  }
  const int64_t per_thread = (nvec + kQThreads - 1) / kQThreads;
  if (aligned && k > 0 && per_thread <= 8) {
    const int vpt = per_thread <= 1 ? 1 : per_thread <= 2 ? 2 : per_thread <= 4 ? 4 : per_thread <= 6 ? 6 : 8;
    if (absmax_in != nullptr) return launch_vec<true>(vpt, xb, ldx, m, k, act, absmax_in, q, scale, stream);
    return launch_vec<false>(vpt, xb, ldx, m, k, act, nullptr, q, scale, stream);
  }
  quantize_rows_scalar_kernel<<<dim3((unsigned)m), dim3(kQThreads), 0, stream>>>(xb, ldx, m, k, act, absmax_in, q,
                                                                                  scale);
  return cudaGetLastError();
}

cudaError_t launch_quantize_rows_f16(const void* x, int64_t ldx, int64_t m, int64_t k, int8_t* q, float* scale,
                                     cudaStream_t stream) {
  if (m == 0) return cudaSuccess;
  quantize_rows_f16_kernel<<<dim3((unsigned)m), dim3(kQThreads), 0, stream>>>(static_cast<const __half*>(x), ldx, m,
                                                                                k, q, scale);
  return cudaGetLastError();
}

cudaError_t launch_quantize_rows_stochastic(const void* x, int64_t ldx, int64_t m, int64_t k, int act,
                                            uint64_t seed, int8_t* q, float* scale, cudaStream_t stream) {
  if (m == 0) return cudaSuccess;
  {
    const cudaError_t e = ensure_act_table(act, stream);
    if (e != cudaSuccess) return e;
  }
  quantize_rows_stochastic_kernel<<<dim3((unsigned)m), dim3(kQThreads), 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, m, k, act, seed, q, scale);
  return cudaGetLastError();
}

}  // namespace h3
