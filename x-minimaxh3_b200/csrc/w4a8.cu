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
    const uint2 q0 = quant_vec8(make_uint4(pw[0], pw[1], pw[2], pw[3]), sb, rcp);
    const uint2 q1 = quant_vec8(make_uint4(pw[4], pw[5], pw[6], pw[7]), sb, rcp);
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
  if (k % 256 || ldx % 8 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(q) & 15))
    return cudaErrorNotSupported;
  if (sx != nullptr && (sum_group < 16 || sum_group > 256 || 256 % sum_group || kp < k / sum_group))
    return cudaErrorNotSupported;
  if (act == H3B200_ACT_GELU_TANH) {
    const cudaError_t e = ensure_gelu_table(stream);
    if (e != cudaSuccess) return e;
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
