// Fused (AdaLN-modulate +) RMSNorm + split-half RoPE on Q and K (HBM-bound).
//
// Reference semantics:
//  * row span: rms_adaln -- F.rms_norm over the hidden row with weight, then
//    mul_(1 + scale) and add_(shift), bf16 after each step
//    (h3serve/native_engine/model/kernels.py:7586-7634, eager order :7623-7631),
//    followed by per-head split-half RoPE (backends/eager/rope.py:39-42).
//  * head span: rms_rope_split_half -- per-head RMSNorm then RoPE, partial
//    rotary through rot_dim (backends/eager/rope.py:67-143; CUDA kernel
//    backends/cuda/ops/rms_rope.cu:36-229).
// RMSNorm: rstd = 1 / sqrt(mean(x^2) + eps) in fp32, y = bf16((x * rstd) * w).
// The sum of squares is accumulated in double so the fp32 mean is the
// correctly rounded one (the reference sums in fp32, order ISA-dependent).
// RoPE: y0 = t00*x0 + t01*x1, y1 = t10*x0 + t11*x1 (fp32, two products and one
// add), bf16 store; table fp32 [m, rot_dim/2, 2, 2].
//
// B200 layout: one warp per token, persistent over tokens. Lane l owns the
// 16-byte vectors v = l + 32*j of the heads*128-wide row, so its position
// inside a head (v mod 16 = l mod 16) is the same for every j: the RoPE
// coefficients it needs are loaded once per token into registers and the
// rotation partner (vector v +- rot_dim/16, same head) sits in lane
// (l & 16) | partner, one shuffle away. Q and K rows of a token are loaded
// together (2 x 6 KB in flight per warp), each byte is read and written once.
#include "common.cuh"
#include "kernels.h"

namespace h3 {
namespace {

constexpr int kNRThreads = 256;

struct NRParams {
  const __nv_bfloat16* x[2];
  __nv_bfloat16* y[2];
  int64_t ldx[2], ldy[2];
  const __nv_bfloat16* w[2];
  const float* freqs;
  const __nv_bfloat16* scale;
  const __nv_bfloat16* shift;
  int64_t m;
  int heads;
  int half_v;   // rot_dim / 16: vectors in each rotation half
  int row_elems;
  float eps;
};

template <int VPL, bool ROW_SPAN, bool MODULATE>
__global__ void __launch_bounds__(kNRThreads) adaln_rms_rope_kernel(const NRParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = ((int64_t)blockIdx.x * kNRThreads + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * kNRThreads) >> 5;
  const int hv = lane & 15;
  const int nvec = p.heads * 16;
  // rotation role of this lane: 0 = first half, 1 = second half, 2 = passthrough
  const int role = hv < p.half_v ? 0 : (hv < 2 * p.half_v ? 1 : 2);
  const int partner = (lane & 16) | (role == 0 ? hv + p.half_v : (role == 1 ? hv - p.half_v : hv));
  const int pair0 = 8 * (role == 0 ? hv : hv - p.half_v);
  const int64_t freq_stride = (int64_t)p.half_v * 8 * 4;

  // head-span weights depend only on the lane's in-head position
  uint4 whead[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
  if (!ROW_SPAN) {
    whead[0] = ldg_nc_v4(p.w[0] + 8 * hv);
    whead[1] = ldg_nc_v4(p.w[1] + 8 * hv);
  }

  for (int64_t tok = gw; tok < p.m; tok += nw) {
    uint4 v[2][VPL];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const __nv_bfloat16* xr = p.x[t] + tok * p.ldx[t];
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const int vi = lane + 32 * j;
        v[t][j] = vi < nvec ? ldg_v4(xr + 8 * vi) : make_uint4(0, 0, 0, 0);
      }
    }
    // RoPE coefficients for this lane's 8 pairs: (t00, t01) or (t10, t11)
    float ca[8], cb[8];
    if (role != 2) {
      const float4* fr = reinterpret_cast<const float4*>(p.freqs + tok * freq_stride) + pair0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float4 c = __ldg(fr + e);
        ca[e] = role == 0 ? c.x : c.z;
        cb[e] = role == 0 ? c.y : c.w;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) ca[e] = cb[e] = 0.0f;
    }

#pragma unroll
    for (int t = 0; t < 2; ++t) {
      // ---- sum of squares (double) ----
      double ss[ROW_SPAN ? 1 : VPL];
#pragma unroll
      for (int j = 0; j < (ROW_SPAN ? 1 : VPL); ++j) ss[j] = 0.0;
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const uint32_t* w = reinterpret_cast<const uint32_t*>(&v[t][j]);
        double acc = 0.0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const double a = (double)bf16_lo(w[e]);
          const double b = (double)bf16_hi(w[e]);
          acc = fma(a, a, acc);
          acc = fma(b, b, acc);
        }
        ss[ROW_SPAN ? 0 : j] += acc;
      }
      float rstd[ROW_SPAN ? 1 : VPL];
      if (ROW_SPAN) {
        double s = ss[0];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        const float ms = (float)(s / (double)p.row_elems);
        rstd[0] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, p.eps)));
      } else {
#pragma unroll
        for (int j = 0; j < (ROW_SPAN ? 1 : VPL); ++j) {
          double s = ss[j];
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
          const float ms = (float)(s / 128.0);
          rstd[j] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, p.eps)));
        }
      }
      // ---- normalise, modulate, rotate, store ----
      __nv_bfloat16* yr = p.y[t] + tok * p.ldy[t];
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const int vi = lane + 32 * j;
        const bool ok = vi < nvec;
        const float rs = rstd[ROW_SPAN ? 0 : j];
        uint4 wv = whead[t], sv = make_uint4(0, 0, 0, 0), hv4 = make_uint4(0, 0, 0, 0);
        if (ok) {
          if (ROW_SPAN) wv = ldg_nc_v4(p.w[t] + 8 * vi);
          if (MODULATE) {
            sv = ldg_nc_v4(p.scale + 8 * vi);
            hv4 = ldg_nc_v4(p.shift + 8 * vi);
          }
        }
        const uint32_t* xw = reinterpret_cast<const uint32_t*>(&v[t][j]);
        const uint32_t* ww = reinterpret_cast<const uint32_t*>(&wv);
        const uint32_t* sw = reinterpret_cast<const uint32_t*>(&sv);
        const uint32_t* hw = reinterpret_cast<const uint32_t*>(&hv4);
        uint32_t nw4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float a = bf16_round(__fmul_rn(__fmul_rn(bf16_lo(xw[e]), rs), bf16_lo(ww[e])));
          float b = bf16_round(__fmul_rn(__fmul_rn(bf16_hi(xw[e]), rs), bf16_hi(ww[e])));
          if (MODULATE) {
            a = bf16_round(__fmul_rn(a, bf16_round(__fadd_rn(1.0f, bf16_lo(sw[e])))));
            b = bf16_round(__fmul_rn(b, bf16_round(__fadd_rn(1.0f, bf16_hi(sw[e])))));
            a = bf16_round(__fadd_rn(a, bf16_lo(hw[e])));
            b = bf16_round(__fadd_rn(b, bf16_hi(hw[e])));
          }
          nw4[e] = pack_bf16(a, b);
        }
        uint32_t pw[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) pw[e] = __shfl_sync(0xffffffffu, nw4[e], partner);
        uint32_t ow[4];
        if (role == 2) {
#pragma unroll
          for (int e = 0; e < 4; ++e) ow[e] = nw4[e];
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float o0 = bf16_lo(nw4[e]), o1 = bf16_hi(nw4[e]);
            const float q0 = bf16_lo(pw[e]), q1 = bf16_hi(pw[e]);
            float r0, r1;
            if (role == 0) {  // own = x0, partner = x1
              r0 = __fadd_rn(__fmul_rn(ca[2 * e], o0), __fmul_rn(cb[2 * e], q0));
              r1 = __fadd_rn(__fmul_rn(ca[2 * e + 1], o1), __fmul_rn(cb[2 * e + 1], q1));
            } else {          // own = x1, partner = x0
              r0 = __fadd_rn(__fmul_rn(ca[2 * e], q0), __fmul_rn(cb[2 * e], o0));
              r1 = __fadd_rn(__fmul_rn(ca[2 * e + 1], q1), __fmul_rn(cb[2 * e + 1], o1));
            }
            ow[e] = pack_bf16(r0, r1);
          }
        }
        if (ok) stg_v4(yr + 8 * vi, make_uint4(ow[0], ow[1], ow[2], ow[3]));
      }
    }
  }
}

template <int VPL>
cudaError_t launch_vpl(const NRParams& p, bool row, bool mod, cudaStream_t st) {
  int dev = 0;
  cudaGetDevice(&dev);
  int per_sm = 1;
  auto go = [&](auto kern) -> cudaError_t {
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kNRThreads, 0);
    if (per_sm < 1) per_sm = 1;
    const int64_t warps_needed = p.m;
    int64_t blocks = (int64_t)num_sms(dev) * per_sm;
    const int64_t max_blocks = (warps_needed + (kNRThreads / 32) - 1) / (kNRThreads / 32);
    if (blocks > max_blocks) blocks = max_blocks;
    if (blocks < 1) blocks = 1;
    kern<<<(unsigned)blocks, kNRThreads, 0, st>>>(p);
    return cudaGetLastError();
  };
  if (row && mod) return go(adaln_rms_rope_kernel<VPL, true, true>);
  if (row) return go(adaln_rms_rope_kernel<VPL, true, false>);
  if (mod) return go(adaln_rms_rope_kernel<VPL, false, true>);
  return go(adaln_rms_rope_kernel<VPL, false, false>);
}

}  // namespace

cudaError_t launch_adaln_rms_rope(const NormRopeArgs& a, cudaStream_t stream) {
  if (a.m == 0) return cudaSuccess;
  const int64_t rot = a.rot_dim == 0 ? a.head_dim : a.rot_dim;
  if (a.head_dim != 128 || rot % 16 != 0 || rot <= 0 || rot > 128 || a.heads <= 0 || a.heads > 32)
    return cudaErrorNotSupported;
  const void* ptrs[6] = {a.q, a.k, a.q_out, a.k_out, a.q_weight, a.k_weight};
  for (const void* ptr : ptrs)
    if (ptr == nullptr || (reinterpret_cast<uintptr_t>(ptr) & 15)) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(a.freqs) & 15) || a.freqs == nullptr) return cudaErrorNotSupported;
  if (a.ldq % 8 || a.ldk % 8 || a.ldqo % 8 || a.ldko % 8) return cudaErrorNotSupported;
  const bool mod = a.scale != nullptr;
  if (mod && (a.shift == nullptr || (reinterpret_cast<uintptr_t>(a.scale) & 15) ||
              (reinterpret_cast<uintptr_t>(a.shift) & 15)))
    return cudaErrorNotSupported;
  if (a.norm_span == 0 && !mod) {
    // plain RMSNorm over the row is allowed (no modulation)
  }
  NRParams p;
  p.x[0] = static_cast<const __nv_bfloat16*>(a.q);
  p.x[1] = static_cast<const __nv_bfloat16*>(a.k);
  p.y[0] = static_cast<__nv_bfloat16*>(a.q_out);
  p.y[1] = static_cast<__nv_bfloat16*>(a.k_out);
  p.ldx[0] = a.ldq;
  p.ldx[1] = a.ldk;
  p.ldy[0] = a.ldqo;
  p.ldy[1] = a.ldko;
  p.w[0] = static_cast<const __nv_bfloat16*>(a.q_weight);
  p.w[1] = static_cast<const __nv_bfloat16*>(a.k_weight);
  p.freqs = a.freqs;
  p.scale = static_cast<const __nv_bfloat16*>(a.scale);
  p.shift = static_cast<const __nv_bfloat16*>(a.shift);
  p.m = a.m;
  p.heads = (int)a.heads;
  p.half_v = (int)(rot / 16);
  p.row_elems = (int)(a.heads * a.head_dim);
  p.eps = a.eps;
  const bool row = a.norm_span == 0;
  const int vpl = (int)((a.heads * 16 + 31) / 32);
  if (vpl <= 4) return launch_vpl<4>(p, row, mod, stream);
  if (vpl <= 8) return launch_vpl<8>(p, row, mod, stream);
  if (vpl <= 12) return launch_vpl<12>(p, row, mod, stream);
  return launch_vpl<16>(p, row, mod, stream);
}

}  // namespace h3
