// Standalone RMS-AdaLN on the hidden stream (HBM-bound), with per-token
// modulation rows:
//   h   = bf16((x * rstd) * w)         (F.rms_norm; without a weight, bf16(x * rstd))
//   out = bf16(bf16(h * bf16(1 + scale[r])) + shift[r])
// where r is the modulation row of the token: row_map[t], or t / tokens_per_row
// (comfy_kitchen's per-sample broadcast of [B, 1, D] scale/shift), or 0.
//
// Reference semantics:
//  * H3's rms_adaln (h3serve/native_engine/model/kernels.py:7586-7634): the
//    RMSNorm module (layers.py:33-48, F.rms_norm with the weight cast to the
//    activation dtype), then per modulation segment
//    hidden[start:stop].mul_(1.0 + scale[row].to(bf16)).add_(shift[row].to(bf16))
//    -- the three bf16 materialisations that its Triton kernel
//    _segmented_rms_adaln_kernel (backends/original/kernels/fused_norm_rope.py:12-44)
//    also keeps.
//  * comfy_kitchen rms_adaln(x, scale, shift, eps) (__init__.py:130-150, eager
//    backends/eager/adaln.py:17-20): F.rms_norm without a weight, then
//    normalized * (1 + scale) + shift in bf16.
//
// B200 design: a persistent CTA per SM. One producer thread streams the CTA's
// tokens (t = blockIdx.x + j * gridDim.x) into a shared-memory ring of one-row
// stages with cp.async.bulk (no multicast); C consumer warps take every C-th
// token of the CTA. The ring has k * C stages and token j uses stage j % (k C),
// so every stage is only ever used by the warp j % C: a warp waits for the
// stage's next fill only after consuming its previous one, so an mbarrier
// parity wait can never pass on the phase before it. A warp reads its row from
// the stage twice -- sum of squares in double (reduced with shuffles), then
// normalise / modulate with packed f32x2 and bf16x2 operations -- and writes
// 128-bit stores. Lane l owns the 16-byte vectors l + 32 j. The norm weight is
// staged once per CTA in shared memory as fp32; modulation rows are read
// through the read-only L1 path (a handful of rows serve every token).
// Every mbarrier wait is bounded (2 s); on expiry the kernel records a status
// code and unwinds (common.cuh).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "norm_math.cuh"
#include "quant_math.cuh"

namespace h3 {
namespace {

constexpr int kRAMaxConsumers = 14;
constexpr int kRAMaxStages = 32;
constexpr int kRASmemLimit = 227 * 1024;
constexpr int kRAWeightOff = 1024;  // after the mbarriers
constexpr unsigned kErrRAFull = 0x401, kErrRAProducer = 0x402, kErrRADrain = 0x403;

struct RAParams {
  const __nv_bfloat16* x;
  __nv_bfloat16* y;
  int64_t ldx, ldy;
  const __nv_bfloat16* w;      // [d] or nullptr
  const __nv_bfloat16* scale;  // [rows, lds]
  const __nv_bfloat16* shift;  // [rows, ldh]
  int64_t lds, ldh;
  const int32_t* row_map;      // [m] or nullptr
  int64_t tokens_per_row;      // without a row map: row = t / tokens_per_row (<= 0: row 0)
  int64_t rows;
  int64_t m;
  int d, nvec, row_bytes, consumers, stages, ring_off;
  float eps;
};

__device__ __forceinline__ void ra_bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ uint64_t f2_from_float2(float2 v) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(v.x), "f"(v.y));
  return r;
}

// EXACT: nvec == 32 * VPL (every lane owns VPL vectors; no predicates).
template <int VPL, bool EXACT, bool HAS_W, bool MODULATE>
__global__ void __launch_bounds__(32 * (1 + kRAMaxConsumers), 1) rms_adaln_kernel(const RAParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty_bar = full_bar + kRAMaxStages;
  float2* wf = reinterpret_cast<float2*>(smem + kRAWeightOff);  // HAS_W: d / 2 fp32 pairs
  uint8_t* ring = smem + p.ring_off;
  const int nvec = EXACT ? 32 * VPL : p.nvec;
  const int C = p.consumers, S = p.stages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t G = gridDim.x;
  const int64_t cnt = p.m > blockIdx.x ? (p.m - blockIdx.x + G - 1) / G : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    fence_barrier_init();
  }
  if (HAS_W) {
    const uint32_t* w2 = reinterpret_cast<const uint32_t*>(p.w);
    for (int i = threadIdx.x; i < p.d / 2; i += blockDim.x) {
      const uint32_t v = __ldg(w2 + i);
      wf[i] = make_float2(bf16_lo(v), bf16_hi(v));
    }
  }
  __syncthreads();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer ----------------
      int64_t j = 0;
      for (; j < cnt; ++j) {
        const int s = (int)(j % S);
        const uint32_t use = (uint32_t)(j / S);
        if (!mbar_wait(&empty_bar[s], (use & 1u) ^ 1u, kErrRAProducer)) break;
        mbar_arrive_expect_tx(&full_bar[s], (uint32_t)p.row_bytes);
        ra_bulk_g2s(ring + (size_t)s * p.row_bytes, p.x + (blockIdx.x + j * G) * p.ldx, (uint32_t)p.row_bytes,
                    &full_bar[s]);
      }
      // every copy issued lands before the CTA may exit
      for (int64_t i = (j > S ? j - S : 0); i < j; ++i)
        mbar_wait(&full_bar[i % S], (uint32_t)(i / S) & 1u, kErrRADrain, 200000000ull);
    }
    return;
  }

  // ---------------- consumers ----------------
  const int cw = warp - 1;
  if (cw >= C) return;
  const uint32_t one2 = 0x3F803F80u;  // bf16x2 (1, 1)
  for (int64_t j = cw; j < cnt; j += C) {
    const int s = (int)(j % S);
    if (!mbar_wait(&full_bar[s], (uint32_t)(j / S) & 1u, kErrRAFull)) break;
    const uint4* xs = reinterpret_cast<const uint4*>(ring + (size_t)s * p.row_bytes);

    // ---- sum of squares (double) ----
    double acc[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
    for (int jj = 0; jj < VPL; ++jj) {
      const int vi = lane + 32 * jj;
      if (EXACT || vi < nvec) sumsq8_fast(xs[vi], acc);
    }
    double sum = (acc[0] + acc[1]) + (acc[2] + acc[3]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    float ms = (float)(sum / (double)p.d);
    if (!isfinite(ms)) {  // inf / NaN / huge row: exact conversions (warp-uniform branch)
      double ex[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll 1
      for (int jj = 0; jj < VPL; ++jj) {
        const int vi = lane + 32 * jj;
        if (EXACT || vi < nvec) sumsq8_exact(xs[vi], ex);
      }
      double se = (ex[0] + ex[1]) + (ex[2] + ex[3]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) se += __shfl_xor_sync(0xffffffffu, se, o);
      ms = (float)(se / (double)p.d);
    }
    const uint64_t rs2 = f2_dup(rms_rstd(ms, p.eps));

    // ---- normalise, modulate, store ----
    const int64_t tok = blockIdx.x + j * G;
    const __nv_bfloat16* scr = nullptr;
    const __nv_bfloat16* shr = nullptr;
    if (MODULATE) {
      int64_t r = p.row_map != nullptr ? (int64_t)__ldg(p.row_map + tok)
                                       : (p.tokens_per_row > 0 ? tok / p.tokens_per_row : 0);
      r = r < 0 ? 0 : (r >= p.rows ? p.rows - 1 : r);  // rows outside the table are clamped, never read
      scr = p.scale + r * p.lds;
      shr = p.shift + r * p.ldh;
    }
    __nv_bfloat16* yr = p.y + tok * p.ldy;
#pragma unroll
    for (int jj = 0; jj < VPL; ++jj) {
      const int vi = lane + 32 * jj;
      if (!EXACT && vi >= nvec) continue;
      const uint4 xv = xs[vi];
      uint4 mv = make_uint4(0, 0, 0, 0), sv = make_uint4(0, 0, 0, 0);
      if (MODULATE) {
        mv = ldg_nc_v4(scr + 8 * vi);
        sv = ldg_nc_v4(shr + 8 * vi);
      }
      const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
      const uint32_t mw[4] = {mv.x, mv.y, mv.z, mv.w};
      const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
      uint32_t h[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        uint64_t v = f2_mul(bf16x2_to_f2(xw[e]), rs2);
        if (HAS_W) v = f2_mul(v, f2_from_float2(wf[4 * vi + e]));
        uint32_t lo, hi;
        f2_bits(v, lo, hi);
        h[e] = bf16x2_from_bits(lo, hi);
        if (MODULATE) h[e] = bf2_add(bf2_mul(h[e], bf2_add(mw[e], one2)), sw[e]);
      }
      stg_v4(yr + 8 * vi, make_uint4(h[0], h[1], h[2], h[3]));
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[s]);  // every lane's reads of the stage are done
  }
}

template <int VPL, bool EXACT>
cudaError_t launch_ra(const RAParams& p, bool has_w, bool mod, int smem, int grid, cudaStream_t stream) {
  auto pick = [&](auto kernel) -> cudaError_t {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    kernel<<<grid, 32 * (1 + p.consumers), smem, stream>>>(p);
    return cudaGetLastError();
  };
  if (has_w && mod) return pick(rms_adaln_kernel<VPL, EXACT, true, true>);
  if (has_w) return pick(rms_adaln_kernel<VPL, EXACT, true, false>);
  if (mod) return pick(rms_adaln_kernel<VPL, EXACT, false, true>);
  return pick(rms_adaln_kernel<VPL, EXACT, false, false>);
}

}  // namespace

cudaError_t launch_rms_adaln(const RmsAdalnArgs& a, cudaStream_t stream) {
  if (a.m == 0) return cudaSuccess;
  if (a.d <= 0 || a.d % 8 || a.d > 8192 || a.ldx % 8 || a.ldy % 8 || a.ldx < a.d || a.ldy < a.d)
    return cudaErrorNotSupported;
  if (a.x == nullptr || a.y == nullptr || (reinterpret_cast<uintptr_t>(a.x) & 15) ||
      (reinterpret_cast<uintptr_t>(a.y) & 15))
    return cudaErrorNotSupported;
  const bool has_w = a.weight != nullptr;
  if (has_w && (reinterpret_cast<uintptr_t>(a.weight) & 3)) return cudaErrorNotSupported;
  const bool mod = a.scale != nullptr;
  if (mod && (a.shift == nullptr || a.rows <= 0 || a.lds % 8 || a.ldh % 8 || a.lds < a.d || a.ldh < a.d ||
              (reinterpret_cast<uintptr_t>(a.scale) & 15) || (reinterpret_cast<uintptr_t>(a.shift) & 15)))
    return cudaErrorNotSupported;
  RAParams p;
  p.x = static_cast<const __nv_bfloat16*>(a.x);
  p.y = static_cast<__nv_bfloat16*>(a.y);
  p.ldx = a.ldx;
  p.ldy = a.ldy;
  p.w = static_cast<const __nv_bfloat16*>(a.weight);
  p.scale = static_cast<const __nv_bfloat16*>(a.scale);
  p.shift = static_cast<const __nv_bfloat16*>(a.shift);
  p.lds = a.lds;
  p.ldh = a.ldh;
  p.row_map = a.row_map;
  p.tokens_per_row = a.tokens_per_row;
  p.rows = a.rows;
  p.m = a.m;
  p.d = (int)a.d;
  p.nvec = (int)(a.d / 8);
  p.row_bytes = (int)(a.d * 2);
  p.eps = a.eps;
  p.ring_off = (kRAWeightOff + (has_w ? (int)a.d * 4 : 0) + 127) & ~127;
  const int avail = kRASmemLimit - 128 - p.ring_off;
  // consumer warps: up to 14, fewer for very wide rows; stages: the largest multiple of the
  // consumer count (at most kRAMaxStages) whose rows fit
  int c = std::min(kRAMaxConsumers, avail / p.row_bytes);
  if (c < 1) return cudaErrorNotSupported;
  int k = std::max(1, std::min(kRAMaxStages / c, avail / (c * p.row_bytes)));
  p.consumers = c;
  p.stages = k * c;
  const int smem = 128 + p.ring_off + p.stages * p.row_bytes;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  const int grid = (int)std::min<int64_t>(sms, a.m);
  const int vpl = (p.nvec + 31) / 32;
  if (p.nvec == 32 * 12) return launch_ra<12, true>(p, has_w, mod, smem, grid, stream);   // d = 3072
  if (p.nvec == 32 * 21) return launch_ra<21, true>(p, has_w, mod, smem, grid, stream);   // d = 5376 (H3)
  if (vpl <= 4) return launch_ra<4, false>(p, has_w, mod, smem, grid, stream);
  if (vpl <= 8) return launch_ra<8, false>(p, has_w, mod, smem, grid, stream);
  if (vpl <= 16) return launch_ra<16, false>(p, has_w, mod, smem, grid, stream);
  return launch_ra<32, false>(p, has_w, mod, smem, grid, stream);
}

}  // namespace h3
