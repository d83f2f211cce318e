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
// |x| is turned into a double with two integer operations on its bf16 bits
// (exact for normal values; zero and subnormals become a value below 2^-126
// whose square cannot change the fp32 mean); a row whose mean is not finite
// is re-summed with exact conversions, so inf and NaN behave as in the reference.
// Modulation: bf16(bf16(h * bf16(1 + scale)) + shift); both steps are one
// correctly rounded bf16x2 operation on bf16 operands, which equals the
// reference's fp32 operation followed by a bf16 rounding (the fp32 product of
// two bf16 values is exact, and the fp32 sum of two bf16 values rounds to the
// same bf16 value as the exact sum).
// RoPE: y0 = t00*x0 + t01*x1, y1 = t10*x0 + t11*x1 (fp32, two products and one
// add, no fusion), bf16 store; table fp32 [m, rot_dim/2, 2, 2].
//
// B200 design: a persistent CTA per SM streams tokens through a shared-memory
// ring with asynchronous copies (no multicast): one producer thread loads a
// token's Q row and K row with cp.async.bulk and its rotation-table row with a
// 128-byte-swizzled TMA tensor load (the swizzle lets the 8 lanes that read 8
// different 128-byte table segments hit 8 different bank groups); each of
// kPairs warp pairs takes every kPairs-th token of the CTA, one warp for Q and
// one for K. A warp reads its row from the stage twice (sum of
// squares, reduced with shuffles; then normalise / modulate / rotate; lane l
// owns the 16-byte vectors l + 32*j), writes the result with coalesced 128-bit
// stores and frees the stage. Lane l's
// position inside a head (l mod 16) is the same for every j, so its RoPE
// coefficients are read once per token and its rotation partner (vector
// v +- rot_dim/16 of the same head) is one shuffle away. Per-column weights,
// bf16(1 + scale) and shift are staged in shared memory once per CTA. The
// normalisation and RoPE products use the packed f32x2 multiply of sm_100
// (two IEEE round-to-nearest products per instruction). The RoPE sums stay
// scalar: a packed multiply followed by a packed add was measured to round like
// a fused multiply-add (last-bit differences in about 1 of 10^5 outputs), even
// with contraction disabled. Row weights are staged as fp32 pairs, and the
// 24-head (3072-wide) case is a separate instantiation without per-vector
// predicates.
#include "common.cuh"
#include "kernels.h"
#include "norm_math.cuh"

namespace h3 {
namespace {

constexpr int kPairs = 7;                          // consumer warp pairs per CTA
constexpr int kNRThreads = 32 * (1 + 2 * kPairs);  // producer warp + consumers
constexpr int kMaxStages = 14;
constexpr int kSmemLimit = 227 * 1024;
constexpr unsigned kErrNRFull = 0x201, kErrNRProducer = 0x202, kErrNRDrain = 0x203;

struct NRParams {
  const __nv_bfloat16* x[2];
  __nv_bfloat16* y[2];
  int64_t ldx[2], ldy[2];
  const __nv_bfloat16* w[2];
  const float* freqs;
  const __nv_bfloat16* scale;
  const __nv_bfloat16* shift;
  // per-token modulation rows (MOD == 2): row_map[t] (clamped to [0, mod_rows)), else
  // t / tokens_per_row (<= 0: row 0); row strides lds / ldh elements
  const int32_t* row_map;
  int64_t tokens_per_row, mod_rows, lds, ldh;
  int64_t m;
  int heads;
  int half_v;     // rot_dim / 16: vectors in each rotation half
  int row_elems;
  int row_bytes;    // heads * 256
  int nseg;         // rot_dim / 16: 128-byte table segments (8 pairs each) per token
  int tab_off;      // table offset inside a stage (1024-aligned for the swizzle)
  int stage_bytes;  // multiple of 1024
  int ring_off;     // ring offset from the 1024-aligned shared-memory base
  int stages;
  float eps;
};

// ---- packed arithmetic -----------------------------------------------------
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
// two fp32 (packed) -> bf16x2 (low half from the low float), round to nearest even
__device__ __forceinline__ uint32_t f2_to_bf16x2(uint64_t v) {
  uint32_t r, lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=r"(lo), "=r"(hi) : "l"(v));
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "r"(hi), "r"(lo));
  return r;
}
// bf16x2 -> two fp32 (packed)
__device__ __forceinline__ uint64_t bf16x2_to_f2(uint32_t w) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(w << 16), "r"(w & 0xFFFF0000u));
  return r;
}
// ---- bulk copy global -> shared, completion counted on an mbarrier ---------
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// EXACT: heads * 16 == 32 * VPL, every lane's VPL vectors exist (no predicates).
// MOD: 0 no modulation, 1 one row (bf16(1 + scale) and shift staged in shared
// memory), 2 a row per token (read through the read-only L1 path).
template <int VPL, bool ROW_SPAN, int MOD, bool FULL_ROT, bool EXACT>
__global__ void __launch_bounds__(kNRThreads, 1)
    adaln_rms_rope_kernel(const __grid_constant__ CUtensorMap tm_table, const NRParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nvec = EXACT ? 32 * VPL : p.heads * 16;
  const int S = p.stages;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty_bar = full_bar + kMaxStages;
  // ROW_SPAN: fp32 weights of Q (wf[0, nvec)) and K (wf[nvec, 2 nvec)), 8 per vector
  float4* wf = reinterpret_cast<float4*>(smem + 256);
  constexpr bool MODULATE = MOD != 0;
  uint4* m_s = reinterpret_cast<uint4*>(wf + (ROW_SPAN ? 4 : 0) * nvec);  // MOD 1: bf16(1 + scale)
  uint4* sh_s = m_s + nvec;                                                 // MOD 1: shift
  uint8_t* ring = smem + p.ring_off;
  const int stage_bytes = p.stage_bytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t G = gridDim.x;
  const int64_t cnt = p.m > blockIdx.x ? (p.m - blockIdx.x + G - 1) / G : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 2);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tm_table);
  }
  for (int i = threadIdx.x; i < nvec; i += kNRThreads) {
    if (ROW_SPAN) {
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const uint4 w = ldg_nc_v4(p.w[t] + 8 * i);
        wf[(t * nvec + i) * 2] = make_float4(bf16_lo(w.x), bf16_hi(w.x), bf16_lo(w.y), bf16_hi(w.y));
        wf[(t * nvec + i) * 2 + 1] = make_float4(bf16_lo(w.z), bf16_hi(w.z), bf16_lo(w.w), bf16_hi(w.w));
      }
    }
    if (MOD == 1) {
      const uint4 sc = ldg_nc_v4(p.scale + 8 * i);
      const uint32_t* sw = reinterpret_cast<const uint32_t*>(&sc);
      uint4 mv;
      uint32_t* mw = reinterpret_cast<uint32_t*>(&mv);
#pragma unroll
      for (int e = 0; e < 4; ++e) mw[e] = pack_bf16(__fadd_rn(1.0f, bf16_lo(sw[e])), __fadd_rn(1.0f, bf16_hi(sw[e])));
      m_s[i] = mv;
      sh_s[i] = ldg_nc_v4(p.shift + 8 * i);
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
        if (!mbar_wait(&empty_bar[s], (use & 1u) ^ 1u, kErrNRProducer)) break;
        const int64_t tok = blockIdx.x + j * G;
        uint8_t* st = ring + (size_t)s * stage_bytes;
        mbar_arrive_expect_tx(&full_bar[s], (uint32_t)(2 * p.row_bytes + p.nseg * 128));
        bulk_g2s(st, p.x[0] + tok * p.ldx[0], (uint32_t)p.row_bytes, &full_bar[s]);
        bulk_g2s(st + p.row_bytes, p.x[1] + tok * p.ldx[1], (uint32_t)p.row_bytes, &full_bar[s]);
        tma_load_2d(st + p.tab_off, &tm_table, &full_bar[s], 0, (int32_t)(tok * p.nseg));
      }
      // every copy issued lands before the CTA may exit
      for (int64_t i = (j > S ? j - S : 0); i < j; ++i)
        mbar_wait(&full_bar[i % S], (uint32_t)(i / S) & 1u, kErrNRDrain, 200000000ull);
    }
    return;
  }

  // ---------------- consumers ----------------
  const int cw = warp - 1;
  const int pair = cw >> 1;
  const int t = cw & 1;  // 0 = Q, 1 = K
  const int hv = lane & 15;
  const int half_v = p.half_v;
  const int role = hv < half_v ? 0 : (hv < 2 * half_v ? 1 : 2);  // first half, second half, pass-through
  const int partner = (lane & 16) | (role == 0 ? hv + half_v : (role == 1 ? hv - half_v : hv));
  const int pair0 = 8 * (role == 0 ? hv : (role == 1 ? hv - half_v : 0));

  const float4* w_row = wf + 2 * t * nvec;
  uint4 whead = make_uint4(0, 0, 0, 0);
  if (!ROW_SPAN) whead = ldg_nc_v4(p.w[t] + 8 * hv);
  __nv_bfloat16* const ybase = p.y[t];
  const int64_t ldy = p.ldy[t];

  for (int64_t j = pair; j < cnt; j += kPairs) {
    const int s = (int)(j % S);
    if (!mbar_wait(&full_bar[s], (uint32_t)(j / S) & 1u, kErrNRFull)) break;
    const uint8_t* st = ring + (size_t)s * stage_bytes;
    const uint4* xs = reinterpret_cast<const uint4*>(st + t * p.row_bytes);
    // RoPE coefficients of this lane's 8 pairs: out = A * own + B * partner.
    // Table segment `seg` (pairs 8 seg .. 8 seg + 7) holds 16-byte chunk c at
    // c ^ seg (128-byte swizzle).
    uint64_t A[4], B[4];
    if (role != 2) {
      const int seg = pair0 >> 3;
      const uint8_t* tb = st + p.tab_off + seg * 128;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float4 c0 = *reinterpret_cast<const float4*>(tb + (((2 * e) ^ seg) << 4));
        const float4 c1 = *reinterpret_cast<const float4*>(tb + (((2 * e + 1) ^ seg) << 4));
        // role 0 (x0): t00 * x0 + t01 * x1; role 1 (x1): t11 * x1 + t10 * x0
        A[e] = role == 0 ? f2_pack(c0.x, c1.x) : f2_pack(c0.w, c1.w);
        B[e] = role == 0 ? f2_pack(c0.y, c1.y) : f2_pack(c0.z, c1.z);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) A[e] = B[e] = 0;
    }

    // ---- sum of squares (double) ----
    float rstd[ROW_SPAN ? 1 : VPL];
    if (ROW_SPAN) {
      double acc[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
      for (int jj = 0; jj < VPL; ++jj) {
        const int vi = lane + 32 * jj;
        sumsq8_fast((EXACT || vi < nvec) ? xs[vi] : make_uint4(0, 0, 0, 0), acc);
      }
      double sum = (acc[0] + acc[1]) + (acc[2] + acc[3]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      float ms = (float)(sum / (double)p.row_elems);
      if (!isfinite(ms)) {  // inf / NaN / huge row: exact conversions (warp-uniform branch)
        double ex[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll 1
        for (int jj = 0; jj < VPL; ++jj) {
          const int vi = lane + 32 * jj;
          sumsq8_exact((EXACT || vi < nvec) ? xs[vi] : make_uint4(0, 0, 0, 0), ex);
        }
        double se = (ex[0] + ex[1]) + (ex[2] + ex[3]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) se += __shfl_xor_sync(0xffffffffu, se, o);
        ms = (float)(se / (double)p.row_elems);
      }
      rstd[0] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, p.eps)));
    } else {
#pragma unroll
      for (int jj = 0; jj < (ROW_SPAN ? 1 : VPL); ++jj) {
        const int vi = lane + 32 * jj;
        const uint4 xv = (EXACT || vi < nvec) ? xs[vi] : make_uint4(0, 0, 0, 0);
        double acc[4] = {0.0, 0.0, 0.0, 0.0};
        sumsq8_fast(xv, acc);
        double sum = (acc[0] + acc[1]) + (acc[2] + acc[3]);
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        float ms = (float)(sum / 128.0);
        const bool bad = !isfinite(ms);
        if (__any_sync(0xffffffffu, bad)) {
          double ex[4] = {0.0, 0.0, 0.0, 0.0};
          sumsq8_exact(xv, ex);
          double se = (ex[0] + ex[1]) + (ex[2] + ex[3]);
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) se += __shfl_xor_sync(0xffffffffu, se, o);
          if (bad) ms = (float)(se / 128.0);
        }
        rstd[jj] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, p.eps)));
      }
    }

    // ---- normalise, modulate, rotate, store ----
    const int64_t tok = blockIdx.x + j * G;
    __nv_bfloat16* yr = ybase + tok * ldy;
    const __nv_bfloat16* scr = nullptr;
    const __nv_bfloat16* shr = nullptr;
    if (MOD == 2) {
      int64_t r = p.row_map != nullptr ? (int64_t)__ldg(p.row_map + tok)
                                       : (p.tokens_per_row > 0 ? tok / p.tokens_per_row : 0);
      r = r < 0 ? 0 : (r >= p.mod_rows ? p.mod_rows - 1 : r);  // rows outside the table are clamped
      scr = p.scale + r * p.lds;
      shr = p.shift + r * p.ldh;
    }
#pragma unroll
    for (int jj = 0; jj < VPL; ++jj) {
      const int vi = lane + 32 * jj;
      const bool ok = EXACT || vi < nvec;
      const int vc = ok ? vi : 0;
      const float rs = rstd[ROW_SPAN ? 0 : jj];
      const uint64_t rs2 = f2_pack(rs, rs);
      uint64_t wpair[4];  // fp32 weight pairs of this vector
      if (ROW_SPAN) {
        const float4 w0 = w_row[2 * vc], w1 = w_row[2 * vc + 1];
        wpair[0] = f2_pack(w0.x, w0.y); wpair[1] = f2_pack(w0.z, w0.w);
        wpair[2] = f2_pack(w1.x, w1.y); wpair[3] = f2_pack(w1.z, w1.w);
      } else {
        wpair[0] = bf16x2_to_f2(whead.x); wpair[1] = bf16x2_to_f2(whead.y);
        wpair[2] = bf16x2_to_f2(whead.z); wpair[3] = bf16x2_to_f2(whead.w);
      }
      uint4 mv = make_uint4(0, 0, 0, 0), sv = make_uint4(0, 0, 0, 0);
      if (MOD == 1) {
        mv = m_s[vc];
        sv = sh_s[vc];
      } else if (MOD == 2) {
        const uint4 sc = ldg_nc_v4(scr + 8 * vc);
        mv = make_uint4(bf2_add(sc.x, 0x3F803F80u), bf2_add(sc.y, 0x3F803F80u), bf2_add(sc.z, 0x3F803F80u),
                        bf2_add(sc.w, 0x3F803F80u));  // bf16(1 + scale)
        sv = ldg_nc_v4(shr + 8 * vc);
      }
      const uint4 xv = xs[vc];
      const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xv);
      const uint32_t* mw = reinterpret_cast<const uint32_t*>(&mv);
      const uint32_t* sw = reinterpret_cast<const uint32_t*>(&sv);
      uint32_t h[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        h[e] = f2_to_bf16x2(f2_mul(f2_mul(bf16x2_to_f2(xw[e]), rs2), wpair[e]));
        if (MODULATE) h[e] = bf2_add(bf2_mul(h[e], mw[e]), sw[e]);
      }
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t pw = __shfl_sync(0xffffffffu, h[e], partner);
        // packed round-to-nearest products, scalar adds (a packed add after a
        // packed multiply was measured to round like a fused multiply-add)
        float p0, p1, q0, q1;
        f2_unpack(f2_mul(A[e], bf16x2_to_f2(h[e])), p0, p1);
        f2_unpack(f2_mul(B[e], bf16x2_to_f2(pw)), q0, q1);
        o[e] = pack_bf16(__fadd_rn(p0, q0), __fadd_rn(p1, q1));
        if (!FULL_ROT && role == 2) o[e] = h[e];
      }
      if (ok) stg_v4(yr + 8 * vi, make_uint4(o[0], o[1], o[2], o[3]));
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[s]);  // every lane's reads of the stage are done
  }
}

int ring_offset(int nvec, bool row, bool mod) {
  const int cst_bytes = (row ? 2 * nvec * 32 : 0) + (mod ? 2 * nvec * 16 : 0);
  return (256 + cst_bytes + 1023) & ~1023;
}

template <int VPL, bool ROW, int MOD, bool FULL, bool EXACT>
cudaError_t launch_one(const CUtensorMap& tm, const NRParams& p, int smem, cudaStream_t st) {
  auto kern = adaln_rms_rope_kernel<VPL, ROW, MOD, FULL, EXACT>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int64_t grid = std::min<int64_t>(p.m, (int64_t)num_sms(dev));
  kern<<<(unsigned)grid, kNRThreads, smem, st>>>(tm, p);
  return cudaGetLastError();
}

template <int VPL, bool EXACT>
cudaError_t launch_vpl(const CUtensorMap& tm, const NRParams& p, bool row, bool mod, bool full, int smem,
                       cudaStream_t st) {
  if (row) {
    if (mod) return full ? launch_one<VPL, true, 1, true, EXACT>(tm, p, smem, st) : launch_one<VPL, true, 1, false, EXACT>(tm, p, smem, st);
    return full ? launch_one<VPL, true, 0, true, EXACT>(tm, p, smem, st) : launch_one<VPL, true, 0, false, EXACT>(tm, p, smem, st);
  }
  if (mod) return full ? launch_one<VPL, false, 1, true, EXACT>(tm, p, smem, st) : launch_one<VPL, false, 1, false, EXACT>(tm, p, smem, st);
  return full ? launch_one<VPL, false, 0, true, EXACT>(tm, p, smem, st) : launch_one<VPL, false, 0, false, EXACT>(tm, p, smem, st);
}

// ---------------------------------------------------------------------------
// Per-head QK-norm + partial split-half RoPE over strided [tokens, heads, 128]
// views, one tensor (single side) or two (Q and K), for any head count and
// for outputs laid out for attention (HND-backed NHD views).
//
// Reference: launch_rms_rope_kernel with has_k = false / true and
// split_half = true (backends/cuda/ops/rms_rope.cu:36-229, launcher :353-384),
// called by single_qknorm_rope.py:69-181 (in place) and :209-236 (into an
// HND-backed view); math as the eager rms_rope_split_half
// (backends/eager/rope.py:67-92): rstd = 1 / sqrt(mean(x^2) + eps) in fp32,
// h = bf16((x * rstd) * w), y0 = t00 h0 + t01 h1, y1 = t10 h0 + t11 h1 in fp32
// (two products and one add), bf16; dims >= rot_dim are normalised only. A
// bf16 or fp16 table is widened to fp32, as the reference's CUDA kernel does.
//
// Layout: one warp per token, two heads at a time (half-warp hsel takes head
// 2 i + hsel), lane (l mod 16) owns dims 8 (l mod 16) .. + 7 as one 16-byte
// vector; its RoPE partner is (l mod 16) +- rot_dim / 16, one shuffle away.
// The rotation coefficients of the lane's 8 pairs are read once per token
// (once per head when the table has a head stride). Heads of the second
// tensor follow those of the first in the same loop, so the paired form reads
// each table row once for Q and K.
// ---------------------------------------------------------------------------
constexpr int kQKWarpsPerBlock = 8;
// per-warp cp.async ring depth (stages - 1 warp iterations in flight): 32 KB of
// static shared memory per block either way
template <int LPH>
constexpr int qk_stages() { return LPH == 16 ? 8 : 4; }

struct QKParams {
  const __nv_bfloat16* x[2];
  __nv_bfloat16* y[2];
  int64_t xs_t[2], xs_h[2], ys_t[2], ys_h[2];  // element strides: token, head
  const __nv_bfloat16* w[2];
  const void* freqs;
  int64_t fs_t, fs_h;  // table element strides: token, head (0: shared by the heads)
  int64_t m;
  int heads;
  int half_v;  // rot_dim / 16: 16-byte vectors in each rotation half (0: no rotation)
  int nt;      // tensors: 1 or 2
  float eps;
};

// fp32 coefficients (A for the lane's own value, B for the partner's) of 8 pairs
// starting at pair0 of a table row; TAB: 0 fp32, 1 bf16, 2 fp16.
template <int TAB>
__device__ __forceinline__ void rope_coeffs(const void* row, int pair0, int role, uint64_t* A, uint64_t* B) {
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float c[2][4];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int pr = pair0 + 2 * e + u;
      if constexpr (TAB == 0) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(row) + pr);
        c[u][0] = v.x; c[u][1] = v.y; c[u][2] = v.z; c[u][3] = v.w;
      } else {
        const uint2 v = __ldg(reinterpret_cast<const uint2*>(row) + pr);
        if constexpr (TAB == 1) {
          c[u][0] = bf16_lo(v.x); c[u][1] = bf16_hi(v.x); c[u][2] = bf16_lo(v.y); c[u][3] = bf16_hi(v.y);
        } else {
          c[u][0] = __half2float(__ushort_as_half((unsigned short)(v.x & 0xFFFFu)));
          c[u][1] = __half2float(__ushort_as_half((unsigned short)(v.x >> 16)));
          c[u][2] = __half2float(__ushort_as_half((unsigned short)(v.y & 0xFFFFu)));
          c[u][3] = __half2float(__ushort_as_half((unsigned short)(v.y >> 16)));
        }
      }
    }
    // role 0 (x0): t00 * x0 + t01 * x1; role 1 (x1): t11 * x1 + t10 * x0
    A[e] = role == 0 ? f2_pack(c[0][0], c[1][0]) : f2_pack(c[0][3], c[1][3]);
    B[e] = role == 0 ? f2_pack(c[0][1], c[1][1]) : f2_pack(c[0][2], c[1][2]);
  }
}

// LPH lanes per head: 16 (one 16-byte vector per lane, two heads per warp
// iteration) or 8 (two vectors per lane, four heads per iteration; needs the
// rotation halves to be whole lanes, rot_dim % 32 == 0). Lane (l mod LPH)
// owns dims 8 VPL (l mod LPH) .. + 8 VPL - 1; its RoPE partner holds the dims
// rot_dim / 2 away, one shuffle across the head's lanes.
template <int TAB, int LPH>
__global__ void __launch_bounds__(32 * kQKWarpsPerBlock) qk_rms_rope_kernel(const QKParams p) {
  constexpr int VPL = 16 / LPH;   // vectors per lane per head
  constexpr int HPI = 32 / LPH;   // heads per warp iteration
  constexpr int S = qk_stages<LPH>();
  const int lane = threadIdx.x & 31;
  const int64_t tok = (int64_t)blockIdx.x * kQKWarpsPerBlock + (threadIdx.x >> 5);
  if (tok >= p.m) return;  // warp-uniform
  const int hv = lane % LPH;
  const int hsel = lane / LPH;
  const int half_l = p.half_v / VPL;  // lanes per rotation half
  const int role = hv < half_l ? 0 : (hv < 2 * half_l ? 1 : 2);  // first half, second half, pass-through
  const int partner = (lane - hv) + (role == 0 ? hv + half_l : (role == 1 ? hv - half_l : hv));
  const int pair0 = 8 * VPL * (role == 0 ? hv : (role == 1 ? hv - half_l : 0));
  constexpr int kTabElemBytes = TAB == 0 ? 4 : 2;
  const uint8_t* trow = static_cast<const uint8_t*>(p.freqs) + tok * p.fs_t * kTabElemBytes;

  uint64_t A[4 * VPL], B[4 * VPL];
#pragma unroll
  for (int e = 0; e < 4 * VPL; ++e) A[e] = B[e] = 0;
  if (role != 2 && p.fs_h == 0) {
#pragma unroll
    for (int v = 0; v < VPL; ++v) rope_coeffs<TAB>(trow, pair0 + 8 * v, role, A + 4 * v, B + 4 * v);
  }
  // the lane's weights of each tensor (bf16 pairs; widened where used)
  uint4 wv0[VPL], wv1[VPL];
#pragma unroll
  for (int v = 0; v < VPL; ++v) {
    wv0[v] = ldg_nc_v4(p.w[0] + 8 * (VPL * hv + v));
    wv1[v] = p.nt > 1 ? ldg_nc_v4(p.w[1] + 8 * (VPL * hv + v)) : wv0[v];
  }

  const int total = p.nt * p.heads;
  const int iters = (total + HPI - 1) / HPI;
  // this token's rows of each tensor (lane offset included); selects, not
  // runtime-indexed arrays, so everything stays in registers
  const __nv_bfloat16* const xrow0 = p.x[0] + tok * p.xs_t[0] + 8 * VPL * hv;
  const __nv_bfloat16* const xrow1 = p.x[1] + tok * p.xs_t[1] + 8 * VPL * hv;
  __nv_bfloat16* const yrow0 = p.y[0] + tok * p.ys_t[0] + 8 * VPL * hv;
  __nv_bfloat16* const yrow1 = p.y[1] + tok * p.ys_t[1] + 8 * VPL * hv;
  const int64_t xsh0 = p.xs_h[0], xsh1 = p.xs_h[1], ysh0 = p.ys_h[0], ysh1 = p.ys_h[1];
  // Each lane streams its own bytes of head HPI i + hsel into a per-warp
  // shared-memory ring with cp.async, S - 1 iterations ahead, and reads back
  // only what it copied itself (cp.async.wait_group orders it, no barrier).
  // The heads read ahead are never the ones being written, so in place is exact.
  __shared__ __align__(16) uint4 ring_s[kQKWarpsPerBlock][S][32 * VPL];
  uint4* const ring = &ring_s[threadIdx.x >> 5][0][lane * VPL];
  auto issue = [&](int it) {
    const int hh = HPI * it + hsel;
    if (it < iters && hh < total) {
      const __nv_bfloat16* src = hh >= p.heads ? xrow1 + (int64_t)(hh - p.heads) * xsh1 : xrow0 + (int64_t)hh * xsh0;
#pragma unroll
      for (int v = 0; v < VPL; ++v)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(ring + (it & (S - 1)) * 32 * VPL + v)),
                     "l"(src + 8 * v)
                     : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
#pragma unroll
  for (int i = 0; i < S - 1; ++i) issue(i);
  for (int it = 0; it < iters; ++it) {
    issue(it + S - 1);
    asm volatile("cp.async.wait_group %0;" ::"n"(S - 1) : "memory");
    const int hh = HPI * it + hsel;
    const bool ok = hh < total;
    uint4 xv[VPL];
#pragma unroll
    for (int v = 0; v < VPL; ++v) xv[v] = ok ? ring[(it & (S - 1)) * 32 * VPL + v] : make_uint4(0, 0, 0, 0);
    const int hc = ok ? hh : total - 1;
    const int t = hc >= p.heads ? 1 : 0;
    const int h = hc - t * p.heads;
    if (role != 2 && p.fs_h != 0) {
#pragma unroll
      for (int v = 0; v < VPL; ++v)
        rope_coeffs<TAB>(trow + h * p.fs_h * kTabElemBytes, pair0 + 8 * v, role, A + 4 * v, B + 4 * v);
    }
    // sum of squares over the head's 128 values (LPH lanes), double
    double acc[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
    for (int v = 0; v < VPL; ++v) sumsq8_fast(xv[v], acc);
    double sum = (acc[0] + acc[1]) + (acc[2] + acc[3]);
#pragma unroll
    for (int o = LPH / 2; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    float ms = (float)(sum * 0.0078125);   // / 128, exact
    const bool bad = !isfinite(ms);
    if (__any_sync(0xffffffffu, bad)) {  // inf / NaN / huge: exact conversions
      double ex[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
      for (int v = 0; v < VPL; ++v) sumsq8_exact(xv[v], ex);
      double se = (ex[0] + ex[1]) + (ex[2] + ex[3]);
#pragma unroll
      for (int o = LPH / 2; o > 0; o >>= 1) se += __shfl_xor_sync(0xffffffffu, se, o);
      if (bad) ms = (float)(se * 0.0078125);
    }
    const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, p.eps)));
    const uint64_t rs2 = f2_pack(rs, rs);
    __nv_bfloat16* const dst = (t ? yrow1 : yrow0) + (int64_t)h * (t ? ysh1 : ysh0);
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      const uint32_t xw[4] = {xv[v].x, xv[v].y, xv[v].z, xv[v].w};
      const uint4 wv = t ? wv1[v] : wv0[v];
      const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t hb[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) hb[e] = f2_to_bf16x2(f2_mul(f2_mul(bf16x2_to_f2(xw[e]), rs2), bf16x2_to_f2(ww[e])));
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t pw = __shfl_sync(0xffffffffu, hb[e], partner);
        float p0, p1, q0, q1;
        f2_unpack(f2_mul(A[4 * v + e], bf16x2_to_f2(hb[e])), p0, p1);
        f2_unpack(f2_mul(B[4 * v + e], bf16x2_to_f2(pw)), q0, q1);
        o[e] = role == 2 ? hb[e] : pack_bf16(__fadd_rn(p0, q0), __fadd_rn(p1, q1));
      }
      if (ok) stg_v4(dst + 8 * v, make_uint4(o[0], o[1], o[2], o[3]));
    }
  }
}

// y[t, h, :] = x[t, h, :] for [m, heads, 128] bf16 views (16-byte vectors; one
// thread per vector, 16 per head).
__global__ void __launch_bounds__(256) copy_heads_kernel(const __nv_bfloat16* __restrict__ x, int64_t xs_t,
                                                         int64_t xs_h, __nv_bfloat16* __restrict__ y, int64_t ys_t,
                                                         int64_t ys_h, int64_t m, int heads) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= m * heads * 16) return;
  const int v = (int)(i & 15);
  const int64_t th = i >> 4;
  const int64_t t = th / heads;
  const int h = (int)(th - t * heads);
  stg_v4(y + t * ys_t + h * ys_h + 8 * v, ldg_nc_v4(x + t * xs_t + h * xs_h + 8 * v));
}

// rope_t[p * m + t] = row p of token t's table as fp32 {t00, t01, t10, t11}
template <int TAB>
__global__ void __launch_bounds__(256) rope_table_transpose_kernel(const void* __restrict__ freqs, int64_t fs_t,
                                                                   int64_t m, int pairs, float4* __restrict__ rope_t) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // i = p * m + t: coalesced stores
  if (i >= m * pairs) return;
  const int p = (int)(i / m);
  const int64_t t = i - (int64_t)p * m;
  float4 v;
  if constexpr (TAB == 0) {
    v = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(freqs) + t * fs_t) + p);
  } else {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(freqs) + t * fs_t) + p);
    if constexpr (TAB == 1) {
      v = make_float4(bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y));
    } else {
      v = make_float4(__half2float(__ushort_as_half((unsigned short)(u.x & 0xFFFFu))),
                      __half2float(__ushort_as_half((unsigned short)(u.x >> 16))),
                      __half2float(__ushort_as_half((unsigned short)(u.y & 0xFFFFu))),
                      __half2float(__ushort_as_half((unsigned short)(u.y >> 16))));
    }
  }
  rope_t[i] = v;
}

}  // namespace

cudaError_t launch_rope_table_transpose(const void* freqs, int table_dtype, int64_t fs_t, int64_t m, int pairs,
                                        float4* rope_t, cudaStream_t stream) {
  if (m == 0 || pairs == 0) return cudaSuccess;
  const int tab_bytes = table_dtype == 0 ? 4 : 2;
  if (freqs == nullptr || table_dtype < 0 || table_dtype > 2 || pairs < 0 || fs_t < 0 ||
      (reinterpret_cast<uintptr_t>(freqs) % (4 * tab_bytes)) || (fs_t % 4) || (reinterpret_cast<uintptr_t>(rope_t) & 15))
    return cudaErrorNotSupported;
  const int64_t total = m * pairs;
  const unsigned grid = (unsigned)((total + 255) / 256);
  if (table_dtype == 0)
    rope_table_transpose_kernel<0><<<grid, 256, 0, stream>>>(freqs, fs_t, m, pairs, rope_t);
  else if (table_dtype == 1)
    rope_table_transpose_kernel<1><<<grid, 256, 0, stream>>>(freqs, fs_t, m, pairs, rope_t);
  else
    rope_table_transpose_kernel<2><<<grid, 256, 0, stream>>>(freqs, fs_t, m, pairs, rope_t);
  return cudaGetLastError();
}

cudaError_t launch_copy_heads(const void* x, int64_t xs_t, int64_t xs_h, void* y, int64_t ys_t, int64_t ys_h,
                              int64_t m, int64_t heads, cudaStream_t stream) {
  if (m == 0) return cudaSuccess;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y) & 15) || xs_t % 8 || xs_h % 8 ||
      ys_t % 8 || ys_h % 8 || heads <= 0 || heads > (1 << 20))
    return cudaErrorNotSupported;
  const int64_t total = m * heads * 16;
  copy_heads_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), xs_t, xs_h, static_cast<__nv_bfloat16*>(y), ys_t, ys_h, m, (int)heads);
  return cudaGetLastError();
}

cudaError_t launch_qk_rms_rope(const QKNormRopeArgs& a, cudaStream_t stream) {
  if (a.m == 0) return cudaSuccess;
  const int64_t rot = a.rot_dim == 0 ? 128 : a.rot_dim;
  if (a.head_dim != 128 || rot % 16 || rot <= 0 || rot > 128 || a.heads <= 0 || a.heads > (1 << 20) ||
      (a.tensors != 1 && a.tensors != 2) || a.table_dtype < 0 || a.table_dtype > 2)
    return cudaErrorNotSupported;
  auto al16 = [](const void* ptr) { return ptr != nullptr && !(reinterpret_cast<uintptr_t>(ptr) & 15); };
  QKParams p;
  for (int t = 0; t < 2; ++t) {
    const bool on = t < a.tensors;
    if (on && (!al16(a.x[t]) || !al16(a.y[t]) || !al16(a.w[t]) || a.xs_t[t] % 8 || a.xs_h[t] % 8 ||
               a.ys_t[t] % 8 || a.ys_h[t] % 8))
      return cudaErrorNotSupported;
    p.x[t] = static_cast<const __nv_bfloat16*>(on ? a.x[t] : a.x[0]);
    p.y[t] = static_cast<__nv_bfloat16*>(on ? a.y[t] : a.y[0]);
    p.w[t] = static_cast<const __nv_bfloat16*>(on ? a.w[t] : a.w[0]);
    p.xs_t[t] = on ? a.xs_t[t] : a.xs_t[0];
    p.xs_h[t] = on ? a.xs_h[t] : a.xs_h[0];
    p.ys_t[t] = on ? a.ys_t[t] : a.ys_t[0];
    p.ys_h[t] = on ? a.ys_h[t] : a.ys_h[0];
  }
  const int tab_bytes = a.table_dtype == 0 ? 4 : 2;
  // table rows: [rot/2, 2, 2] contiguous, each row start 16-byte (fp32) / 8-byte (16-bit) aligned;
  // no table: RMSNorm only (every lane passes its normalised values through)
  const bool rope = a.freqs != nullptr;
  if (rope && ((reinterpret_cast<uintptr_t>(a.freqs) % (2 * tab_bytes * 2)) || (a.fs_t * tab_bytes) % (4 * tab_bytes) ||
               (a.fs_h * tab_bytes) % (4 * tab_bytes) || a.fs_t < 0 || a.fs_h < 0))
    return cudaErrorNotSupported;
  p.freqs = a.freqs;
  p.fs_t = rope ? a.fs_t : 0;
  p.fs_h = rope ? a.fs_h : 0;
  p.m = a.m;
  p.heads = (int)a.heads;
  p.half_v = rope ? (int)(rot / 16) : 0;
  p.nt = a.tensors;
  p.eps = a.eps;
  const int64_t blocks = (a.m + kQKWarpsPerBlock - 1) / kQKWarpsPerBlock;
  if (blocks > 0x7FFFFFFF) return cudaErrorNotSupported;
  const dim3 grid((unsigned)blocks), block(32 * kQKWarpsPerBlock);
  // eight lanes per head when the rotation halves are whole lanes of 16 dims
  const bool lph8 = p.half_v % 2 == 0;
#define H3_QK(TAB)                                                               \
  (lph8 ? qk_rms_rope_kernel<TAB, 8><<<grid, block, 0, stream>>>(p)              \
        : qk_rms_rope_kernel<TAB, 16><<<grid, block, 0, stream>>>(p))
  if (a.table_dtype == 0)
    H3_QK(0);
  else if (a.table_dtype == 1)
    H3_QK(1);
  else
    H3_QK(2);
#undef H3_QK
  return cudaGetLastError();
}

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
  // a modulation row per token (row map or token groups): row span only, rows read through L1
  const bool mod_rows = mod && (a.row_map != nullptr || a.tokens_per_row > 0 || a.mod_rows > 1);
  if (mod_rows && (a.norm_span != 0 || a.mod_rows < 1 || a.lds % 8 || a.ldh % 8 ||
                   a.lds < a.heads * a.head_dim || a.ldh < a.heads * a.head_dim))
    return cudaErrorNotSupported;
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
  p.row_map = a.row_map;
  p.tokens_per_row = a.tokens_per_row;
  p.mod_rows = a.mod_rows < 1 ? 1 : a.mod_rows;
  p.lds = a.lds;
  p.ldh = a.ldh;
  p.m = a.m;
  p.heads = (int)a.heads;
  p.half_v = (int)(rot / 16);
  p.row_elems = (int)(a.heads * a.head_dim);
  p.row_bytes = (int)(a.heads * a.head_dim * 2);
  p.nseg = (int)(rot / 16);
  p.eps = a.eps;
  const bool row = a.norm_span == 0;
  const int nvec = (int)(a.heads * 16);
  p.tab_off = (2 * p.row_bytes + 1023) & ~1023;
  p.stage_bytes = (p.tab_off + p.nseg * 128 + 1023) & ~1023;
  p.ring_off = ring_offset(nvec, row, mod && !mod_rows);
  // deepest ring (a multiple of the pair count, so each stage always serves the same pair) that fits
  int stages = 0;
  for (int s = kMaxStages; s >= kPairs; s -= kPairs)
    if (1024 + p.ring_off + s * p.stage_bytes <= kSmemLimit) {
      stages = s;
      break;
    }
  if (stages == 0) return cudaErrorNotSupported;
  p.stages = stages;
  const int smem = 1024 + p.ring_off + stages * p.stage_bytes;
  // rotation table as rows of 128 bytes (8 pairs), one box = one token's nseg rows
  CUtensorMap tm;
  if (!encode_tmap_2d(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.freqs, 32, (uint64_t)a.m * (uint64_t)p.nseg, 128, 32,
                      (uint32_t)p.nseg, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  const bool full = rot == 128;
  const int vpl = (int)((a.heads * 16 + 31) / 32);
  if (mod_rows) {
    if (a.heads == 24)
      return full ? launch_one<12, true, 2, true, true>(tm, p, smem, stream) : launch_one<12, true, 2, false, true>(tm, p, smem, stream);
    return full ? launch_one<16, true, 2, true, false>(tm, p, smem, stream) : launch_one<16, true, 2, false, false>(tm, p, smem, stream);
  }
  if (a.heads == 24) return launch_vpl<12, true>(tm, p, row, mod, full, smem, stream);  // 3072-wide rows
  if (vpl <= 4) return launch_vpl<4, false>(tm, p, row, mod, full, smem, stream);
  if (vpl <= 8) return launch_vpl<8, false>(tm, p, row, mod, full, smem, stream);
  if (vpl <= 12) return launch_vpl<12, false>(tm, p, row, mod, full, smem, stream);
  return launch_vpl<16, false>(tm, p, row, mod, full, smem, stream);
}

}  // namespace h3
