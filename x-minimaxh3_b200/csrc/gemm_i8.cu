// Persistent, warp-specialised INT8 GEMM for sm_100a with fused epilogues.
//
//   D[m, n] = sum_k A[m, k] * W[n, k]      (int8 x int8 -> int32, exact)
//
// Replaces the reference's SM80 CUTLASS FusedInt8Gemm
// (backends/cuda/ops/cutlass_gemm_int8.cu:242-324) and cuBLASLt INT8 GEMM
// (backends/cuda/ops/cublas_gemm_int8.cu:204); epilogue arithmetic follows the
// eager path (backends/eager/quantization.py:1034-1053).
//
// Structure (one CTA per SM, 384 threads):
//   warp 0      TMA producer: A tile 128x128 B and W tile 256x128 B per stage,
//               128-byte swizzle, 4-stage ring guarded by full/empty mbarriers.
//   warp 1      MMA issuer: 4 x tcgen05.mma.cta_group::1.kind::i8 (128x256x32)
//               per stage into a TMEM accumulator; tcgen05.commit frees the
//               stage and, after the last k-block, publishes the accumulator.
//   warp 2      TMEM allocator (512 columns = two 128x256 s32 accumulators).
//   warps 4-11  epilogue: tcgen05.ld 32 columns at a time, fused dequant /
//               activation / gated residual; each warp stages its 32x32 bf16
//               result in shared memory (64-byte swizzle, conflict-free) and one
//               lane writes it with a TMA tensor store (int32 results use
//               128-bit global stores). The gated-residual epilogues TMA-load
//               the residual's 32x32 box into the same staging box first. The
//               two accumulators let the epilogue of tile i overlap the
//               mainloop of tile i+1.
// W4A8 epilogues (kEpi*Corr) add the asymmetric correction sx . corr_t^T, a
// rank-kp bf16 product (kp <= 128), on the tensor cores inside the same TMEM
// accumulator: a first epilogue pass replaces each int32 accumulator by its
// dequantized bf16 value as fp32 (tcgen05.st); one epilogue thread then issues
// kind::f16 MMAs that accumulate sx[rows, :kp] . corr_t[cols, :kp]^T onto it,
// their operands TMA-loaded into shared memory reserved for them (the stage
// ring shrinks to make room); a second pass reads the corrected sums.
// Tiles are visited N-fastest when the weight fits in L2 (it stays resident and
// the running CTAs share A rows), else in groups of 8 M-blocks with M fastest
// inside a group (the weight streams past L2 once per group; see tile_coords).
// No cluster multicast is used anywhere (the same binary runs in multi-GPU jobs).
#include "common.cuh"
#include "kernels.h"
#include "quant_math.cuh"

namespace h3 {

__device__ unsigned int g_status = 0u;
__device__ unsigned int* g_status_host = nullptr;

namespace {

constexpr int BM = 128, BN = 256, BK = 128, STAGES = 4;
constexpr int A_BYTES = BM * BK;
constexpr int B_BYTES = BN * BK;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int NUM_THREADS = 384;
constexpr int EPI_WARP0 = 4;
constexpr int NUM_EPI_WARPS = 8;
constexpr uint32_t TMEM_COLS = 2 * BN;
constexpr uint32_t IDESC_I8 = umma_idesc_i8(BM, BN);
constexpr uint32_t IDESC_I8_PAIR = umma_idesc_i8(2 * BM, BN);  // cta_group::2: 256 x 256 per CTA pair
constexpr uint32_t IDESC_BF16 = umma_idesc_bf16(BM, BN);
constexpr uint32_t IDESC_BF16_PAIR = umma_idesc_bf16(2 * BM, BN);
constexpr int kMaxCorrKp = 128;  // correction groups (padded) held in shared memory
constexpr int BAR_BYTES = 256;
constexpr int STAGE_OPS_BYTES = NUM_EPI_WARPS * 2 * 128 * 4;   // per-warp column scales + bias/gate
constexpr int GELU_TAB_BYTES = 2 * 19 * 128 * 2;
constexpr int EPI_STAGE_BYTES = 32 * 32 * 2;                    // one 32x32 bf16 box per epilogue warp
constexpr int OFF_BAR = STAGES * STAGE_BYTES;
constexpr int OFF_OPS = OFF_BAR + BAR_BYTES;
constexpr int OFF_GELU = OFF_OPS + STAGE_OPS_BYTES;
constexpr int OFF_EPI = (OFF_GELU + GELU_TAB_BYTES + 1023) / 1024 * 1024;  // swizzled boxes: 1024-aligned
constexpr int SMEM_BYTES = OFF_EPI + NUM_EPI_WARPS * EPI_STAGE_BYTES + 1024;
static_assert(SMEM_BYTES <= 232448, "GEMM shared memory exceeds the 227 KB per-block limit");

// status codes recorded when a bounded wait expires
constexpr unsigned kErrProducer = 0x101, kErrMmaAcc = 0x102, kErrMmaFull = 0x103, kErrEpi = 0x104,
                   kErrDrain = 0x105, kErrEpiIn = 0x106, kErrCorr = 0x107;

struct KParams {
  int m, n, k;
  int num_n_blk, num_k_blk, num_tiles;
  int num_m_blk, group_m;  // tile order: groups of group_m M-blocks (see tile_coords)
  const float* a_scale;
  const float* w_scale;
  int w_pc;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* gate;
  const __nv_bfloat16* residual;
  int64_t ldr;
  void* out;
  int64_t ldo;
  float* row_absmax;
  int corr_kb;  // 64-group k-blocks of the correction operands (kEpi*Corr)
  const int32_t* row_map;  // kEpiGatedResidual: gate row of each output row (nullptr: gate is one row)
  int64_t ldg;             // row stride of the gate rows (elements)
  // kEpiQKV (see GemmArgs): output maps tmO / tmR / tmS are sections Q / K / V;
  // bit s of qkv_hmaj: section s's map is (dim, head, token) instead of (dim, token, head)
  int qkv_inner, qkv_sec0, qkv_rot, qkv_hmaj;
  const __nv_bfloat16* qk_w[2];
  const float4* rope_t;
  float qk_eps;
  int up_row;  // kEpiSwiGLU: first up row of W (the output width f)
  // in-kernel requantization of A (kEpiGatedResidual, GemmArgs::requant_src)
  const __nv_bfloat16* rq_src;
  int64_t rq_lds;
  int8_t* rq_dst;
  unsigned int* rq_ready;     // one count of finished units per block of tile rows (zero at launch)
  unsigned int* rq_horizon;   // highest block the tiles have asked for (zero at launch)
  int64_t rq_units;           // m * rq_upr
  int rq_upr;                 // units of kRqUnit elements per row
  // kEpiI32 rows routed to their owners (GemmArgs::peer_out / peer_world)
  int32_t* peer_out[kTpMaxWorld];
  int peer_world;
  int out_f16;  // kEpiBF16: fp16 out and bias (GemmArgs::out_f16)
};

template <int EPI>
constexpr bool is_corr_epi() {
  return EPI == kEpiBF16Corr || EPI == kEpiBF16CorrGelu || EPI == kEpiGatedResidualCorr;
}

// Exact bf16 tanh-GELU by table. The activation input is a bf16 value, so the
// GELU is a function on at most 65,536 inputs. Every CTA of the GELU variant
// fills a shared-memory table with gelu_tanh_exact (bit-identical to the
// reference, verified on all bf16 inputs) for |x| in [2^-16, 8) and both signs
// (2 x 19 binades x 128 mantissas). The lookup itself is branch-free (the
// index is clamped into the table); a lane whose chunk holds an input outside
// that range (zero, |x| < 2^-16 or >= 8, non-finite) recomputes the chunk
// through gelu_lookup, whose closed forms leave only subnormal and non-finite
// inputs to gelu_tanh_exact.
constexpr uint32_t kGeluE0 = 111;   // exponent field of 2^-16
constexpr uint32_t kGeluNE = 19;    // binades 2^-16 .. 2^2
constexpr int kGeluEntries = 2 * kGeluNE * 128;

__device__ __forceinline__ uint32_t gelu_table_bits(uint32_t i) {
  const uint32_t sgn = i / (kGeluNE * 128);
  const uint32_t rem = i - sgn * (kGeluNE * 128);
  return (sgn << 15) | ((kGeluE0 + rem / 128) << 7) | (rem & 127u);
}

constexpr uint32_t kGeluHalf = kGeluNE * 128;  // entries per sign
constexpr uint32_t kGeluBase = kGeluE0 << 7;   // |x| bits of 2^-16

// Table lookup. Inside the table the entry of |x| is its bits minus those of 2^-16
// (binade and mantissa are consecutive in the encoding); `span` collects that
// unclamped offset, so span >= kGeluHalf afterwards flags an input outside it.
__device__ __forceinline__ uint32_t gelu_lookup_fast(uint32_t hb, const uint16_t* tab, uint32_t& span) {
  const uint32_t u = (hb & 0x7FFFu) - kGeluBase;  // wraps below 2^-16
  span = max(span, u);
  return tab[((hb >> 15) & 1u) * kGeluHalf + min(u, kGeluHalf - 1u)];
}

// The exact value of any bf16 input. Outside the table the reference's result has
// a closed form (checked against its all-inputs fixture): +-0 -> +-0; 2^-125 <= |x|
// < 2^-16 -> 0.5 x exactly (the tanh term is below half an ulp); |x| >= 8 -> x or -0
// (its tanh is exactly +-1). Only subnormal and non-finite inputs are evaluated.
__device__ __forceinline__ uint32_t gelu_lookup(uint32_t hb, const uint16_t* tab) {
  hb &= 0xFFFFu;
  const uint32_t u = (hb & 0x7FFFu) - kGeluBase;
  if (u < kGeluHalf) return tab[(hb >> 15) * kGeluHalf + u];
  const uint32_t e = (hb >> 7) & 0xFFu;
  if ((hb & 0x7FFFu) == 0u) return hb;
  if (e >= 2u && e < kGeluE0) return hb - 0x80u;
  if (e >= kGeluE0 + kGeluNE && e < 255u) return (hb & 0x8000u) ? 0x8000u : hb;
  return bf16_bits(gelu_tanh_exact(__uint_as_float(hb << 16)));
}

// GELU of 16 packed bf16 pairs, in place.
__device__ __forceinline__ void gelu_pairs(uint32_t (&ob)[16], const uint16_t* gtab) {
  uint32_t span = 0u;
  uint32_t g[16];
#pragma unroll
  for (int j = 0; j < 16; ++j)
    g[j] = gelu_lookup_fast(ob[j] & 0xFFFFu, gtab, span) | (gelu_lookup_fast(ob[j] >> 16, gtab, span) << 16);
  if (span >= kGeluHalf) {
#pragma unroll
    for (int j = 0; j < 16; ++j) g[j] = gelu_lookup(ob[j] & 0xFFFFu, gtab) | (gelu_lookup(ob[j] >> 16, gtab) << 16);
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) ob[j] = g[j];
}

// Dequantized bf16 bits of the 32 accumulators of one chunk (GELU variant input).
__device__ __forceinline__ uint32_t dequant_bits(uint32_t acc, float xs, float ws) {
  return bf16_bits(__fmul_rn(__int2float_rn((int)acc), __fmul_rn(xs, ws)));
}

// First pass of the W4A8 epilogues: each int32 accumulator of the chunk becomes
// its dequantized bf16 value bf16(acc * (xs * ws)), held as fp32 bits.
__device__ __forceinline__ void dequant_to_f32(uint32_t (&r)[32], float xs, const float* ws_s) {
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 w4 = *reinterpret_cast<const float4*>(ws_s + 4 * q);
    r[4 * q + 0] = dequant_bits(r[4 * q + 0], xs, w4.x) << 16;
    r[4 * q + 1] = dequant_bits(r[4 * q + 1], xs, w4.y) << 16;
    r[4 * q + 2] = dequant_bits(r[4 * q + 2], xs, w4.z) << 16;
    r[4 * q + 3] = dequant_bits(r[4 * q + 3], xs, w4.w) << 16;
  }
}

// The same with the bias of a W4A8 linear: bf16(bf16(acc * (xs * ws)) + bias), as fp32
// bits (the correction is then added to this value, one rounding at the end).
__device__ __forceinline__ void dequant_bias_to_f32(uint32_t (&r)[32], float xs, const float* ws_s,
                                                    const float* bias_s) {
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float d = __uint_as_float(dequant_bits(r[j], xs, ws_s[j]) << 16);
    r[j] = (uint32_t)bf16_bits(__fadd_rn(d, bias_s[j])) << 16;
  }
}

// Two dequantized values bf16(acc * (xs * ws)) as a packed bf16 pair (f32x2 products,
// the same roundings as dequant_bits).
__device__ __forceinline__ uint32_t dequant_pair(uint32_t a0, uint32_t a1, float xs, float w0, float w1) {
  uint64_t w, a;
  asm("mov.b64 %0, {%1, %2};" : "=l"(w) : "f"(w0), "f"(w1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(__int2float_rn((int)a0)), "f"(__int2float_rn((int)a1)));
  uint32_t lo, hi;
  f2_bits(f2_mul(a, f2_mul(f2_dup(xs), w)), lo, hi);
  return bf16x2_from_bits(lo, hi);
}

__device__ __forceinline__ uint32_t max_u16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.u16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// fc1 chunk: out bits (packed pairs) = gelu(bf16(acc * (xs * ws))); chunk absmax bits.
__device__ __forceinline__ void gelu_chunk(const uint32_t (&r)[32], float xs, const float* ws_s, const uint16_t* gtab,
                                           uint32_t (&ob)[16], uint32_t& amax_bits) {
  uint32_t span = 0u, cmax = 0u;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 w4 = *reinterpret_cast<const float4*>(ws_s + 4 * q);
    const uint32_t h01 = dequant_pair(r[4 * q + 0], r[4 * q + 1], xs, w4.x, w4.y);
    const uint32_t h23 = dequant_pair(r[4 * q + 2], r[4 * q + 3], xs, w4.z, w4.w);
    ob[2 * q] = gelu_lookup_fast(h01, gtab, span) | (gelu_lookup_fast(h01 >> 16, gtab, span) << 16);
    ob[2 * q + 1] = gelu_lookup_fast(h23, gtab, span) | (gelu_lookup_fast(h23 >> 16, gtab, span) << 16);
    cmax = max_u16x2(cmax, max_u16x2(ob[2 * q] & 0x7FFF7FFFu, ob[2 * q + 1] & 0x7FFF7FFFu));
  }
  if (span >= kGeluHalf) {  // an input outside the table: the exact path for the chunk
    cmax = 0u;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 w4 = *reinterpret_cast<const float4*>(ws_s + 4 * q);
      const uint32_t h01 = dequant_pair(r[4 * q + 0], r[4 * q + 1], xs, w4.x, w4.y);
      const uint32_t h23 = dequant_pair(r[4 * q + 2], r[4 * q + 3], xs, w4.z, w4.w);
      ob[2 * q] = gelu_lookup(h01, gtab) | (gelu_lookup(h01 >> 16, gtab) << 16);
      ob[2 * q + 1] = gelu_lookup(h23, gtab) | (gelu_lookup(h23 >> 16, gtab) << 16);
      cmax = max_u16x2(cmax, max_u16x2(ob[2 * q] & 0x7FFF7FFFu, ob[2 * q + 1] & 0x7FFF7FFFu));
    }
  }
  amax_bits = max(amax_bits, max(cmax & 0xFFFFu, cmax >> 16));
}

// int32 accumulators of one 32-column chunk of one row, 128-bit stores.
__device__ __forceinline__ void store_i32_chunk(const KParams& p, int row, int col0, const uint32_t (&r)[32]) {
  if (row < p.m) {
    int32_t* o = static_cast<int32_t*>(p.out) + (int64_t)row * p.ldo + col0;
#pragma unroll
    for (int g = 0; g < 8; ++g)
      if (col0 + 4 * g < p.n) stg_v4(o + 4 * g, make_uint4(r[4 * g], r[4 * g + 1], r[4 * g + 2], r[4 * g + 3]));
  }
}

// Routed int32 rows (p.peer_world > 0), usually another GPU's memory: lane t holds row
// row_base + t's 32 columns [col0, col0 + 32). The warp passes them through its 2 KB
// staging box (32 rows x 64 bytes, 16-byte chunks swizzled by (row >> 1) & 3), one
// 16-column half at a time, so that each store instruction writes 8 rows x 64
// contiguous bytes instead of 32 rows x 16 bytes: fewer, larger writes over NVLink.
__device__ __forceinline__ void store_i32_chunk_routed(const KParams& p, int row_base, int col0,
                                                       const uint32_t (&r)[32], uint8_t* box, int lane) {
  uint8_t* my_row = box + lane * 64;
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    __syncwarp();  // the previous half's reads of the box are done
#pragma unroll
    for (int q = 0; q < 4; ++q)
      *reinterpret_cast<uint4*>(my_row + ((q ^ sw) << 4)) =
          make_uint4(r[16 * h + 4 * q], r[16 * h + 4 * q + 1], r[16 * h + 4 * q + 2], r[16 * h + 4 * q + 3]);
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int rr = 8 * i + (lane >> 2), q = lane & 3;
      const uint4 v = *reinterpret_cast<const uint4*>(box + rr * 64 + ((q ^ ((rr >> 1) & 3)) << 4));
      const int row = row_base + rr, col = col0 + 16 * h + 4 * q;
      if (row < p.m && col < p.n)
        stg_v4(p.peer_out[tp_owner(row, p.peer_world)] + tp_local_row(row, p.peer_world) * p.ldo + col, v);
    }
  }
}

// bf16 results (packed pairs) of one 32-column chunk of one accumulator row.
// ws_s / aux_s: this warp's staged per-column weight scales and bias-or-gate
// (fp32) for the chunk; in_w: the row's 32 bf16 residual values for the
// gated-residual epilogues. For the W4A8 epilogues r holds the fp32 sums
// dequant + correction of the second pass.
// For kEpiGatedResidual, bias_s holds the staged bias (when p.bias is set) and
// gw the row's own 32 gate values (when p.row_map is set; else aux_s has the
// single gate row).
template <int EPI>
__device__ __forceinline__ void epilogue_values(const KParams& p, const uint32_t (&r)[32], float xs,
                                                const float* ws_s, const float* aux_s, const uint16_t* gtab,
                                                uint32_t& amax_bits, const uint32_t (&in_w)[16],
                                                const float* bias_s, const uint32_t (&gw)[16],
                                                uint32_t (&ob)[16]) {
  if constexpr (EPI == kEpiGeluAbsmax) {
    gelu_chunk(r, xs, ws_s, gtab, ob, amax_bits);
  } else if constexpr (is_corr_epi<EPI>()) {
#pragma unroll
    for (int j = 0; j < 16; ++j) ob[j] = pack_bf16(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
    if constexpr (EPI == kEpiBF16CorrGelu) gelu_pairs(ob, gtab);
    if constexpr (EPI == kEpiGatedResidualCorr) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 a4 = *reinterpret_cast<const float4*>(aux_s + 4 * q);
        const uint32_t y0 = ob[2 * q], y1 = ob[2 * q + 1], r0 = in_w[2 * q], r1 = in_w[2 * q + 1];
        ob[2 * q] = pack_bf16(__fadd_rn(bf16_lo(r0), __fmul_rn(bf16_lo(y0), a4.x)),
                              __fadd_rn(bf16_hi(r0), __fmul_rn(bf16_hi(y0), a4.y)));
        ob[2 * q + 1] = pack_bf16(__fadd_rn(bf16_lo(r1), __fmul_rn(bf16_lo(y1), a4.z)),
                                  __fadd_rn(bf16_hi(r1), __fmul_rn(bf16_hi(y1), a4.w)));
      }
    }
  } else {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 w4 = *reinterpret_cast<const float4*>(ws_s + 4 * q);
      const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
      const float4 a4 = *reinterpret_cast<const float4*>(aux_s + 4 * q);
      const float av[4] = {a4.x, a4.y, a4.z, a4.w};
      uint32_t hb[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = 4 * q + e;
        uint32_t b;
        if (EPI == kEpiBF16 && p.out_f16) {  // fp16 out: the same association, fp16 roundings
          b = __half_as_ushort(__float2half_rn(__fmul_rn(__int2float_rn((int)r[j]), __fmul_rn(xs, wv[e]))));
          if (p.bias != nullptr)
            b = __half_as_ushort(__float2half_rn(__fadd_rn(__half2float(__ushort_as_half((unsigned short)b)), av[e])));
        } else {
          b = dequant_bits(r[j], xs, wv[e]);
          if constexpr (EPI == kEpiBF16) {
            if (p.bias != nullptr) b = bf16_bits(__fadd_rn(__uint_as_float(b << 16), av[e]));
          }
        }
        if constexpr (EPI == kEpiGatedResidual) {
          if (p.bias != nullptr) b = bf16_bits(__fadd_rn(__uint_as_float(b << 16), bias_s[j]));
          const uint32_t rw = in_w[j >> 1];
          const float rv = (j & 1) ? bf16_hi(rw) : bf16_lo(rw);
          float gv = av[e];
          if (p.row_map != nullptr) gv = (j & 1) ? bf16_hi(gw[j >> 1]) : bf16_lo(gw[j >> 1]);
          b = bf16_bits(__fadd_rn(rv, __fmul_rn(__uint_as_float(b << 16), gv)));
        }
        hb[e] = b;
      }
      ob[2 * q] = hb[0] | (hb[1] << 16);
      ob[2 * q + 1] = hb[2] | (hb[3] << 16);
    }
  }
}

// Tile order of the persistent walkers: groups of group_m M-blocks; inside a group
// the M-block changes fastest, then the N-block. With group_m = 1 (weights up to
// 64 MB) this is N-fastest: the running CTAs share one A row block and the whole
// weight stays resident in L2. For a larger weight (the H3 projections, 77-154 MB)
// group_m = 8: the running CTAs cover about 8 M-blocks x (CTAs / 8) N-blocks, the
// group's activation rows stay in L2 and the weight streams past once per group,
// num_m_blk / 8 times instead of once per M-block.
__device__ __forceinline__ void tile_coords(int tile, const KParams& p, int& m_blk, int& n_blk) {
  const int per_group = p.group_m * p.num_n_blk;
  const int g = tile / per_group;
  const int rem = tile - g * per_group;
  const int gm = min(p.group_m, p.num_m_blk - g * p.group_m);  // the last group may be shorter
  n_blk = rem / gm;
  m_blk = g * p.group_m + (rem - n_blk * gm);
}

// ---- in-kernel requantization of A (fc2 of the fused MLP, kEpiGatedResidualRq) ----
// The A operand of fc2 is quantize_int8_rowwise(gelu(fc1)) with the row absmax that
// fc1's epilogue already reduced. Instead of a separate pass, the CTAs' non-MMA warps
// produce it while the tensor cores run: warps 2-3 (idle otherwise) and the eight
// epilogue warps whenever their next accumulator is not ready yet (fc2's epilogue is
// short next to its mainloop). A unit is kRqUnit consecutive elements of one row;
// unit u belongs to quantizing warp u mod (kRqSlots * CTAs), so each warp walks the rows
// in order. A unit's 16-byte vectors and its row absmax are loaded at once, quantized
// like quantize_int8_rowwise and stored, and the unit is counted for its block of tile
// rows; the TMA producer loads a tile's A rows only once that block's count is
// complete. A warp takes its next unit only while that unit's block is at most `lead`
// blocks past the highest block the tiles have asked for, so quantized rows wait in L2
// briefly. No quantizing warp holds a unit while waiting on anything, units of blocks
// the tiles already asked for are never held back, and an epilogue warp whose tile
// waits for A has its accumulator not ready, so it quantizes: the dependency cannot
// deadlock (the persistent grid is resident).
constexpr int kRqUnit = 4096;      // elements per unit: 16 vectors of 8 per lane
constexpr int kRqSlots = 2 + NUM_EPI_WARPS;
constexpr unsigned kErrRequant = 0x108;

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned int* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_relaxed_gpu(const unsigned int* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// non-blocking test of a barrier phase
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Blocks the quantizing warps may run ahead of the tiles: the blocks of the first wave of
// tiles (ncl walkers) plus two.
__device__ __forceinline__ int requant_lead(const KParams& p, int ncl) {
  int mb_first = 0;
  for (int t = 0; t < ncl && t < p.num_tiles; ++t) {
    int mb, nb;
    tile_coords(t, p, mb, nb);
    mb_first = max(mb_first, mb);
  }
  return mb_first + 2;
}

// One quantizing warp's walk over its units.
struct RqCursor {
  int64_t u;       // next unit of this warp
  int64_t stride;  // kRqSlots * CTAs
  int lead;
  unsigned hz;     // lane 0's last view of the tiles' horizon
};

// Quantize and count unit c.u if its block is inside the window (lane 0 refreshes its
// view of the horizon only when the cached one says no). Returns false when the warp
// has no unit left or the window is closed.
template <int TILE_ROWS>
__device__ __forceinline__ bool requant_step(const KParams& p, RqCursor& c, int lane) {
  if (c.u >= p.rq_units) return false;
  const int row = (int)(c.u / p.rq_upr);
  uint32_t go = 1u;
  if (lane == 0 && row / TILE_ROWS > (int)c.hz + c.lead) {
    c.hz = ld_relaxed_gpu(p.rq_horizon);
    go = row / TILE_ROWS <= (int)c.hz + c.lead ? 1u : 0u;
  }
  if (__shfl_sync(0xffffffffu, go, 0) == 0u) return false;
  const int c0 = (int)(c.u - (int64_t)row * p.rq_upr) * kRqUnit;
  const int lim = p.k - c0;  // elements of the row from c0 on
  const __nv_bfloat16* src = p.rq_src + (int64_t)row * p.rq_lds + c0;
  int8_t* dst = p.rq_dst + (int64_t)row * p.k + c0;
  const float am = __ldg(p.row_absmax + row);
  uint4 v[kRqUnit / 256];
#pragma unroll
  for (int j = 0; j < kRqUnit / 256; ++j) {
    const int e = 8 * (lane + 32 * j);
    v[j] = e < lim ? ldg_nc_v4(src + e) : make_uint4(0u, 0u, 0u, 0u);
  }
  const float r = __frcp_rn(quant_divisor(row_scale(am)));
#pragma unroll
  for (int j = 0; j < kRqUnit / 256; ++j) {
    const int e = 8 * (lane + 32 * j);
    if (e < lim) *reinterpret_cast<uint2*>(dst + e) = quant_vec8(v[j], r);
  }
  // these generic-proxy stores are read by TMA (async proxy) after the count: fence
  // them towards the async proxy, then release the count at GPU scope
  fence_proxy_async_global();
  __syncwarp();
  if (lane == 0) {
    __threadfence();
    atomicAdd(p.rq_ready + row / TILE_ROWS, 1u);
  }
  c.u += c.stride;
  return true;
}

// Every remaining unit of the warp, waiting (bounded) whenever the window is closed.
template <int TILE_ROWS>
__device__ __forceinline__ void requant_finish(const KParams& p, RqCursor& c, int lane) {
  unsigned long long t0 = 0ull;
  while (c.u < p.rq_units) {
    if (requant_step<TILE_ROWS>(p, c, lane)) {
      t0 = 0ull;
      continue;
    }
    if (t0 == 0ull) t0 = global_ns();
    __nanosleep(256);
    if (status_bad()) return;
    if (global_ns() - t0 > kWaitTimeoutNs) {
      set_status(kErrRequant);
      return;
    }
  }
}

// Producer side: wait (bounded) until block b's A rows are all written.
__device__ __forceinline__ bool requant_wait(const KParams& p, int b, int tile_rows) {
  const unsigned need = (unsigned)(min(tile_rows, p.m - b * tile_rows) * p.rq_upr);
  const unsigned int* c = p.rq_ready + b;
  if (ld_acquire_gpu(c) < need) {
    const unsigned long long t0 = global_ns();
    while (ld_acquire_gpu(c) < need) {
      __nanosleep(256);
      if (status_bad()) return false;
      if (global_ns() - t0 > kWaitTimeoutNs) {
        set_status(kErrRequant);
        return false;
      }
    }
  }
  fence_proxy_async_global();
  return true;
}

// ---- kEpiQKV helpers: one thread holds one head (128 values) of one token ----
// |bf16| of the low / high half of w as a double, built from its bits (exact for
// normal values; zero and subnormals become a value below 2^-126 whose square
// cannot change the fp32 mean; non-finite rows are re-summed exactly)
__device__ __forceinline__ double qkv_abs_lo(uint32_t w) {
  return __hiloint2double((int)(((w & 0x7FFFu) << 13) + 0x38000000u), 0);
}
__device__ __forceinline__ double qkv_abs_hi(uint32_t w) {
  return __hiloint2double((int)(((w >> 3) & 0x0FFFE000u) + 0x38000000u), 0);
}

__device__ __forceinline__ uint64_t qkv_f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

// split-half RoPE over dims [0, 2R) of the head held as bf16 pairs h[j] = (2j, 2j + 1):
// y_i = t00 h_i + t01 h_{i+R}, y_{i+R} = t10 h_i + t11 h_{i+R} (fp32, two rounded
// products and one add, then bf16). rt: rows of pair p at rt[p * m], this token's
// column `row` (coalesced across the warp's 32 consecutive tokens).
template <int R>
__device__ __forceinline__ void qkv_rope(uint32_t (&h)[64], const float4* __restrict__ rt, int64_t m, int row) {
  const bool live = row < m;
#pragma unroll
  for (int i = 0; i < R; i += 2) {
    const float4 ta = live ? __ldg(rt + (int64_t)i * m + row) : make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 tb = live ? __ldg(rt + (int64_t)(i + 1) * m + row) : make_float4(0.f, 0.f, 0.f, 0.f);
    const uint32_t x0w = h[i / 2], x1w = h[(i + R) / 2];
    const float a0 = bf16_lo(x0w), a1 = bf16_hi(x0w), b0 = bf16_lo(x1w), b1 = bf16_hi(x1w);
    h[i / 2] = pack_bf16(__fadd_rn(__fmul_rn(ta.x, a0), __fmul_rn(ta.y, b0)),
                         __fadd_rn(__fmul_rn(tb.x, a1), __fmul_rn(tb.y, b1)));
    h[(i + R) / 2] = pack_bf16(__fadd_rn(__fmul_rn(ta.z, a0), __fmul_rn(ta.w, b0)),
                               __fadd_rn(__fmul_rn(tb.z, a1), __fmul_rn(tb.w, b1)));
  }
}

// CG = 1: one CTA per tile of 128 x 256. CG = 2: a cluster of two CTAs on an SM
// pair computes a 256 x 256 tile with tcgen05.mma.cta_group::2 issued by the
// rank-0 CTA: rank r loads A rows [128 r, 128 r + 128) and W rows
// [128 r, 128 r + 128) of the tile into its own shared memory (32 KB per
// k-block instead of 48, 6 stages), both CTAs' loads complete on rank 0's
// full barrier, each commit of rank 0 arrives on the barriers of both CTAs, and
// rank r's TMEM receives output rows [128 r, 128 r + 128) of the tile. Both
// epilogues release an accumulator on rank 0's barrier.
template <int EPI_ID, int CG>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmR,
                   const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmC,
                   const KParams p) {
  // kEpiGatedResidualRq / kEpiI32Rq: the gated-residual / int32 epilogue on an A operand
  // this kernel quantizes
  constexpr bool kRq = EPI_ID == kEpiGatedResidualRq || EPI_ID == kEpiI32Rq;
  constexpr int EPI = EPI_ID == kEpiGatedResidualRq ? kEpiGatedResidual : EPI_ID == kEpiI32Rq ? kEpiI32 : EPI_ID;
  constexpr bool kCorr = is_corr_epi<EPI>();
  constexpr bool kInBox = EPI == kEpiGatedResidual || EPI == kEpiGatedResidualCorr;
  constexpr int kBBytes = B_BYTES / CG;
  constexpr int kStageBytes = A_BYTES + kBBytes;
  // W4A8 correction operands for one tile: sx rows [BM x kMaxCorrKp] and
  // corr_t rows [BN / CG x kMaxCorrKp], bf16, as 64-group k-blocks
  constexpr int kCorrSxBytes = kCorr ? BM * kMaxCorrKp * 2 : 0;
  constexpr int kCorrCtBytes = kCorr ? (BN / CG) * kMaxCorrKp * 2 : 0;
  constexpr int kStagesMax = CG == 2 ? 6 : STAGES;
  constexpr int kStagesFit = (OFF_BAR - kCorrSxBytes - kCorrCtBytes) / kStageBytes;
  constexpr int kStages = kStagesMax < kStagesFit ? kStagesMax : kStagesFit;
  constexpr int kOffCorr = kStages * kStageBytes;
  static_assert(kStages >= 2 && kOffCorr + kCorrSxBytes + kCorrCtBytes <= OFF_BAR, "stage ring overflows its region");
  constexpr int kTileRows = BM * CG;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t rank = CG == 2 ? cluster_ctarank() : 0u;
  const int cid = (int)blockIdx.x / CG;      // tile walker (cluster) index
  const int ncl = (int)gridDim.x / CG;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* empty_bar = full_bar + kStages;
  uint64_t* tfull_bar = empty_bar + kStages;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint64_t* in_bar = drain_bar + 1;                   // [NUM_EPI_WARPS]: input-box loads of the epilogue warps
  uint64_t* corr_full_bar = in_bar + NUM_EPI_WARPS;   // correction operands landed (rank 0 counts both CTAs)
  uint64_t* dq_bar = corr_full_bar + 1;               // first epilogue pass written back (rank 0, all warps)
  uint64_t* cf_bar = dq_bar + 1;                      // correction MMAs complete (each CTA)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(cf_bar + 1);
  float* ops_smem = reinterpret_cast<float*>(smem + OFF_OPS);
  uint16_t* gelu_tab = reinterpret_cast<uint16_t*>(smem + OFF_GELU);
  uint8_t* corr_sx = smem + kOffCorr;
  uint8_t* corr_ct = corr_sx + kCorrSxBytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], NUM_EPI_WARPS * CG);  // CG = 2: both CTAs' epilogue warps
    }
    mbar_init(drain_bar, 1);
    for (int w = 0; w < NUM_EPI_WARPS; ++w) mbar_init(&in_bar[w], 1);
    mbar_init(corr_full_bar, 1);
    mbar_init(dq_bar, NUM_EPI_WARPS * CG);
    mbar_init(cf_bar, 1);
    fence_barrier_init();
    fence_proxy_async_shared();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (EPI != kEpiI32) tma_prefetch_desc(&tmO);
    if (kInBox) tma_prefetch_desc(&tmR);
    if (kCorr) {
      tma_prefetch_desc(&tmS);
      tma_prefetch_desc(&tmC);
    }
  }
  if (warp == 2) {
    if constexpr (CG == 2) {
      tmem_alloc_pair(tmem_slot, TMEM_COLS);  // collective with the peer CTA's warp 2
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, TMEM_COLS);
      tmem_relinquish();
    }
  }
  if constexpr (EPI == kEpiGeluAbsmax || EPI == kEpiBF16CorrGelu) {
    for (int i = threadIdx.x; i < kGeluEntries; i += NUM_THREADS)
      gelu_tab[i] = (uint16_t)bf16_bits(gelu_tanh_exact(__uint_as_float(gelu_table_bits((uint32_t)i) << 16)));
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) cluster_sync_all();  // the peer's barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  RqCursor rq{};  // warps 2-11: this warp's units of A (kEpiGatedResidualRq)
  if constexpr (kRq) {
    if (warp >= 2) {
      rq.u = (int64_t)blockIdx.x * kRqSlots + (warp - 2);
      rq.stride = (int64_t)gridDim.x * kRqSlots;
      rq.lead = requant_lead(p, ncl);
      rq.hz = 0u;
      if (warp < EPI_WARP0) requant_finish<kTileRows>(p, rq, lane);
    }
  }

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int it = 0;
      bool ok = true;
      for (int tile = cid; tile < p.num_tiles && ok; tile += ncl) {
        int m_blk, n_blk;
        tile_coords(tile, p, m_blk, n_blk);
        const int a_row = m_blk * kTileRows + (int)rank * BM;
        // kEpiSwiGLU: a tile is 128 output columns; its B rows are the 128 gate rows
        // then the 128 up rows of those columns (rank 1 of a pair loads the up rows)
        const int b_row = EPI == kEpiSwiGLU ? n_blk * (BN / 2) + (int)rank * p.up_row
                                            : n_blk * BN + (int)rank * (BN / CG);
        if constexpr (kRq) {
          atomicMax(p.rq_horizon, (unsigned)m_blk);
          if (!requant_wait(p, m_blk, kTileRows)) break;  // A rows not written in time
        }
        for (int kb = 0; kb < p.num_k_blk; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t ph = (uint32_t)(it / kStages) & 1u;
          if (!mbar_wait(&empty_bar[s], ph ^ 1u, kErrProducer)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * kStageBytes;
          if constexpr (CG == 2) {
            if (rank == 0) mbar_arrive_expect_tx(&full_bar[s], 2 * kStageBytes);  // both CTAs' bytes
            const uint32_t bar0 = mapa_shared(&full_bar[s], 0);
            tma_load_2d_pair(sa, &tmA, bar0, kb * BK, a_row);
            tma_load_2d_pair(sa + A_BYTES, &tmB, bar0, kb * BK, b_row);
          } else {
            mbar_arrive_expect_tx(&full_bar[s], kStageBytes);
            tma_load_2d(sa, &tmA, &full_bar[s], kb * BK, a_row);
            tma_load_2d(sa + A_BYTES, &tmB, &full_bar[s], kb * BK, b_row);
            if constexpr (EPI == kEpiSwiGLU)  // 128-row box: the up rows fill B rows [128, 256)
              tma_load_2d(sa + A_BYTES + (BN / 2) * BK, &tmB, &full_bar[s], kb * BK, b_row + p.up_row);
          }
        }
      }
      // Let every copy this thread issued land before the CTA can exit: its
      // full barrier (CG = 1), or the release of the stage by the MMA that read
      // it (CG = 2: the full barrier is rank 0's).
      for (int j = (it > kStages ? it - kStages : 0); j < it; ++j) {
        if constexpr (CG == 2)
          mbar_wait(&empty_bar[j % kStages], (uint32_t)(j / kStages) & 1u, kErrDrain, 200000000ull);
        else
          mbar_wait(&full_bar[j % kStages], (uint32_t)(j / kStages) & 1u, kErrDrain, 200000000ull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------- MMA issuer (rank 0 of a pair) ----------------
      int it = 0;
      int tcount = 0;
      bool ok = true;
      bool issued = false;
      for (int tile = cid; tile < p.num_tiles && ok; tile += ncl, ++tcount) {
        const int acc = tcount & 1;
        const uint32_t acc_ph = (uint32_t)(tcount >> 1) & 1u;
        const bool freed = CG == 2 ? mbar_wait_cluster(&tempty_bar[acc], acc_ph ^ 1u, kErrMmaAcc)
                                   : mbar_wait(&tempty_bar[acc], acc_ph ^ 1u, kErrMmaAcc);
        if (!freed) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < p.num_k_blk; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t ph = (uint32_t)(it / kStages) & 1u;
          if (!mbar_wait(&full_bar[s], ph, kErrMmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * kStageBytes);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk) {
            const uint32_t accum = (kb > 0 || kk > 0) ? 1u : 0u;
            if constexpr (CG == 2)
              umma_i8_pair(d_tmem, umma_desc_sw128(a_addr + kk * 32), umma_desc_sw128(b_addr + kk * 32),
                           IDESC_I8_PAIR, accum);
            else
              umma_i8(d_tmem, umma_desc_sw128(a_addr + kk * 32), umma_desc_sw128(b_addr + kk * 32), IDESC_I8,
                      accum);
          }
          issued = true;
          if constexpr (CG == 2) {  // the stage is free in both CTAs
            umma_commit_pair(mapa_shared(&empty_bar[s], 0));
            umma_commit_pair(mapa_shared(&empty_bar[s], 1));
          } else {
            umma_commit(&empty_bar[s]);
          }
        }
        if (ok) {
          if constexpr (CG == 2) {  // accumulator ready in both CTAs
            umma_commit_pair(mapa_shared(&tfull_bar[acc], 0));
            umma_commit_pair(mapa_shared(&tfull_bar[acc], 1));
          } else {
            umma_commit(&tfull_bar[acc]);
          }
        }
      }
      if (issued) {
        // All MMAs this thread issued complete before TMEM can be released.
        if constexpr (CG == 2)
          umma_commit_pair(mapa_shared(drain_bar, 0));
        else
          umma_commit(drain_bar);
        mbar_wait(drain_bar, 0u, kErrDrain, 200000000ull);
      }
    }
  } else if (warp >= EPI_WARP0) {
    // ---------------- epilogue ----------------
    const int ew = warp - EPI_WARP0;
    const int quarter = warp & 3;          // TMEM lanes [32*quarter, 32*quarter + 32)
    const int half = ew >> 2;              // columns [128*half, 128*half + 128)
    float* ws_s = ops_smem + ew * 256;     // this warp's 128 column scales ...
    float* aux_s = ws_s + 128;             // ... and 128 bias / gate values
    // kEpiGatedResidual with a bias: 128 staged bias values per warp in the GELU
    // table's region (unused by this epilogue)
    float* bias_s = reinterpret_cast<float*>(gelu_tab) + ew * 128;
    uint8_t* box = smem + OFF_EPI + ew * EPI_STAGE_BYTES;  // this warp's 32x32 bf16 output box
    // row `lane` of the box, 16-byte chunk q, at the 64-byte-swizzle position q ^ ((lane >> 1) & 3)
    uint8_t* box_row = box + lane * 64;
    const int box_sw = (lane >> 1) & 3;
    const bool corr_thread = kCorr && ew == 0 && lane == 0;  // loads the correction operands, issues its MMAs
    int tcount = 0;
    uint32_t in_phase = 0;
    bool in_pending = false;  // an input-box load was issued and not yet waited for
    bool ok = true;
    for (int tile = cid; tile < p.num_tiles && ok; tile += ncl, ++tcount) {
      int m_blk, n_blk;
      tile_coords(tile, p, m_blk, n_blk);
      const int acc = tcount & 1;
      const uint32_t acc_ph = (uint32_t)(tcount >> 1) & 1u;
      const int row0 = m_blk * kTileRows + (int)rank * BM;  // this CTA's first row of the tile
      const int row = row0 + quarter * 32 + lane;
      // kEpiSwiGLU: output columns [64 half, 64 half + 64) of the tile's 128
      const int col_base = EPI == kEpiSwiGLU ? n_blk * (BN / 2) + half * 64 : n_blk * BN + half * 128;
      if constexpr (kCorr) {
        // This tile's correction operands. The previous tile's correction MMAs
        // have completed (its cf_bar phase), so their buffers are free.
        if (corr_thread) {
          const uint32_t bytes = (uint32_t)p.corr_kb * (uint32_t)(BM + BN / CG) * 128u;
          if constexpr (CG == 2) {
            if (rank == 0) mbar_arrive_expect_tx(corr_full_bar, 2 * bytes);  // both CTAs' bytes
            const uint32_t bar0 = mapa_shared(corr_full_bar, 0);
            for (int kb = 0; kb < p.corr_kb; ++kb) {
              tma_load_2d_pair(corr_sx + kb * (BM * 128), &tmS, bar0, kb * 64, row0);
              tma_load_2d_pair(corr_ct + kb * ((BN / CG) * 128), &tmC, bar0, kb * 64,
                               n_blk * BN + (int)rank * (BN / CG));
            }
          } else {
            mbar_arrive_expect_tx(corr_full_bar, bytes);
            for (int kb = 0; kb < p.corr_kb; ++kb) {
              tma_load_2d(corr_sx + kb * (BM * 128), &tmS, corr_full_bar, kb * 64, row0);
              tma_load_2d(corr_ct + kb * (BN * 128), &tmC, corr_full_bar, kb * 64, n_blk * BN);
            }
          }
        }
      }
      if constexpr (EPI != kEpiI32) {
        // stage this tile's per-column operands while the MMAs run
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int c = lane + 32 * i;
          // kEpiSwiGLU: entries [0, 64) are the warp's gate columns, [64, 128) their up rows
          const int col = EPI == kEpiSwiGLU ? col_base + (c & 63) : col_base + c;
          const int wrow = EPI == kEpiSwiGLU && c >= 64 ? col + p.up_row : col;  // row of W
          const bool cok = col < p.n;
          ws_s[c] = cok ? __ldg(p.w_scale + (p.w_pc ? wrow : 0)) : 0.0f;
          float a = 0.0f;
          if ((EPI == kEpiBF16 || EPI == kEpiBF16Corr || EPI == kEpiQKV || EPI == kEpiSwiGLU) && p.bias != nullptr &&
              cok)
            a = (EPI == kEpiBF16 && p.out_f16) ? __half2float(reinterpret_cast<const __half*>(p.bias)[wrow])
                                               : __bfloat162float(p.bias[wrow]);
          if (kInBox && cok && (EPI != kEpiGatedResidual || p.row_map == nullptr)) a = __bfloat162float(p.gate[col]);
          aux_s[c] = a;
          if (EPI == kEpiGatedResidual && p.bias != nullptr) bias_s[c] = cok ? __bfloat162float(p.bias[col]) : 0.0f;
          if constexpr (EPI == kEpiQKV) {  // this head's RMSNorm weight (Q and K sections)
            const int sec = p.qkv_sec0 + col_base / p.qkv_inner;
            bias_s[c] = sec < 2 ? __bfloat162float(p.qk_w[sec][c]) : 0.0f;
          }
        }
        __syncwarp();
      }
      if constexpr (kRq) {
        // quantize this warp's units of A while the accumulator is not ready
        for (;;) {
          const uint32_t ready = mbar_test(&tfull_bar[acc], acc_ph) ? 1u : 0u;
          if (__shfl_sync(0xffffffffu, ready, 0) != 0u) break;
          if (!requant_step<kTileRows>(p, rq, lane)) break;
        }
      }
      if (!mbar_wait(&tfull_bar[acc], acc_ph, kErrEpi)) break;
      tc_fence_after();
      float xs = 0.0f;
      if constexpr (kRq) {  // A was quantized in this kernel: its row scale from the row absmax
        xs = (row < p.m) ? row_scale(__ldg(p.row_absmax + row)) : 0.0f;
      } else if constexpr (EPI != kEpiI32) {
        xs = (row < p.m) ? __ldg(p.a_scale + row) : 0.0f;
      }
      uint32_t amax_bits = 0u;
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN + half * 128);
      const int box_row0 = row0 + quarter * 32;
      if constexpr (EPI == kEpiSwiGLU) {
        // Accumulator columns [0, 128) are the gate and [128, 256) the up projection
        // of the tile's 128 output columns; this warp combines its 64 of them.
        const uint32_t tg = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN + half * 64);
#pragma unroll 1
        for (int c = 0; c < 64; c += 32) {
          uint32_t rg[32], ru[32];
          tmem_ld32(tg + c, rg);
          tmem_ld32(tg + 128 + c, ru);
          tmem_wait_ld();
          if (col_base + c >= p.n || box_row0 >= p.m) continue;  // warp-uniform: nothing to store
          if (lane == 0) bulk_wait_read_all();  // the previous box has been read by its store
          uint32_t ob[16];
#pragma unroll
          for (int q = 0; q < 8; ++q) {  // 4 columns: one float4 of each staged operand
            const float4 wg = *reinterpret_cast<const float4*>(ws_s + c + 4 * q);
            const float4 wu = *reinterpret_cast<const float4*>(ws_s + 64 + c + 4 * q);
            const float wgv[4] = {wg.x, wg.y, wg.z, wg.w}, wuv[4] = {wu.x, wu.y, wu.z, wu.w};
            float bgv[4] = {0.f, 0.f, 0.f, 0.f}, buv[4] = {0.f, 0.f, 0.f, 0.f};
            if (p.bias != nullptr) {
              const float4 bg = *reinterpret_cast<const float4*>(aux_s + c + 4 * q);
              const float4 bu = *reinterpret_cast<const float4*>(aux_s + 64 + c + 4 * q);
              bgv[0] = bg.x; bgv[1] = bg.y; bgv[2] = bg.z; bgv[3] = bg.w;
              buv[0] = bu.x; buv[1] = bu.y; buv[2] = bu.z; buv[3] = bu.w;
            }
            uint32_t hb[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              uint32_t g = dequant_bits(rg[4 * q + e], xs, wgv[e]), u = dequant_bits(ru[4 * q + e], xs, wuv[e]);
              if (p.bias != nullptr) {
                g = bf16_bits(__fadd_rn(__uint_as_float(g << 16), bgv[e]));
                u = bf16_bits(__fadd_rn(__uint_as_float(u << 16), buv[e]));
              }
              // bf16(bf16(silu(g)) * u): the product of two bf16 values is exact in fp32
              hb[e] = bf16_bits(__fmul_rn(__uint_as_float(silu_bf16_fast(g) << 16), __uint_as_float(u << 16)));
            }
            ob[2 * q] = hb[0] | (hb[1] << 16);
            ob[2 * q + 1] = hb[2] | (hb[3] << 16);
          }
          __syncwarp();
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4*>(box_row + ((q ^ box_sw) << 4)) =
                make_uint4(ob[4 * q], ob[4 * q + 1], ob[4 * q + 2], ob[4 * q + 3]);
          fence_proxy_async_shared();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmO, box, col_base + c, box_row0);  // rows >= m and columns >= n are clipped
            bulk_commit_group();
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {  // release the accumulator on the MMA issuer's barrier
          if constexpr (CG == 2)
            mbar_arrive_cluster(mapa_shared(&tempty_bar[acc], 0));
          else
            mbar_arrive(&tempty_bar[acc]);
        }
      } else if constexpr (EPI == kEpiQKV) {
        // The warp's 128 columns are one head of one section; each thread holds its
        // token's head in registers: dequant (+ bias), then for Q / K the RMSNorm over
        // the 128 values (sum of squares in double, in-thread) and the RoPE pairs,
        // then four 32x32 boxes stored by TMA into the section's [m, heads, 128] view.
        const bool live_cols = col_base < p.n;  // warp-uniform
        const int sec = p.qkv_sec0 + col_base / p.qkv_inner;
        const int head = (col_base % p.qkv_inner) >> 7;
        uint32_t h[64];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld32(taddr + 32 * c, r);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            uint32_t b0 = dequant_bits(r[2 * j], xs, ws_s[32 * c + 2 * j]);
            uint32_t b1 = dequant_bits(r[2 * j + 1], xs, ws_s[32 * c + 2 * j + 1]);
            if (p.bias != nullptr) {
              b0 = bf16_bits(__fadd_rn(__uint_as_float(b0 << 16), aux_s[32 * c + 2 * j]));
              b1 = bf16_bits(__fadd_rn(__uint_as_float(b1 << 16), aux_s[32 * c + 2 * j + 1]));
            }
            h[16 * c + j] = b0 | (b1 << 16);
          }
        }
        // the accumulator is in registers: release it to the MMA issuer
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (CG == 2)
            mbar_arrive_cluster(mapa_shared(&tempty_bar[acc], 0));
          else
            mbar_arrive(&tempty_bar[acc]);
        }
        if (!live_cols || box_row0 >= p.m) continue;  // warp-uniform: nothing of this head to store
        if (sec < 2) {
          double sq[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            const double a = qkv_abs_lo(h[j]), b = qkv_abs_hi(h[j]);
            sq[j & 3] = fma(a, a, sq[j & 3]);
            sq[j & 3] = fma(b, b, sq[j & 3]);
          }
          float ms = (float)(((sq[0] + sq[1]) + (sq[2] + sq[3])) * 0.0078125);
          if (!isfinite(ms)) {  // inf / NaN / huge: exact conversions
            double se = 0.0;
#pragma unroll
            for (int j = 0; j < 64; ++j) {
              const double a = (double)bf16_lo(h[j]), b = (double)bf16_hi(h[j]);
              se = fma(a, a, se);
              se = fma(b, b, se);
            }
            ms = (float)(se * 0.0078125);
          }
          const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, p.qk_eps)));
          const uint64_t rs2 = f2_dup(rs);
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            uint32_t lo, hi;
            f2_bits(f2_mul(f2_mul(bf16x2_to_f2(h[j]), rs2), qkv_f2(bias_s[2 * j], bias_s[2 * j + 1])), lo, hi);
            h[j] = bf16x2_from_bits(lo, hi);
          }
          switch (p.qkv_rot) {
            case 32: qkv_rope<16>(h, p.rope_t, p.m, row); break;
            case 64: qkv_rope<32>(h, p.rope_t, p.m, row); break;
            case 96: qkv_rope<48>(h, p.rope_t, p.m, row); break;
            case 128: qkv_rope<64>(h, p.rope_t, p.m, row); break;
            default: break;  // RMSNorm only
          }
        }
        const CUtensorMap* omap = sec == 0 ? &tmO : (sec == 1 ? &tmR : &tmS);
        const bool hmaj = (p.qkv_hmaj >> sec) & 1;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (lane == 0) bulk_wait_read_all();  // the previous box has been read by its store
          __syncwarp();
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4*>(box_row + ((q ^ box_sw) << 4)) =
                make_uint4(h[16 * c + 4 * q], h[16 * c + 4 * q + 1], h[16 * c + 4 * q + 2], h[16 * c + 4 * q + 3]);
          fence_proxy_async_shared();
          __syncwarp();
          if (lane == 0) {
            if (hmaj)
              tma_store_3d(omap, box, 32 * c, head, box_row0);   // tokens >= m are clipped
            else
              tma_store_3d(omap, box, 32 * c, box_row0, head);
            bulk_commit_group();
          }
        }
      } else {
        if constexpr (kCorr) {
          // pass 1: the dequantized values replace the int32 accumulators
  #pragma unroll 1
          for (int c = 0; c < 128; c += 32) {
            uint32_t r[32];
            tmem_ld32(taddr + c, r);
            tmem_wait_ld();
            if (EPI == kEpiBF16Corr && p.bias != nullptr)
              dequant_bias_to_f32(r, xs, ws_s + c, aux_s + c);
            else
              dequant_to_f32(r, xs, ws_s + c);
            tmem_st32(taddr + c, r);
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if constexpr (CG == 2)
              mbar_arrive_cluster(mapa_shared(dq_bar, 0));
            else
              mbar_arrive(dq_bar);
          }
          const uint32_t ph = (uint32_t)tcount & 1u;
          if (corr_thread && rank == 0) {
            // D[rows, cols] += sx[rows, :kp] . corr_t[cols, :kp]^T: kind::f16, fp32 accumulate
            const bool ready = (CG == 2 ? mbar_wait_cluster(dq_bar, ph, kErrCorr) : mbar_wait(dq_bar, ph, kErrCorr)) &&
                               mbar_wait(corr_full_bar, ph, kErrCorr);
            if (ready) {
              tc_fence_after();
              const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
              for (int kb = 0; kb < p.corr_kb; ++kb) {
                const uint32_t a_addr = smem_u32(corr_sx + kb * (BM * 128));
                const uint32_t b_addr = smem_u32(corr_ct + kb * ((BN / CG) * 128));
  #pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                  if constexpr (CG == 2)
                    umma_bf16_pair(d_tmem, umma_desc_sw128(a_addr + kk * 32), umma_desc_sw128(b_addr + kk * 32),
                                   IDESC_BF16_PAIR, 1u);
                  else
                    umma_bf16(d_tmem, umma_desc_sw128(a_addr + kk * 32), umma_desc_sw128(b_addr + kk * 32),
                              IDESC_BF16, 1u);
                }
              }
              if constexpr (CG == 2) {
                umma_commit_pair(mapa_shared(cf_bar, 0));
                umma_commit_pair(mapa_shared(cf_bar, 1));
              } else {
                umma_commit(cf_bar);
              }
            }
          }
          if (!mbar_wait(cf_bar, ph, kErrEpi)) break;
          tc_fence_after();
        }
  #pragma unroll 1
        for (int c = 0; c < 128; c += 32) {
          uint32_t r[32];
          tmem_ld32(taddr + c, r);
          tmem_wait_ld();
          if (col_base + c >= p.n) continue;  // warp-uniform
          if constexpr (EPI == kEpiI32) {
            if (p.peer_world > 0)
              store_i32_chunk_routed(p, box_row0, col_base + c, r, box, lane);
            else
              store_i32_chunk(p, row, col_base + c, r);
          } else {
            if (box_row0 >= p.m) continue;      // warp-uniform: no row of this box exists
            if (lane == 0) bulk_wait_read_all();  // the previous box has been read by its store
            uint32_t in_w[16];
            if constexpr (kInBox) {
              if (lane == 0) {
                mbar_arrive_expect_tx(&in_bar[ew], EPI_STAGE_BYTES);
                tma_load_2d(box, &tmR, &in_bar[ew], col_base + c, box_row0);
              }
              in_pending = true;
              if (!mbar_wait(&in_bar[ew], in_phase, kErrEpiIn)) {
                ok = false;
                break;
              }
              in_pending = false;
              in_phase ^= 1u;
  #pragma unroll
              for (int q = 0; q < 4; ++q) {
                const uint4 v = *reinterpret_cast<const uint4*>(box_row + ((q ^ box_sw) << 4));
                in_w[4 * q] = v.x; in_w[4 * q + 1] = v.y; in_w[4 * q + 2] = v.z; in_w[4 * q + 3] = v.w;
              }
            } else {
  #pragma unroll
              for (int j = 0; j < 16; ++j) in_w[j] = 0u;
            }
            uint32_t gw[16];  // the row's gate values (kEpiGatedResidual with a row map)
  #pragma unroll
            for (int j = 0; j < 16; ++j) gw[j] = 0u;
            if constexpr (EPI == kEpiGatedResidual) {
              if (p.row_map != nullptr && row < p.m) {
                const __nv_bfloat16* grow = p.gate + (int64_t)__ldg(p.row_map + row) * p.ldg + col_base + c;
  #pragma unroll
                for (int q = 0; q < 4; ++q) {
                  if (col_base + c + 8 * q < p.n) {
                    const uint4 v = __ldg(reinterpret_cast<const uint4*>(grow + 8 * q));
                    gw[4 * q] = v.x; gw[4 * q + 1] = v.y; gw[4 * q + 2] = v.z; gw[4 * q + 3] = v.w;
                  }
                }
              }
            }
            uint32_t ob[16];
            epilogue_values<EPI>(p, r, xs, ws_s + c, aux_s + c, gelu_tab, amax_bits, in_w, bias_s + c, gw, ob);
            __syncwarp();
  #pragma unroll
            for (int q = 0; q < 4; ++q)
              *reinterpret_cast<uint4*>(box_row + ((q ^ box_sw) << 4)) =
                  make_uint4(ob[4 * q], ob[4 * q + 1], ob[4 * q + 2], ob[4 * q + 3]);
            fence_proxy_async_shared();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmO, box, col_base + c, box_row0);  // rows >= m and columns >= n are clipped
              bulk_commit_group();
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {  // release the accumulator on the MMA issuer's barrier
          if constexpr (CG == 2)
            mbar_arrive_cluster(mapa_shared(&tempty_bar[acc], 0));
          else
            mbar_arrive(&tempty_bar[acc]);
        }
        if constexpr (EPI == kEpiGeluAbsmax) {
          if (row < p.m) atomicMax(reinterpret_cast<unsigned int*>(p.row_absmax) + row, amax_bits << 16);
        }
      }
    }
    if constexpr (kRq) requant_finish<kTileRows>(p, rq, lane);  // units other tiles may still need
    if constexpr (kInBox) {
      if (in_pending) mbar_wait(&in_bar[ew], in_phase, kErrDrain, 200000000ull);  // let a late box land
    }
    if constexpr (EPI != kEpiI32) {
      if (lane == 0) bulk_wait_all();  // every output box written before the CTA exits
      __syncwarp();
    }
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) cluster_sync_all();  // the pair's MMAs, remote arrivals and epilogues are all done
  if (warp == 2) {
    tc_fence_after();
    if constexpr (CG == 2)
      tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else
      tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
bool make_tmap_i8(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld_bytes, int box_rows) {
  return encode_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, base, (uint64_t)cols, (uint64_t)rows, (uint64_t)ld_bytes,
                        (uint32_t)BK, (uint32_t)box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
}

struct TensorMaps {
  CUtensorMap a, b, out, res, sx, corr;
};

template <int EPI, int CG>
cudaError_t launch_epi(const TensorMaps& t, const KParams& kp, int grid, cudaStream_t stream) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(gemm_i8_kernel<EPI, CG>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  if constexpr (CG == 1) {
    gemm_i8_kernel<EPI, 1><<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(t.a, t.b, t.out, t.res, t.sx, t.corr, kp);
    return cudaGetLastError();
  } else {
    // a persistent grid must be fully resident: clamp to the clusters of two
    // 227 KB CTAs the device can co-schedule
    static int max_clusters[64] = {0};
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(NUM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (dev >= 0 && dev < 64 && max_clusters[dev] == 0) {
      cfg.gridDim = dim3((unsigned)grid, 1, 1);
      int n = 0;
      cudaError_t e = cudaOccupancyMaxActiveClusters(&n, gemm_i8_kernel<EPI, 2>, &cfg);
      if (e != cudaSuccess) return e;
      if (n < 1) return cudaErrorNotSupported;
      max_clusters[dev] = n;
    }
    if (dev >= 0 && dev < 64 && grid > 2 * max_clusters[dev]) grid = 2 * max_clusters[dev];
    cfg.gridDim = dim3((unsigned)grid, 1, 1);
    cfg.blockDim = dim3(NUM_THREADS, 1, 1);
    return cudaLaunchKernelEx(&cfg, gemm_i8_kernel<EPI, 2>, t.a, t.b, t.out, t.res, t.sx, t.corr, kp);
  }
}

template <int CG>
cudaError_t launch_cg(int epilogue, const TensorMaps& t, const KParams& kp, int grid, cudaStream_t stream) {
  switch (epilogue) {
    case kEpiI32:
      if (kp.rq_src != nullptr) return launch_epi<kEpiI32Rq, CG>(t, kp, grid, stream);
      return launch_epi<kEpiI32, CG>(t, kp, grid, stream);
    case kEpiBF16: return launch_epi<kEpiBF16, CG>(t, kp, grid, stream);
    case kEpiGeluAbsmax: return launch_epi<kEpiGeluAbsmax, CG>(t, kp, grid, stream);
    case kEpiGatedResidual:
      if (kp.rq_src != nullptr) return launch_epi<kEpiGatedResidualRq, CG>(t, kp, grid, stream);
      return launch_epi<kEpiGatedResidual, CG>(t, kp, grid, stream);
    case kEpiBF16Corr: return launch_epi<kEpiBF16Corr, CG>(t, kp, grid, stream);
    case kEpiBF16CorrGelu: return launch_epi<kEpiBF16CorrGelu, CG>(t, kp, grid, stream);
    case kEpiGatedResidualCorr: return launch_epi<kEpiGatedResidualCorr, CG>(t, kp, grid, stream);
    case kEpiQKV: return launch_epi<kEpiQKV, CG>(t, kp, grid, stream);
    case kEpiSwiGLU: return launch_epi<kEpiSwiGLU, CG>(t, kp, grid, stream);
    default: return cudaErrorNotSupported;
  }
}

}  // namespace

namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}
}  // namespace

bool encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t rows,
                    uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return false;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 3-D tiled map over bf16 [d2][d1][d0] with byte strides s1, s2 (box b0 x b1 x b2)
bool encode_tmap_3d_bf16(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
                         uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return false;
  cuuint64_t dims[3] = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)d2};
  cuuint64_t strides[2] = {(cuuint64_t)s1, (cuuint64_t)s2};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int num_sms(int device) {
  static int cache[64] = {0};
  if (device < 0 || device >= 64) return 148;
  if (cache[device] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0) v = 148;
    cache[device] = v;
  }
  return cache[device];
}

cudaError_t launch_gemm_i8(const GemmArgs& a, cudaStream_t stream) {
  if (a.m <= 0 || a.n <= 0) return cudaSuccess;
  if (a.k <= 0 || a.k % 16 != 0 || a.n % 8 != 0 || a.lda % 16 != 0 || a.ldw % 16 != 0 || a.m > (1ll << 30) ||
      a.n > (1ll << 30) || a.k > (1ll << 30))
    return cudaErrorNotSupported;
  const bool qkv = a.epilogue == kEpiQKV;
  if ((reinterpret_cast<uintptr_t>(a.a) & 15) || (reinterpret_cast<uintptr_t>(a.w) & 15) ||
      (!qkv && ((reinterpret_cast<uintptr_t>(a.out) & 15) || a.ldo % 8 != 0)))
    return cudaErrorNotSupported;
  int qkv_hmaj = 0;
  if (qkv) {
    const int64_t inner = a.qkv_heads * 128;
    const int nsec = inner > 0 ? (int)(a.n / inner) : 0;
    if (a.qkv_heads <= 0 || a.n % inner != 0 || a.qkv_sec0 < 0 || a.qkv_sec0 + nsec > 3 || nsec < 1 ||
        inner > (1ll << 30) || (a.rope_t == nullptr ? a.qkv_rot != 0 : (a.qkv_rot % 32 || a.qkv_rot < 32 || a.qkv_rot > 128)))
      return cudaErrorNotSupported;
    for (int s = a.qkv_sec0; s < a.qkv_sec0 + nsec; ++s) {
      if (a.qkv_out[s] == nullptr || (reinterpret_cast<uintptr_t>(a.qkv_out[s]) & 15) || a.qkv_st[s] % 8 ||
          a.qkv_sh[s] % 8 || a.qkv_st[s] <= 0 || a.qkv_sh[s] <= 0 || (s < 2 && a.qk_w[s] == nullptr))
        return cudaErrorNotSupported;
      if (a.qkv_sh[s] < a.qkv_st[s]) qkv_hmaj |= 1 << s;  // heads inside a token row: (dim, head, token) order
    }
  }
  // kEpiSwiGLU: W's n rows are [gate | up]; the output is n / 2 columns wide
  const bool swiglu = a.epilogue == kEpiSwiGLU;
  if (swiglu && a.n % 16 != 0) return cudaErrorNotSupported;
  const int64_t n_out = swiglu ? a.n / 2 : a.n;
  if (swiglu) {
    const cudaError_t e = ensure_act_table(H3B200_ACT_SWIGLU, stream);
    if (e != cudaSuccess) return e;
  }
  const bool gated = a.epilogue == kEpiGatedResidual || a.epilogue == kEpiGatedResidualCorr;
  if (gated && ((reinterpret_cast<uintptr_t>(a.residual) & 15) || a.ldr % 8 != 0)) return cudaErrorNotSupported;
  if (a.row_map != nullptr && (a.epilogue != kEpiGatedResidual || a.ldg < a.n || a.ldg % 8 != 0 ||
                               (reinterpret_cast<uintptr_t>(a.gate) & 15)))
    return cudaErrorNotSupported;
  if (a.requant_src != nullptr &&
      ((a.epilogue != kEpiGatedResidual && a.epilogue != kEpiI32) || a.lda != a.k || a.k % 8 != 0 || a.requant_lds < a.k ||
       a.requant_lds % 8 != 0 || (reinterpret_cast<uintptr_t>(a.requant_src) & 15) || a.row_absmax == nullptr ||
       a.requant_ready == nullptr))
    return cudaErrorNotSupported;
  if (a.out_f16 != 0 && a.epilogue != kEpiBF16) return cudaErrorNotSupported;
  if (a.peer_world != 0) {
    if (a.epilogue != kEpiI32 || a.peer_world < 0 || a.peer_world > kTpMaxWorld || a.ldo % 4 != 0)
      return cudaErrorNotSupported;
    for (int o = 0; o < a.peer_world; ++o)
      if (a.peer_out[o] == nullptr || (reinterpret_cast<uintptr_t>(a.peer_out[o]) & 15)) return cudaErrorNotSupported;
  }
  const bool corr = a.epilogue == kEpiBF16Corr || a.epilogue == kEpiBF16CorrGelu || a.epilogue == kEpiGatedResidualCorr;
  if (corr && (a.sx == nullptr || a.corr_t == nullptr || a.kp <= 0 || a.kp % 64 != 0 || a.kp > kMaxCorrKp ||
               (reinterpret_cast<uintptr_t>(a.sx) & 15) || (reinterpret_cast<uintptr_t>(a.corr_t) & 15)))
    return cudaErrorNotSupported;
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = num_sms(dev);
  // CTA pairs (256 x 256 tiles, cta_group::2) for the GEMMs with enough tiles
  // to give every SM pair work; single CTAs otherwise.
  const int64_t n_blk = swiglu ? (n_out + BN / 2 - 1) / (BN / 2) : (a.n + BN - 1) / BN;
  const bool pair = ((a.m + 2 * BM - 1) / (2 * BM)) * n_blk >= sms / 2;
  const int cg = pair ? 2 : 1;
  TensorMaps t;
  if (!make_tmap_i8(&t.a, a.a, a.m, a.k, a.lda, BM) || !make_tmap_i8(&t.b, a.w, a.n, a.k, a.ldw, swiglu ? BN / 2 : BN / cg))
    return cudaErrorInvalidValue;
  if (qkv) {
    // one [m, heads, 128] map per present section, boxes of 32 dims x 32 tokens
    CUtensorMap* maps[3] = {&t.out, &t.res, &t.sx};
    const int nsec = (int)(a.n / (a.qkv_heads * 128));
    for (int s = 0; s < 3; ++s) {
      const int src_s = (s >= a.qkv_sec0 && s < a.qkv_sec0 + nsec) ? s : a.qkv_sec0;  // absent: any valid map
      const bool hm = (qkv_hmaj >> src_s) & 1;
      const uint64_t st = (uint64_t)a.qkv_st[src_s] * 2, sh = (uint64_t)a.qkv_sh[src_s] * 2;
      // (dim, token, head) with boxes 32 x 32 x 1, or (dim, head, token) with 32 x 1 x 32:
      // either way a box is 32 token rows of 64 bytes in shared memory
      if (!(hm ? encode_tmap_3d_bf16(maps[s], a.qkv_out[src_s], 128, (uint64_t)a.qkv_heads, (uint64_t)a.m, sh, st,
                                     32, 1, 32, CU_TENSOR_MAP_SWIZZLE_64B)
               : encode_tmap_3d_bf16(maps[s], a.qkv_out[src_s], 128, (uint64_t)a.m, (uint64_t)a.qkv_heads, st, sh,
                                     32, 32, 1, CU_TENSOR_MAP_SWIZZLE_64B)))
        return cudaErrorInvalidValue;
    }
  } else if (a.epilogue == kEpiI32) {
    t.out = t.b;  // unused: int32 results are stored directly
  } else if (!encode_tmap_2d(&t.out, a.out_f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                             a.out, (uint64_t)n_out, (uint64_t)a.m,
                             (uint64_t)a.ldo * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B)) {
    return cudaErrorInvalidValue;
  }
  if (qkv) {
    // t.res holds the K map
  } else if (gated) {
    if (!encode_tmap_2d(&t.res, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.residual, (uint64_t)a.n, (uint64_t)a.m,
                        (uint64_t)a.ldr * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
      return cudaErrorInvalidValue;
  } else {
    t.res = t.out;  // unused
  }
  if (corr) {
    // 64 groups (128 bytes) per k-block row, 128-byte swizzle: the UMMA operand layout of the mainloop tiles
    if (!encode_tmap_2d(&t.sx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.sx, (uint64_t)a.kp, (uint64_t)a.m,
                        (uint64_t)a.kp * 2, 64, BM, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tmap_2d(&t.corr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.corr_t, (uint64_t)a.kp, (uint64_t)a.n,
                        (uint64_t)a.kp * 2, 64, BN / cg, CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
  } else if (!qkv) {
    t.sx = t.a;  // unused
    t.corr = t.a;
  } else {
    t.corr = t.a;  // unused; t.sx holds the V map
  }
  KParams kp;
  kp.m = (int)a.m;
  kp.n = (int)n_out;
  kp.k = (int)a.k;
  kp.num_n_blk = (int)n_blk;
  kp.num_k_blk = (int)((a.k + BK - 1) / BK);
  const int64_t num_m_blk = (a.m + cg * BM - 1) / (cg * BM);
  const int64_t tiles = num_m_blk * kp.num_n_blk;
  if (tiles > (1ll << 30)) return cudaErrorNotSupported;
  kp.num_tiles = (int)tiles;
  kp.num_m_blk = (int)num_m_blk;
  // a weight that fits comfortably in the 126 MB L2 stays resident with N-fastest
  // order (group of one M-block); a larger one streams past once per group of 8
  kp.group_m = a.n * a.k <= (64ll << 20) ? 1 : (int)std::min<int64_t>(num_m_blk, 8);
  kp.a_scale = a.a_scale;
  kp.w_scale = a.w_scale;
  kp.w_pc = a.w_scale_per_channel;
  kp.bias = static_cast<const __nv_bfloat16*>(a.bias);
  kp.gate = static_cast<const __nv_bfloat16*>(a.gate);
  kp.residual = static_cast<const __nv_bfloat16*>(a.residual);
  kp.ldr = a.ldr;
  kp.out = a.out;
  kp.ldo = a.ldo;
  kp.row_absmax = a.row_absmax;
  kp.corr_kb = corr ? (int)(a.kp / 64) : 0;
  kp.row_map = a.epilogue == kEpiGatedResidual ? a.row_map : nullptr;
  kp.ldg = a.ldg;
  kp.qkv_inner = qkv ? (int)(a.qkv_heads * 128) : 1;
  kp.qkv_sec0 = a.qkv_sec0;
  kp.qkv_rot = a.rope_t != nullptr ? a.qkv_rot : 0;
  kp.qkv_hmaj = qkv_hmaj;
  kp.qk_w[0] = static_cast<const __nv_bfloat16*>(a.qk_w[0]);
  kp.qk_w[1] = static_cast<const __nv_bfloat16*>(a.qk_w[1]);
  kp.rope_t = a.rope_t;
  kp.qk_eps = a.qk_eps;
  kp.up_row = swiglu ? (int)n_out : 0;
  kp.rq_src = static_cast<const __nv_bfloat16*>(a.requant_src);
  kp.rq_lds = a.requant_lds;
  kp.rq_dst = const_cast<int8_t*>(a.a);
  kp.rq_ready = a.requant_ready;
  kp.rq_horizon = a.requant_ready == nullptr ? nullptr : a.requant_ready + (a.m + 127) / 128;
  kp.rq_upr = (int)((a.k + kRqUnit - 1) / kRqUnit);
  kp.rq_units = a.m * kp.rq_upr;
  for (int o = 0; o < kTpMaxWorld; ++o) kp.peer_out[o] = a.peer_out[o];
  kp.peer_world = a.peer_world;
  kp.out_f16 = a.out_f16;
  if (pair) return launch_cg<2>(a.epilogue, t, kp, 2 * (int)std::min<int64_t>(tiles, (int64_t)(sms / 2)), stream);
  return launch_cg<1>(a.epilogue, t, kp, (int)std::min<int64_t>(tiles, (int64_t)sms), stream);
}

}  // namespace h3
