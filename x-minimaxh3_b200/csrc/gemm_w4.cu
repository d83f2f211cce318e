// Small-M W4A8 linear: INT8 GEMM whose int4 weights are unpacked to int8 in shared
// memory, never materialised as an int8 grid in global memory.
//
//   out[m, n] = bf16(bf16(acc * (xs[m] * s_channel[n])) (+ bias[n]) (+ sum_g sx[m, g] * corr[g, n]))
//   acc = xq . W^T, W[n, k] = clamp(rne(level(u[n, k]) * s_rel[n, k / group]), -127, 127)
//
// Reference: w4a8_int8_linear (tensor/w4a8_int8.py:89-115; CUDA backends/cuda/__init__.py:
// 2139-2298, which decodes the int4 weight into an int8 workspace or an L2-resident
// N-chunk, backends/cuda/ops/w4a8_gemm.cu:36-164, before a CUTLASS GEMM). Decode arithmetic
// as the standalone decode kernel (w4_math.cuh), bit for bit.
//
// Why only for small M: with few token rows the linear is bound by reading the weight,
// and the per-call global decode (read 4 bits, write and re-read 8 bits per weight) costs
// more than the GEMM. Unpacking per tile reads the packed weight once per M block, so for
// M <= 32 (one block) the weight crosses HBM once at 4 bits per element; for large M the
// unpack would repeat per M block and the global decode wins (measured: above 32 rows, or
// 16 with the asymmetric correction, which this kernel sums on CUDA cores).
//
// Few rows make few output tiles (n / 256), so K is split over CTAs to fill the GPU in one
// wave: split z adds its int32 partial tile into a zeroed [m, n] buffer with red.add, and
// the last CTA of each tile (a per-tile counter) runs the epilogue on the sums.
//
// Structure (one CTA per 128 x 256 output tile and K split, 384 threads):
//   warp 0      TMA producer: per 128-deep k-block the int8 activation tile
//               (128 rows x 128 B, 128-byte swizzle) and the packed weight tile
//               (256 rows x 64 B, 64-byte swizzle) into a 3-stage ring.
//   warp 1      MMA issuer: tcgen05.mma.cta_group::1.kind::i8 (128 x 256 x 32) into one
//               TMEM accumulator once the stage's weights are unpacked.
//   warp 2      TMEM allocator.
//   warps 4-11  converters, then the epilogue. During the mainloop thread t unpacks weight
//               row t of each stage: a 16-entry int8 table of decode(level(u), s) for the
//               row's group scale, looked up four codes at a time with byte permutes, stored
//               as the 128-byte-swizzled K-major operand the tensor core reads. After the
//               last k-block they add the accumulator into the sums; in the tile's last CTA
//               thread t then finishes column t of every row: dequant (+ bias, rounded to
//               bf16) (+ the asymmetric correction from shared-memory copies of corr and
//               sx, fp32 sum, one rounding) and a bf16 store.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "quant_math.cuh"
#include "w4_math.cuh"

namespace h3 {
namespace {

constexpr int W4_BM = 128, W4_BN = 256, W4_BK = 128;
constexpr int W4_A_BYTES = W4_BM * W4_BK;       // int8 activations (TMA)
constexpr int W4_BQ_BYTES = W4_BN * W4_BK;      // unpacked int8 weights (converters)
constexpr int W4_BP_BYTES = W4_BN * W4_BK / 2;  // packed int4 weights (TMA)
constexpr int W4_OFF_BQ = W4_A_BYTES;
constexpr int W4_OFF_BP = W4_A_BYTES + W4_BQ_BYTES;
constexpr int W4_STAGE = W4_A_BYTES + W4_BQ_BYTES + W4_BP_BYTES;  // 64 KB
constexpr int W4_STAGES = 3;
constexpr int W4_OFF_BAR = W4_STAGES * W4_STAGE;
constexpr int W4_OFF_LV = W4_OFF_BAR + 128;  // 16 fp32 levels
constexpr int W4_SMEM = W4_OFF_LV + 64 + 1024;
constexpr int W4_THREADS = 384;
constexpr int W4_EPI0 = 4;
constexpr int W4_MAX_CORR_GROUPS = W4_STAGE / (W4_BN * 2);  // corr copy fits one stage
constexpr uint32_t W4_IDESC = umma_idesc_i8(W4_BM, W4_BN);
static_assert(W4_SMEM <= 232448, "small-M W4 GEMM shared memory exceeds the per-block limit");
constexpr unsigned kErrW4Prod = 0x201, kErrW4Mma = 0x202, kErrW4Conv = 0x203, kErrW4Epi = 0x204,
                   kErrW4Drain = 0x205;

struct W4Params {
  int m, n, k, nkb;
  const float* a_scale;       // [m]
  const float* s_channel;     // [n]
  const __nv_bfloat16* bias;  // [n] or null
  const void* s_rel;          // [n, gpr] fp32, or fp8-e4m3 bytes
  int e4m3;
  const float* codebook;      // 16 levels or null (level = u - 8)
  int group, gpr;             // group size along k, groups per row
  const __nv_bfloat16* sx;    // [m, kp] correction operand, or null
  int kp;
  const __nv_bfloat16* corr;  // [gpr, n] asymmetric correction, or null
  __nv_bfloat16* out;         // [m, ldo]
  int64_t ldo;
  // split-K: CTA z takes k-blocks [z * kb_per, (z + 1) * kb_per) and adds its int32
  // partials into acc_ws [m, n] (zero at launch); the last CTA of each output tile
  // (tile_cnt, zero at launch) runs the epilogue on the sums
  int splits, kb_per;
  int32_t* acc_ws;
  unsigned int* tile_cnt;
};

__device__ __forceinline__ float w4_scale(const W4Params& p, int row, int col) {
  const int64_t i = (int64_t)row * p.gpr + col / p.group;
  return p.e4m3 ? e4m3_to_f32(__ldg(static_cast<const uint8_t*>(p.s_rel) + i))
                : __ldg(static_cast<const float*>(p.s_rel) + i);
}

// Table of the 16 decoded bytes for scale s: byte u of word u / 4 is decode(level(u), s).
__device__ __forceinline__ void w4_table(const float (&lv)[16], bool lv_ok, float s, uint32_t (&t)[4]) {
  const bool fast = lv_ok && fabsf(s) <= 2048.0f;  // false for NaN
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t b[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) b[j] = fast ? decode_fast_bits(lv[4 * q + j], s) : decode_one(lv[4 * q + j], s);
    t[q] = __byte_perm(__byte_perm(b[0], b[1], 0x0040u), __byte_perm(b[2], b[3], 0x0040u), 0x5410u);
  }
}

// Four decoded bytes for the four codes in the low 16 bits of c (nibble i = code of
// output byte i): the low three bits pick a byte of the table's first or second half,
// bit 3 picks the half.
__device__ __forceinline__ uint32_t w4_lookup4(const uint32_t (&t)[4], uint32_t c) {
  const uint32_t idx = c & 0x7777u;
  const uint32_t lo = __byte_perm(t[0], t[1], idx);
  const uint32_t hi = __byte_perm(t[2], t[3], idx);
  return __byte_perm(lo, hi, 0x3210u | ((c >> 1) & 0x4444u));
}

__global__ void __launch_bounds__(W4_THREADS, 1)
    gemm_w4_smallm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmP,
                          const W4Params p) {
  extern __shared__ uint8_t w4_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(w4_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + W4_OFF_BAR);
  uint64_t* conv_bar = full_bar + W4_STAGES;
  uint64_t* empty_bar = conv_bar + W4_STAGES;
  uint64_t* acc_bar = empty_bar + W4_STAGES;
  uint64_t* corr_bar = acc_bar + 1;  // the epilogue warps' copy of corr and sx is complete
  uint64_t* split_bar = corr_bar + 1;  // the epilogue warps' partial sums are added
  uint64_t* flag_bar = split_bar + 1;  // the tile counter has been read
  uint32_t* last_flag = reinterpret_cast<uint32_t*>(flag_bar + 1);
  uint32_t* tmem_slot = last_flag + 1;
  float* lv_s = reinterpret_cast<float*>(smem + W4_OFF_LV);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * W4_BN, m0 = blockIdx.y * W4_BM;
  const int kb0 = blockIdx.z * p.kb_per;                 // this CTA's first k-block
  const int nkb = min(p.nkb - kb0, p.kb_per);            // and how many

  if (threadIdx.x == 0) {
    for (int s = 0; s < W4_STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&conv_bar[s], 8);  // one arrival per converter warp
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(acc_bar, 1);
    mbar_init(corr_bar, 8);
    mbar_init(split_bar, 8);
    mbar_init(flag_bar, 1);
    fence_barrier_init();
    fence_proxy_async_shared();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmP);
  }
  if (threadIdx.x < 16) lv_s[threadIdx.x] = p.codebook ? p.codebook[threadIdx.x] : (float)threadIdx.x - 8.0f;
  if (warp == 2) {
    tmem_alloc(tmem_slot, W4_BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int kb = 0;
      for (; kb < nkb; ++kb) {
        const int s = kb % W4_STAGES;
        const uint32_t ph = (uint32_t)(kb / W4_STAGES) & 1u;
        if (!mbar_wait(&empty_bar[s], ph ^ 1u, kErrW4Prod)) break;
        uint8_t* st = smem + s * W4_STAGE;
        mbar_arrive_expect_tx(&full_bar[s], W4_A_BYTES + W4_BP_BYTES);
        tma_load_2d(st, &tmA, &full_bar[s], (kb0 + kb) * W4_BK, m0);
        tma_load_2d(st + W4_OFF_BP, &tmP, &full_bar[s], (kb0 + kb) * (W4_BK / 2), n0);
      }
      for (int j = (kb > W4_STAGES ? kb - W4_STAGES : 0); j < kb; ++j)  // issued copies land before exit
        mbar_wait(&full_bar[j % W4_STAGES], (uint32_t)(j / W4_STAGES) & 1u, kErrW4Drain, 200000000ull);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      bool issued = false;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % W4_STAGES;
        const uint32_t ph = (uint32_t)(kb / W4_STAGES) & 1u;
        if (!mbar_wait(&full_bar[s], ph, kErrW4Mma) || !mbar_wait(&conv_bar[s], ph, kErrW4Mma)) break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem + s * W4_STAGE);
        const uint32_t b_addr = a_addr + W4_OFF_BQ;
#pragma unroll
        for (int kk = 0; kk < W4_BK / 32; ++kk)
          umma_i8(tmem_base, umma_desc_sw128(a_addr + kk * 32), umma_desc_sw128(b_addr + kk * 32), W4_IDESC,
                  (kb > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&empty_bar[s]);
        issued = true;
      }
      if (issued) umma_commit(acc_bar);  // arrives once every MMA above has completed
    }
  } else if (warp >= W4_EPI0) {
    const int ew = warp - W4_EPI0;
    // ---------------- converters: thread t unpacks weight row t of each stage ----------------
    const int t = ew * 32 + lane;
    const int nrow = n0 + t;
    float lv[16];
    bool lv_ok = true;
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      lv[u] = lv_s[u];
      lv_ok = lv_ok && fabsf(lv[u]) <= 8.0f;
    }
    const bool one_scale = p.group % W4_BK == 0;  // else the group divides 128
    bool ok = true;
    const int chunks_per_group = one_scale ? 8 : p.group / 16;
    for (int kb = 0; kb < nkb && ok; ++kb) {
      const int s = kb % W4_STAGES;
      const uint32_t ph = (uint32_t)(kb / W4_STAGES) & 1u;
      float sc[8];  // the k-block's group scales (chunk j uses sc[j - j % chunks_per_group]), loaded before the wait
#pragma unroll
      for (int j = 0; j < 8; ++j)
        sc[j] = (nrow < p.n && j % chunks_per_group == 0) ? w4_scale(p, nrow, (kb0 + kb) * W4_BK + 16 * j) : 0.0f;
      if (!mbar_wait(&full_bar[s], ph, kErrW4Conv)) {
        ok = false;
        break;
      }
      uint8_t* st = smem + s * W4_STAGE;
      if (nrow < p.n) {
        uint32_t w[16];  // packed word j: codes of k-block columns 8 j .. 8 j + 7, low nibble first
        const uint8_t* bp = st + W4_OFF_BP + t * 64;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 v = *reinterpret_cast<const uint4*>(bp + ((c ^ ((t >> 1) & 3)) << 4));
          w[4 * c] = v.x; w[4 * c + 1] = v.y; w[4 * c + 2] = v.z; w[4 * c + 3] = v.w;
        }
        uint8_t* bq = st + W4_OFF_BQ + t * 128;
        uint32_t tab[4];
        w4_table(lv, lv_ok, sc[0], tab);
#pragma unroll
        for (int j = 0; j < 8; ++j) {  // 16 columns 16 j .. 16 j + 15, stored as 16-byte chunk j of the row
          if (j > 0 && j % chunks_per_group == 0) w4_table(lv, lv_ok, sc[j], tab);
          const uint4 o = make_uint4(w4_lookup4(tab, w[2 * j]), w4_lookup4(tab, w[2 * j] >> 16),
                                     w4_lookup4(tab, w[2 * j + 1]), w4_lookup4(tab, w[2 * j + 1] >> 16));
          *reinterpret_cast<uint4*>(bq + ((j ^ (t & 7)) << 4)) = o;
        }
      }
      fence_proxy_async_shared();  // generic writes, read by the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv_bar[s]);
    }
    // ---------------- epilogue ----------------
    const int quarter = warp & 3, half = ew >> 2;
    const int row = m0 + quarter * 32 + lane;
    // this split's int32 partials (rows < m) are added into acc_ws (red.add, no return
    // value); the tile's last CTA (tile counter) finishes the tile from the sums
    bool done = ok && mbar_wait(acc_bar, 0u, kErrW4Epi);
    if (done) {
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(half * 128);
#pragma unroll 1
      for (int c = 0; c < 128; c += 32) {
        uint32_t r[32];
        tmem_ld32(taddr + c, r);
        tmem_wait_ld();
        const int col0 = n0 + half * 128 + c;
        if (row < p.m && col0 < p.n) {
          int32_t* a = p.acc_ws + (int64_t)row * p.n + col0;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col0 + j < p.n) atomicAdd(a + j, (int)r[j]);
        }
        __syncwarp();  // converge before the next tcgen05.ld
      }
      __threadfence();
      __syncwarp();
      if (lane == 0) mbar_arrive(split_bar);
      if (t == 0) {
        uint32_t flag = 2u;
        if (mbar_wait(split_bar, 0u, kErrW4Epi)) {
          __threadfence();
          const unsigned old = atomicAdd(p.tile_cnt + blockIdx.y * gridDim.x + blockIdx.x, 1u);
          flag = old == (unsigned)(p.splits - 1) ? 1u : 0u;
        }
        *reinterpret_cast<volatile uint32_t*>(last_flag) = flag;
        mbar_arrive(flag_bar);
      }
      done = mbar_wait(flag_bar, 0u, kErrW4Epi) && *reinterpret_cast<volatile uint32_t*>(last_flag) == 1u;
    }
    if (done) {
      __threadfence();  // every split's partials are visible before they are read
      // the ring is free: corr [gpr][256] bf16 and the tile's sx rows [rows][gpr] fp32 in shared memory
      const int rows = min(W4_BM, p.m - m0);
      __nv_bfloat16* corr_s = reinterpret_cast<__nv_bfloat16*>(smem);
      float* sx_s = reinterpret_cast<float*>(smem + W4_STAGE);
      bool staged = true;
      if (p.corr != nullptr) {
        for (int i = t; i < p.gpr * (W4_BN / 8); i += 256) {
          const int g = i / (W4_BN / 8), c8 = (i - g * (W4_BN / 8)) * 8;
          uint4 v = make_uint4(0u, 0u, 0u, 0u);
          if (n0 + c8 < p.n) v = __ldg(reinterpret_cast<const uint4*>(p.corr + (int64_t)g * p.n + n0 + c8));
          *reinterpret_cast<uint4*>(corr_s + g * W4_BN + c8) = v;
        }
        for (int i = t; i < rows * p.gpr; i += 256) {
          const int r = i / p.gpr, g = i - r * p.gpr;
          sx_s[i] = __bfloat162float(p.sx[(int64_t)(m0 + r) * p.kp + g]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(corr_bar);
        staged = mbar_wait(corr_bar, 0u, kErrW4Epi);
      }
      // thread t finishes column n0 + t of every row of the tile: consecutive threads on
      // consecutive columns (coalesced sums and stores); the sums of eight rows are loaded
      // together so the loads overlap
      const int col = n0 + t;
      if (staged && col < p.n) {
        const float ws = __ldg(p.s_channel + col);
        const float bv = p.bias != nullptr ? __bfloat162float(p.bias[col]) : 0.0f;
        for (int r0 = 0; r0 < rows; r0 += 8) {
          int32_t acc[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] = r0 + i < rows ? __ldcg(p.acc_ws + (int64_t)(m0 + r0 + i) * p.n + col) : 0;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            if (r0 + i >= rows) break;
            const int orow = m0 + r0 + i;
            float y = __uint_as_float(
                (uint32_t)bf16_bits(__fmul_rn(__int2float_rn(acc[i]), __fmul_rn(__ldg(p.a_scale + orow), ws))) << 16);
            if (p.bias != nullptr) y = bf16_round(__fadd_rn(y, bv));
            if (p.corr != nullptr) {
              const float* sr = sx_s + (r0 + i) * p.gpr;
              for (int g = 0; g < p.gpr; ++g) y = __fmaf_rn(sr[g], __bfloat162float(corr_s[g * W4_BN + t]), y);
            }
            p.out[(int64_t)orow * p.ldo + col] = __float2bfloat16_rn(y);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, W4_BN);
  }
}

}  // namespace

int gemm_w4_smallm_splits(int64_t m, int64_t n, int64_t k, int sms) {
  const int64_t tiles = ((n + W4_BN - 1) / W4_BN) * ((m + W4_BM - 1) / W4_BM);
  const int64_t nkb = k / W4_BK;
  if (tiles >= sms || nkb <= 1) return 1;
  // one wave (one CTA per SM): at most sms / tiles splits
  const int64_t want = std::max<int64_t>(1, std::min<int64_t>(nkb, sms / tiles));
  const int64_t per = (nkb + want - 1) / want;
  return (int)((nkb + per - 1) / per);  // every split non-empty
}

bool gemm_w4_smallm_supported(int64_t m, int64_t n, int64_t k, int64_t group, int64_t groups_corr) {
  // few rows: the weight read and its unpack dominate; the correction is summed on CUDA
  // cores in the epilogue, so with it the limit is lower (measured crossover: 32 rows without
  // a correction, 16 with one)
  return m > 0 && m <= (groups_corr > 0 ? 16 : 32) && n > 0 && n % 8 == 0 && k > 0 && k % W4_BK == 0 && group >= 16 && group % 16 == 0 &&
         (W4_BK % group == 0 || group % W4_BK == 0) && k % group == 0 && k < (1ll << 30) && n < (1ll << 30) &&
         groups_corr <= W4_MAX_CORR_GROUPS;
}

cudaError_t launch_gemm_w4_smallm(const W4SmallMArgs& a, cudaStream_t stream) {
  if (a.m <= 0 || a.n <= 0) return cudaSuccess;
  const int64_t gpr = a.k / a.group;
  if (!gemm_w4_smallm_supported(a.m, a.n, a.k, a.group, a.corr ? gpr : 0) || (a.corr && a.sx == nullptr) ||
      (reinterpret_cast<uintptr_t>(a.xq) & 15) || (reinterpret_cast<uintptr_t>(a.qdata) & 15) || a.ldo < a.n)
    return cudaErrorNotSupported;
  CUtensorMap tmA, tmP;
  if (!encode_tmap_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.xq, (uint64_t)a.k, (uint64_t)a.m, (uint64_t)a.k,
                      (uint32_t)W4_BK, (uint32_t)W4_BM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tmap_2d(&tmP, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.qdata, (uint64_t)(a.k / 2), (uint64_t)a.n,
                      (uint64_t)(a.k / 2), (uint32_t)(W4_BK / 2), (uint32_t)W4_BN, CU_TENSOR_MAP_SWIZZLE_64B))
    return cudaErrorInvalidValue;
  W4Params p;
  p.m = (int)a.m;
  p.n = (int)a.n;
  p.k = (int)a.k;
  p.nkb = (int)(a.k / W4_BK);
  p.a_scale = a.xs;
  p.s_channel = a.s_channel;
  p.bias = static_cast<const __nv_bfloat16*>(a.bias);
  p.s_rel = a.s_rel;
  p.e4m3 = a.s_rel_e4m3 ? 1 : 0;
  p.codebook = a.codebook;
  p.group = (int)a.group;
  p.gpr = (int)gpr;
  p.sx = static_cast<const __nv_bfloat16*>(a.sx);
  p.kp = (int)a.kp;
  p.corr = static_cast<const __nv_bfloat16*>(a.corr);
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.ldo = a.ldo;
  const int64_t n_tiles = (a.n + W4_BN - 1) / W4_BN, m_tiles = (a.m + W4_BM - 1) / W4_BM;
  p.splits = (int)a.splits;
  if (p.splits < 1 || p.splits > p.nkb || a.acc_ws == nullptr || a.tile_cnt == nullptr) return cudaErrorNotSupported;
  p.kb_per = (p.nkb + p.splits - 1) / p.splits;
  if ((p.nkb + p.kb_per - 1) / p.kb_per != p.splits) return cudaErrorNotSupported;  // no empty split
  p.acc_ws = a.acc_ws;
  p.tile_cnt = a.tile_cnt;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(gemm_w4_smallm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, W4_SMEM);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const dim3 grid((unsigned)n_tiles, (unsigned)m_tiles, (unsigned)p.splits);
  gemm_w4_smallm_kernel<<<grid, W4_THREADS, W4_SMEM, stream>>>(tmA, tmP, p);
  return cudaGetLastError();
}

}  // namespace h3
