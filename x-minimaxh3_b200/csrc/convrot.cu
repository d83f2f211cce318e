// ConvRot-256 rotation + per-row INT8 quantization: the activation quantizer
// of the W4A8 linears and of the ConvRot INT8 linears, with the rotation
// correctly rounded.
//
// Reference: quantize_and_rotate_rowwise (backends/eager/quantization.py:878-895)
// = _rotate_activation (tensor/int8_utils.py:58-74: x_grouped @ H per 256-group,
// H = H4^(x)4 / 16, :11-38) then quantize_int8_rowwise (:857-875); its CUDA twin
// is the ConvRot quantizer of backends/cuda/ops/int8_linear.cu:256-340 (H3:
// h3serve/native_engine/model/convrot_nvrtc.py:20-200). The reference forms the
// rotation as a bf16 matmul whose fp32 summation order depends on the CPU's BLAS
// kernel; this kernel returns the correctly rounded bf16 of the exact rotation
// (convrot_math.cuh), the value those fp32 sums approximate, so its int8 output
// is one well-defined function of the input. Input activations (tanh-GELU, or
// SwiGLU of [gate | up] rows) are applied exactly before the rotation.
//
// B200 design: a persistent CTA per SM with two teams of TW warps (6 for rows of up
// to 24 groups, 8 above: 12 or 16 warps); the teams take alternate rows. Rows stream into a shared-memory ring of one-row
// stages with cp.async.bulk (no multicast), issued by each team's first lane for
// its own rows (the ring has an even number of stages, so each stage always
// serves the same team; a stage is refilled as soon as the team's row-absmax
// barrier shows every warp has read it). A team's 2 TW half-warps split the row's
// 256-groups (GPH per half-warp). Per group, lane l of
// a half-warp reads column l of the group's 16 x 16 matrix (natural index
// 16 a + b: a = high base-4 digits, b = low) with 2-byte loads (the second
// half-warp reads rows in the order a ^ 1, which keeps the two half-warps on
// different banks; H4 commutes with that relabelling), transforms the high
// digits in doubles, exchanges the 16 x 16 doubles through a swizzled tile
// (conflict-free 8-byte writes, 16-byte reads), transforms the low digits and
// so holds outputs 16 l .. 16 l + 15: contiguous, so the int8 result is stored
// with one 16-byte store per lane and no byte transpose. The rotated bf16 pairs
// wait in registers until the team's row absmax is known (a bounded mbarrier
// wait), then are quantized like quantize_int8_rowwise and stored; the W4A8
// correction operand sx[m, g] = bf16(bf16(sum q) * bf16(scale)) is summed from
// the int8 bytes.
#include <algorithm>

#include "common.cuh"
#include "convrot_math.cuh"
#include "kernels.h"
#include "quant_math.cuh"

namespace h3 {
namespace {

// NT teams of TW warps: 2 x 6, 2 x 8 or 4 x 3 (12 or 16 warps per CTA, at most 4 per SM
// sub-partition)
constexpr int kCvMaxTeams = 4;
constexpr int kCvMaxGph = 6;  // groups per half-warp: K <= 16 * 6 * 256
constexpr int kCvMaxStages = 16;
constexpr int kCvTileBytes = 2 * 16 * cv::kXRow;  // per consumer warp: one padded double tile per half-warp
constexpr int kCvOffRed = 512;      // [team][phase][warp] row-max words, after the mbarriers
constexpr int kCvOffTiles = 1024;
constexpr int cv_off_ring(int warps) { return kCvOffTiles + warps * kCvTileBytes; }
constexpr int kCvSmemLimit = 232448;
constexpr unsigned kErrCvFull = 0x312, kErrCvTeam = 0x313, kErrCvDrain = 0x314;

__device__ __forceinline__ void cv_bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// activation applied to one bf16 input (low 16 bits): GELU from the exact table,
// SwiGLU = bf16(silu(gate) * up) (the product of two bf16 values is exact in fp32)
template <int ACT>
__device__ __forceinline__ uint32_t cv_act(uint32_t gate, uint32_t up) {
  if constexpr (ACT == H3B200_ACT_GELU_TANH) return gelu_bf16_bits(gate);
  if constexpr (ACT == H3B200_ACT_SWIGLU)
    return bf16_bits(__fmul_rn(bf16_lo(silu_bf16_fast(gate)), bf16_lo(up)));
  return gate;
}

struct Words8 {
  uint32_t w[8];
};

// running max of |bf16| over a bf16x2 pair (the sign of the result is not used)
__device__ __forceinline__ uint32_t bf16x2_absmax(uint32_t acc, uint32_t w) {
  uint32_t r;
  asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(acc), "r"(w));
  return r;
}

// Exact rotation of group g (natural order in the stage; up rows 2K bytes later for
// SwiGLU) for any inputs: lane li returns outputs 16 li .. 16 li + 15 as bf16 pairs.
// Inlined so that it is register-allocated within the kernel's limit (a separately
// compiled function would be sized at link time, outside it).
template <int ACT>
__device__ __forceinline__ Words8 cv_group_slow(const uint8_t* st, int K, int g, int li) {
  const uint8_t* grp = st + g * 512;
  auto load = [&](uint32_t i) -> uint32_t {
    const uint32_t gate = *reinterpret_cast<const uint16_t*>(grp + 2 * i);
    const uint32_t up = ACT == H3B200_ACT_SWIGLU ? *reinterpret_cast<const uint16_t*>(grp + 2 * K + 2 * i) : 0u;
    return cv_act<ACT>(gate, up);
  };
  bool nan = false;
  int fmin = 255;
  for (uint32_t i = 0; i < 256u; ++i) {
    const uint32_t a = load(i) & 0x7FFFu;
    if (a > 0x7F80u) nan = true;
    else if (a != 0u && a != 0x7F80u) fmin = min(fmin, max((int)(a >> 7), 1));
  }
  if (fmin == 255) fmin = 1;
  Words8 r;
  for (int k = 0; k < 8; ++k) {
    const uint32_t lo = cv::slow_output(load, (uint32_t)(16 * li + 2 * k), nan, fmin);
    const uint32_t hi = cv::slow_output(load, (uint32_t)(16 * li + 2 * k + 1), nan, fmin);
    r.w[k] = lo | (hi << 16);
  }
  return r;
}

template <int TW, int GPH, int ACT, int NT>
__global__ void __maxnreg__(128)
    convrot_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int64_t m, int8_t* __restrict__ q,
                   float* __restrict__ scale, __nv_bfloat16* __restrict__ sx, int sum_group, int64_t kp, int stages,
                   int ng) {
  const int K = 256 * ng;
  const int row_bytes = (ACT == H3B200_ACT_SWIGLU ? 4 : 2) * K;
  // 16-byte alignment is all this kernel needs (bulk copies, f64 pairs, mbarriers); the
  // array is used directly so the compiler keeps every access in the shared space
  extern __shared__ __align__(128) uint8_t cv_smem[];
  uint8_t* smem = cv_smem;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem);
  static_assert(NT * TW <= 16 && NT <= kCvMaxTeams, "team layout");
  uint64_t* team_bar = full_bar + kCvMaxStages;  // [NT]
  uint32_t* red = reinterpret_cast<uint32_t*>(smem + kCvOffRed);
  uint8_t* ring = smem + cv_off_ring(NT * TW);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t G = gridDim.x;
  const int64_t cnt = m > (int64_t)blockIdx.x ? (m - blockIdx.x + G - 1) / G : 0;  // rows of this CTA
  const int S = stages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&full_bar[s], 1);
    for (int t = 0; t < NT; ++t) mbar_init(&team_bar[t], TW);
    fence_barrier_init();
  }
  __syncthreads();

  const int cw = warp;
  const int team = cw / TW, tw = cw - team * TW;
  // The first lane of each team fills that team's stages: S is a multiple of NT, so stage
  // j % S always holds rows of team j % NT. Rows team, team + NT, ... below S first; then row
  // j + S as soon as the team has read row j (its row-absmax barrier completes after
  // every warp of the team has read the stage), overlapping the quantization of row j.
  const bool leader = tw == 0 && lane == 0;
  auto fill = [&](int64_t j) {
    const int s = (int)(j % S);
    mbar_arrive_expect_tx(&full_bar[s], (uint32_t)row_bytes);
    cv_bulk_g2s(ring + (size_t)s * row_bytes, x + (blockIdx.x + j * G) * ldx, (uint32_t)row_bytes, &full_bar[s]);
  };
  int64_t filled = team;  // (leader) next row of the team to fill
  if (leader)
    for (; filled < cnt && filled < S; filled += NT) fill(filled);
  const int h = lane >> 4, li = lane & 15;
  const int hw = 2 * tw + h;  // groups hw, hw + 2 TW, ...
  uint8_t* tile = smem + kCvOffTiles + cw * kCvTileBytes + h * (16 * cv::kXRow);
  uint8_t* const wr_even = tile + cv::xtile_off(h, li);         // row e ^ h for even e: e + h
  uint8_t* const wr_odd = tile + cv::xtile_off(0, li) - h * cv::kXRow;  // odd e: e - h
  const uint8_t* const rd_row = tile + cv::xtile_pair_off(li, 0);
  uint32_t* rteam = red + team * (2 * TW);
  const int lanes_per_sum = sum_group / 16;
  uint32_t team_phase = 0;
  int64_t waited = team;  // next row of the team whose fill has not been waited for
  for (int64_t j = team; j < cnt; j += NT) {
    const int s = (int)(j % S);
    const int64_t row = blockIdx.x + j * G;
    if (!mbar_wait(&full_bar[s], (uint32_t)(j / S) & 1u, kErrCvFull)) break;
    waited = j + NT;
    const uint8_t* st = ring + (size_t)s * row_bytes;
    uint32_t park[GPH][8];
    uint32_t amax = 0u;
    uint32_t slow_mask = 0u;  // groups of this half-warp that take the exact integer path
#pragma unroll
    for (int i = 0; i < GPH; ++i) {
      const int g = hw + 2 * TW * i;
      const bool ok = g < ng;  // the same for the 16 lanes of a half-warp; empty slots carry zeros
      // register e holds row e ^ h of column li: row e + h (e even) or e - h (e odd)
      const uint16_t* col_even = reinterpret_cast<const uint16_t*>(st + (ok ? g : 0) * 512 + 2 * li) + 16 * h;
      const uint16_t* col_odd = col_even - 32 * h;
      uint32_t v[16];
      float xf[16];
      // |x| statistics of this lane's 16 inputs (a bf16 is the high half of its fp32):
      // the largest and the smallest, zeros included. Both drop NaN; a NaN input makes
      // every output of its group NaN on either path, and a NaN bf16 quantizes the same
      // whatever its payload, so NaN needs no exact path.
      float fmx = 0.0f, fmn = __uint_as_float(0x7F800000u);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const uint16_t* p = (e & 1 ? col_odd : col_even) + 16 * e;
        // an empty slot reads group 0 (valid memory); its values are never used
        const uint32_t a = cv_act<ACT>(p[0], ACT == H3B200_ACT_SWIGLU ? (uint32_t)p[K] : 0u);
        v[e] = a;
        xf[e] = __uint_as_float(a << 16);
        fmx = fmaxf(fmx, fabsf(xf[e]));
        fmn = fminf(fmn, fabsf(xf[e]));
      }
      if (!ok) {  // an empty slot does not constrain the other half-warp's group
        fmx = 0.0f;
        fmn = __uint_as_float(0x7F800000u);
      }
      // One exactness test for the slot's two groups (both half-warps): the exponent
      // spread over both is at least each group's own, so passing it proves both exact.
      const uint32_t umax = __reduce_max_sync(0xffffffffu, __float_as_uint(fmx));
      uint32_t umin = __reduce_min_sync(0xffffffffu, __float_as_uint(fmn));
      uint32_t min1;
      if (umin != 0u) {
        min1 = (umin >> 16) - 1u;  // umin = 0x7F800000 (no valid input) passes through fast_path_ok's inf check
      } else {  // a zero among the inputs: the smallest nonzero magnitude, zeros wrapping to the top
        uint32_t m1 = 0xFFFFFFFFu;
#pragma unroll
        for (int e = 0; e < 16; ++e) m1 = min(m1, (v[e] & 0x7FFFu) - 1u);
        min1 = __reduce_min_sync(0xffffffffu, ok ? m1 : 0xFFFFFFFFu);
      }
      if (!cv::fast_path_ok(umax >> 16, min1)) {
        // rare: the per-group test decides which of the two groups need the exact path
        uint32_t kmax = 0u, kmin = 0xFFFFFFFFu;
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          kmax = max(kmax, v[e] & 0x7FFFu);
          kmin = min(kmin, (v[e] & 0x7FFFu) - 1u);
        }
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) {
          kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
          kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
        }
        if (ok && !cv::fast_path_ok(kmax, kmin)) slow_mask |= 1u << i;
      }
      // Fast path for both groups of the slot (a group marked slow gets its values
      // replaced below). The exchange is warp-synchronous.
      double d[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) d[e] = (double)xf[e];
#pragma unroll
      for (int a4 = 0; a4 < 4; ++a4) cv::h4<false>(d[4 * a4], d[4 * a4 + 1], d[4 * a4 + 2], d[4 * a4 + 3]);
#pragma unroll
      for (int a4 = 0; a4 < 4; ++a4) cv::h4<false>(d[a4], d[4 + a4], d[8 + a4], d[12 + a4]);
      // exchange: this lane holds column li (register e = row e ^ h); it reads back row li.
      // Row e ^ h is row e + 1 (e even) or e - 1 (e odd) in the second half-warp.
#pragma unroll
      for (int e = 0; e < 16; ++e) *reinterpret_cast<double*>((e & 1 ? wr_odd : wr_even) + e * cv::kXRow) = d[e];
      __syncwarp();
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const double2 t = *reinterpret_cast<const double2*>(rd_row + 16 * k);
        d[2 * k] = t.x;
        d[2 * k + 1] = t.y;
      }
      __syncwarp();  // the tile is rewritten for the next group
#pragma unroll
      for (int b4 = 0; b4 < 4; ++b4) cv::h4<false>(d[4 * b4], d[4 * b4 + 1], d[4 * b4 + 2], d[4 * b4 + 3]);
#pragma unroll
      for (int b4 = 0; b4 < 4; ++b4) cv::h4<true>(d[b4], d[4 + b4], d[8 + b4], d[12 + b4]);
#pragma unroll
      for (int k = 0; k < 8; ++k)
        park[i][k] = pack_bf16(cv::bits_float(cv::rto21_signed_bits(d[2 * k])),
                               cv::bits_float(cv::rto21_signed_bits(d[2 * k + 1])));
    }
    if (__any_sync(0xffffffffu, slow_mask != 0u)) {
      // Exact integer path for the marked groups, one group slot at a time for the whole
      // warp. Each lane's 16 results replace the group's inputs in the stage (its own 32
      // bytes, after every lane of the half-warp has read them) and are read back into
      // the parked registers.
#pragma unroll 1
      for (int i = 0; i < GPH; ++i) {
        const bool mine = (slow_mask >> i) & 1u;
        const int g = hw + 2 * TW * i;
        Words8 r = {{0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u}};
        if (mine) r = cv_group_slow<ACT>(st, K, g, li);
        __syncwarp();
        if (mine) {
          uint8_t* dst = const_cast<uint8_t*>(st) + g * 512 + 32 * li;
          *reinterpret_cast<uint4*>(dst) = make_uint4(r.w[0], r.w[1], r.w[2], r.w[3]);
          *reinterpret_cast<uint4*>(dst + 16) = make_uint4(r.w[4], r.w[5], r.w[6], r.w[7]);
        }
      }
      __syncwarp();
#pragma unroll
      for (int i = 0; i < GPH; ++i)
        if ((slow_mask >> i) & 1u) {
          const uint8_t* src = st + (hw + 2 * TW * i) * 512 + 32 * li;
          const uint4 a = *reinterpret_cast<const uint4*>(src), b = *reinterpret_cast<const uint4*>(src + 16);
          park[i][0] = a.x; park[i][1] = a.y; park[i][2] = a.z; park[i][3] = a.w;
          park[i][4] = b.x; park[i][5] = b.y; park[i][6] = b.z; park[i][7] = b.w;
        }
      fence_proxy_async_shared();  // generic writes to the stage before its next asynchronous fill
    }
#pragma unroll
    for (int i = 0; i < GPH; ++i)
      if (hw + 2 * TW * i < ng) {
#pragma unroll
        for (int k = 0; k < 8; ++k) amax = bf16x2_absmax(amax, park[i][k]);
      }
    // row absmax over the team (its barrier also marks every read of the stage done)
    amax &= 0x7FFF7FFFu;
    amax = max(amax & 0xFFFFu, amax >> 16);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    uint32_t* rr = rteam + (team_phase & 1u) * TW;
    if (lane == 0) {
      rr[tw] = amax;
      mbar_arrive(&team_bar[team]);
    }
    if (!mbar_wait(&team_bar[team], team_phase & 1u, kErrCvTeam)) break;
    ++team_phase;
    if (leader && j + S < cnt) {
      fill(j + S);
      filled = j + S + NT;
    }
    uint32_t rowbits = rr[0];
#pragma unroll
    for (int t = 1; t < TW; ++t) rowbits = max(rowbits, rr[t]);
    const float s_row = fmaxf(__fdiv_rn(__uint_as_float(rowbits << 16), 127.0f), 1e-30f);
    const float rcp = __frcp_rn(quant_divisor(s_row));
#pragma unroll
    for (int i = 0; i < GPH; ++i) {
      const int g = hw + 2 * TW * i;
      const bool ok = g < ng;
      const uint32_t w0[4] = {park[i][0], park[i][1], park[i][2], park[i][3]};
      const uint32_t w1[4] = {park[i][4], park[i][5], park[i][6], park[i][7]};
      const uint2 q0 = quant_vec8(make_uint4(w0[0], w0[1], w0[2], w0[3]), rcp);
      const uint2 q1 = quant_vec8(make_uint4(w1[0], w1[1], w1[2], w1[3]), rcp);
      if (ok) stg_v4(q + row * K + g * 256 + 16 * li, make_uint4(q0.x, q0.y, q1.x, q1.y));
      if (sx != nullptr) {  // all lanes shuffle; partners stay inside the half-warp (offsets < 16)
        int isum = __dp4a((int)q0.x, 0x01010101, __dp4a((int)q0.y, 0x01010101,
                          __dp4a((int)q1.x, 0x01010101, __dp4a((int)q1.y, 0x01010101, 0))));
        for (int o = 1; o < lanes_per_sum; o <<= 1) isum += __shfl_xor_sync(0xffffffffu, isum, o);
        if (ok && (li % lanes_per_sum) == 0)
          sx[row * kp + (g * 256 + 16 * li) / sum_group] =
              __float2bfloat16_rn(__fmul_rn(bf16_round((float)isum), bf16_round(s_row)));
      }
    }
    if (tw == 0) {
      if (lane == 0) scale[row] = s_row;
      if (sx != nullptr)  // zero the K padding of the correction operand
        for (int64_t i2 = K / sum_group + lane; i2 < kp; i2 += 32) sx[row * kp + i2] = __float2bfloat16_rn(0.0f);
    }
  }
  // every copy this team's leader issued lands before the CTA may exit (rows left
  // unconsumed only after a bounded wait failed)
  if (leader)
    for (int64_t i = waited; i < filled; i += NT)
      mbar_wait(&full_bar[i % S], (uint32_t)(i / S) & 1u, kErrCvDrain, 200000000ull);
}

template <int TW, int GPH, int NT = 2>
cudaError_t cv_launch(int act, const __nv_bfloat16* x, int64_t ldx, int64_t m, int8_t* q, float* scale,
                      __nv_bfloat16* sx, int sum_group, int64_t kp, int stages, int ng, int smem, unsigned grid,
                      cudaStream_t stream) {
  constexpr int threads = 32 * NT * TW;
  auto go = [&](auto kern) -> cudaError_t {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kCvSmemLimit);
    if (e != cudaSuccess) return e;
    cudaFuncAttributes fa;
    if ((e = cudaFuncGetAttributes(&fa, kern)) != cudaSuccess) return e;
    // 16 warps put 4 on each SM sub-partition (a quarter of the register file), hence
    // the 128-register limit on the kernel
    if (fa.maxThreadsPerBlock < threads) return cudaErrorLaunchOutOfResources;
    kern<<<grid, threads, smem, stream>>>(x, ldx, m, q, scale, sx, sum_group, kp, stages, ng);
    return cudaGetLastError();
  };
  if (act == H3B200_ACT_GELU_TANH) return go(convrot_kernel<TW, GPH, H3B200_ACT_GELU_TANH, NT>);
  if (act == H3B200_ACT_SWIGLU) return go(convrot_kernel<TW, GPH, H3B200_ACT_SWIGLU, NT>);
  return go(convrot_kernel<TW, GPH, H3B200_ACT_NONE, NT>);
}

// Team layout for a row of ng groups: rows of up to 24 groups go to four 3-warp teams
// (each row's work per team pass is short, so more rows in flight per CTA hide the
// per-row barrier and copy latency: 32,760 x 3,072 216 -> 157 us, x 5,376 320 -> 293 us
// against two 6-warp teams); longer rows use two 8-warp teams (16 warps).
// (Four teams need at least two row stages each in shared memory, or a team would wait for
// every row's copy; launch_quantize_convrot falls back to two teams otherwise.)
int cv_team_warps(int64_t ng, bool four) { return four ? 3 : ng <= 24 ? 6 : 8; }

}  // namespace

int64_t convrot_max_k(int act) {
  // rows of at most 16 half-warps x 6 groups, and at least two stages of the raw row in shared memory
  const int64_t by_regs = (int64_t)2 * 8 * kCvMaxGph * 256;
  const int64_t per_elem = act == H3B200_ACT_SWIGLU ? 4 : 2;
  const int64_t by_smem = ((kCvSmemLimit - 1024 - cv_off_ring(16)) / 2 / per_elem) / 256 * 256;
  return std::min(by_regs, by_smem);
}

cudaError_t launch_quantize_convrot(const void* x, int64_t ldx, int64_t m, int64_t k, int act, int8_t* q,
                                    float* scale, void* sx, int64_t sum_group, int64_t kp, cudaStream_t stream) {
  if (m == 0) return cudaSuccess;
  if (k <= 0 || k % 256 || ldx % 8 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(q) & 15))
    return cudaErrorNotSupported;
  if (k > convrot_max_k(act)) return cudaErrorNotSupported;
  if (sx != nullptr && (sum_group < 16 || sum_group > 256 || 256 % sum_group || kp < k / sum_group))
    return cudaErrorNotSupported;
  {
    const cudaError_t e = ensure_act_table(act, stream);
    if (e != cudaSuccess) return e;
  }
  const int ng = (int)(k / 256);
  const int64_t row_bytes = (act == H3B200_ACT_SWIGLU ? 4 : 2) * k;
  auto stages_for = [&](int warps, int teams) {
    const int st = (int)std::min<int64_t>(kCvMaxStages, (kCvSmemLimit - 1024 - cv_off_ring(warps)) / row_bytes);
    return st - st % teams;  // a multiple of the team count: each stage serves one team
  };
  const bool four = ng <= 24 && stages_for(12, 4) >= 8;
  const int tw = cv_team_warps(ng, four), nt = four ? 4 : 2;
  const int gph = (ng + 2 * tw - 1) / (2 * tw);
  const int stages = stages_for(nt * tw, nt);
  if (stages < nt) return cudaErrorNotSupported;
  const int smem = 1024 + cv_off_ring(nt * tw) + stages * (int)row_bytes;
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned grid = (unsigned)std::min<int64_t>(m, (int64_t)num_sms(dev));
  const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
  __nv_bfloat16* sxb = static_cast<__nv_bfloat16*>(sx);
  const int sg = sx != nullptr ? (int)sum_group : 16;
  if (tw == 3) {
    switch (gph) {
      case 1: return cv_launch<3, 1, 4>(act, xb, ldx, m, q, scale, sxb, sg, kp, stages, ng, smem, grid, stream);
      case 2: return cv_launch<3, 2, 4>(act, xb, ldx, m, q, scale, sxb, sg, kp, stages, ng, smem, grid, stream);
      case 3: return cv_launch<3, 3, 4>(act, xb, ldx, m, q, scale, sxb, sg, kp, stages, ng, smem, grid, stream);
      default: return cv_launch<3, 4, 4>(act, xb, ldx, m, q, scale, sxb, sg, kp, stages, ng, smem, grid, stream);
    }
  }
  if (tw == 6) {
    if (gph == 1) return cv_launch<6, 1>(act, xb, ldx, m, q, scale, sxb, sg, kp, stages, ng, smem, grid, stream);
    return cv_launch<6, 2>(act, xb, ldx, m, q, scale, sxb, sg, kp, stages, ng, smem, grid, stream);
  }
  switch (gph) {
    case 2: return cv_launch<8, 2>(act, xb, ldx, m, q, scale, sxb, sg, kp, stages, ng, smem, grid, stream);
    case 3: return cv_launch<8, 3>(act, xb, ldx, m, q, scale, sxb, sg, kp, stages, ng, smem, grid, stream);
    case 4: return cv_launch<8, 4>(act, xb, ldx, m, q, scale, sxb, sg, kp, stages, ng, smem, grid, stream);
    case 5: return cv_launch<8, 5>(act, xb, ldx, m, q, scale, sxb, sg, kp, stages, ng, smem, grid, stream);
    default: return cv_launch<8, 6>(act, xb, ldx, m, q, scale, sxb, sg, kp, stages, ng, smem, grid, stream);
  }
}

}  // namespace h3
