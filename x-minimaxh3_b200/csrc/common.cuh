// Shared device helpers for the sm_100a kernels: bf16 rounding, the exact
// tanh-GELU, bounded mbarrier waits, TMA loads and tcgen05 (TMEM / UMMA) PTX.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/h3b200.h"

namespace h3 {

// ---------------------------------------------------------------------------
// Device status word. 0 = healthy; the first failing wait records its code.
// Every spin-wait in this library is bounded; on timeout the kernel records a
// code here and unwinds instead of hanging the GPU. The first recorder also
// writes the code to a mapped pinned host word (g_status_host, set up per device
// by the C-ABI layer), so the host sees the failure without synchronising and
// every later entry point refuses to launch until the status is cleared.
// ---------------------------------------------------------------------------
extern __device__ unsigned int g_status;
extern __device__ unsigned int* g_status_host;

constexpr unsigned long long kWaitTimeoutNs = 2000000000ull;  // 2 s per wait

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void set_status(unsigned int code) {
  if (atomicCAS(&g_status, 0u, code) == 0u) {
    unsigned int* h = *((unsigned int* volatile*)&g_status_host);
    if (h != nullptr) {
      *((volatile unsigned int*)h) = code;
      __threadfence_system();
    }
  }
}

__device__ __forceinline__ bool status_bad() {
  return *((volatile unsigned int*)&g_status) != 0u;
}

// ---------------------------------------------------------------------------
// bf16 helpers (round to nearest even, like torch's c10::BFloat16)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}
__device__ __forceinline__ uint16_t bf16_bits(float x) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
// two floats -> bf16x2 (lo in the low half), each rounded to nearest even: one cvt
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// ---------------------------------------------------------------------------
// tanh-GELU on a bf16 input, bit-identical to the reference's CPU result.
//
// The reference (torch 2.11 ATen GeluKernel, reduced-float vector path, tanh
// from SLEEF tanhf_u10) evaluates in fp32 without fused multiply-add:
//   cube = (x*x)*x;  inner = beta*(x + kappa*cube);  r = (0.5*x)*(1 + tanh(inner))
// with tanh faithfully rounded and exactly +-1 for |inner| > 8.664339742.
// Here inner is formed with the same rounded operations. tanh comes from
// tanhf (documented max error 2 ulp); the bf16 result is accepted when the
// whole +-4 ulp band around it rounds to one bf16 value (the composition is
// monotone in tanh), otherwise tanh is recomputed in double precision and
// rounded to fp32, which is the correctly rounded value the reference sees.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float gelu_finish(float hx, float t) {
  return __fmul_rn(hx, __fadd_rn(1.0f, t));
}

__device__ __forceinline__ float gelu_tanh_exact(float x) {
  const float kBeta = 0.7978845834732056f;   // f32(sqrt(2) * 2/sqrt(pi) * 0.5)
  const float kKappa = 0.044715f;
  const float cube = __fmul_rn(__fmul_rn(x, x), x);
  const float inner = __fmul_rn(kBeta, __fadd_rn(x, __fmul_rn(kKappa, cube)));
  const float hx = __fmul_rn(0.5f, x);
  if (fabsf(inner) > 8.664339742f) {
    return gelu_finish(hx, copysignf(1.0f, inner));
  }
  const float t = tanhf(inner);
  const float d = fabsf(t) * 4.8e-7f + 1e-37f;
  const float r = gelu_finish(hx, t);
  const float ra = gelu_finish(hx, __fsub_rn(t, d));
  const float rb = gelu_finish(hx, __fadd_rn(t, d));
  if (bf16_bits(ra) == bf16_bits(rb)) return r;
  const float tc = (float)tanh((double)inner);
  return gelu_finish(hx, tc);
}

// Exact tanh-GELU of every bf16 input (index = the input's bits), filled once
// per device from gelu_tanh_exact by ensure_gelu_table() before the first
// kernel that reads it.
extern __device__ uint16_t g_gelu_bf16[65536];

__device__ __forceinline__ uint32_t gelu_bf16_bits(uint32_t xbits16) { return g_gelu_bf16[xbits16 & 0xFFFFu]; }

// ---------------------------------------------------------------------------
// SiLU on a bf16 input, bit-identical to the reference's CPU result.
//
// apply_input_act(x, "swiglu") (backends/_activations.py:40-53) evaluates
// torch.nn.functional.silu(gate) on bf16 CPU tensors as x / (1 + exp(-x)) in
// fp32 (ATen silu kernel, reduced-float path) and stores bf16. The result
// here uses the same rounded operations; exp comes from expf (documented max
// error 2 ulp) and the bf16 result is accepted when a +-4 ulp band around it
// rounds to one bf16 value (x / (1 + e) is monotone in e), otherwise exp is
// recomputed in double precision and rounded to fp32 (the correctly rounded
// value; it matches the reference on all 65,536 inputs).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float silu_exact(float x) {
  const float e = expf(-x);
  const float r = __fdiv_rn(x, __fadd_rn(1.0f, e));
  const float de = fabsf(e) * 4.8e-7f + 1e-45f;
  const float ra = __fdiv_rn(x, __fadd_rn(1.0f, __fsub_rn(e, de)));
  const float rb = __fdiv_rn(x, __fadd_rn(1.0f, __fadd_rn(e, de)));
  if (bf16_bits(ra) == bf16_bits(rb)) return r;
  const float ec = (float)exp(-(double)x);
  return __fdiv_rn(x, __fadd_rn(1.0f, ec));
}

// Exact SiLU of every bf16 input, filled once per device by ensure_act_table().
extern __device__ uint16_t g_silu_bf16[65536];

__device__ __forceinline__ uint32_t silu_bf16_bits(uint32_t xbits16) { return g_silu_bf16[xbits16 & 0xFFFFu]; }

__device__ __forceinline__ float ex2_approx(float a) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
  return r;
}
__device__ __forceinline__ float rcp_approx(float a) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
  return r;
}

// The bf16 SiLU of the table above, computed in registers where that is safe.
// For |x| in [2^-14, 8): y = x * rcp(1 + 2^(-x log2 e)) from the hardware
// exp2 / reciprocal approximations is within about 2^-20 of silu(x) (the
// rounding of x log2 e dominates), and the reference's fp32 quotient within
// about 2^-22. When y (1 - 2^-18) and y (1 + 2^-18) round to the same bf16
// value, so does the reference's result; otherwise (about 0.3% of inputs), and
// outside that range, the exact table answers. Every operation is an explicit
// rounded intrinsic, so the result does not depend on the calling context; it
// equals the table on all 65,536 inputs (checked exhaustively on the GPU).
// No shared-memory traffic: the INT8 GEMM's SwiGLU epilogue shares that pipe
// with the tensor cores' operand reads.
__device__ __forceinline__ uint32_t silu_bf16_fast(uint32_t xbits16) {
  const uint32_t hb = xbits16 & 0xFFFFu;
  if (((hb >> 7) & 0xFFu) - 113u < 17u) {  // exponent field 113..129: |x| in [2^-14, 8)
    const float x = __uint_as_float(hb << 16);
    const float t = ex2_approx(__fmul_rn(x, -1.44269504f));
    const float y = __fmul_rn(x, rcp_approx(__fadd_rn(1.0f, t)));
    const uint32_t b = bf16_bits(__fmul_rn(y, 0.999996185302734375f));  // 1 - 2^-18
    if (b == bf16_bits(__fmul_rn(y, 1.000003814697265625f))) return b;  // 1 + 2^-18
  }
  return silu_bf16_bits(hb);
}

// SwiGLU of packed bf16 pairs (gate g, up u): bf16(bf16(silu(g)) * u) per half,
// torch's silu(gate).mul_(up); a product of two bf16 values is exact in fp32,
// so it is rounded once.
__device__ __forceinline__ uint32_t swiglu_bf16x2(uint32_t g, uint32_t u) {
  const uint32_t s = silu_bf16_fast(g) | (silu_bf16_fast(g >> 16) << 16);
  return pack_bf16(__fmul_rn(bf16_lo(s), bf16_lo(u)), __fmul_rn(bf16_hi(s), bf16_hi(u)));
}

// ---------------------------------------------------------------------------
// mbarrier (shared::cta) with bounded waits
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait until the phase with the given parity has completed. Returns false (and
// records `code`) if it does not complete within the timeout or another wait in
// the grid has already failed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int code,
                                          unsigned long long timeout_ns = kWaitTimeoutNs) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const unsigned long long t0 = global_ns();
  uint32_t spins = 0;
  while (!mbar_try_wait(a, parity)) {
    if ((++spins & 255u) == 0u) {
      if (status_bad()) return false;
      if (global_ns() - t0 > timeout_ns) {
        set_status(code);
        return false;
      }
    }
  }
  return true;
}

// mbar_wait with cluster-scope acquire: for phases completed by arrivals from
// the peer CTA of a pair (release.cluster) that order the peer's TMEM accesses.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar_addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, unsigned int code,
                                                  unsigned long long timeout_ns = kWaitTimeoutNs) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait_cluster(a, parity)) return true;
  const unsigned long long t0 = global_ns();
  uint32_t spins = 0;
  while (!mbar_try_wait_cluster(a, parity)) {
    if ((++spins & 255u) == 0u) {
      if (status_bad()) return false;
      if (global_ns() - t0 > timeout_ns) {
        set_status(code);
        return false;
      }
    }
  }
  return true;
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// TMA (tiled, no multicast)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)map) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x,
                                            int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(smem_dst)),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// TMA tiled store shared -> global (bulk-group completion, clipped at the
// tensor bounds) and the bulk-group waits.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"((uint64_t)map),
               "r"(x), "r"(y), "r"(smem_u32(smem_src))
               : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* smem_src, int32_t x, int32_t y,
                                             int32_t z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"((uint64_t)map),
               "r"(x), "r"(y), "r"(z), "r"(smem_u32(smem_src))
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the shared-memory sources of every committed store have been read
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// every committed store has completed
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, UMMA issue, commit, TMEM loads
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with 128-byte swizzling: rows of 128 bytes, 8-row groups 1024 bytes apart.
// Fields: start>>4 [0,14), LBO>>4 [16,30) (unused for swizzled K-major, 1),
// SBO>>4 [32,46), version 1 at [46,48), layout SWIZZLE_128B (2) at [61,64).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// Instruction descriptor for kind::i8: s32 accumulator, signed A and B, both
// K-major, shape M x N.
__host__ __device__ constexpr uint32_t umma_idesc_i8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor for kind::f16 with bf16 A and B (both K-major) and an
// fp32 accumulator, shape M x N.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns; thread i of the warp receives lane
// (quarter*32 + i) of the accumulator.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns written back (same layout as tmem_ld32).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------------------
// CTA pairs (cluster of 2) for cta_group::2 MMAs. No multicast load anywhere:
// each CTA loads its own operand halves; completions reach the peer's
// barriers through explicit shared::cluster addresses (mapa).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of `p` (a shared::cta pointer) in the CTA of cluster rank `rank`
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// arrive (release, cluster scope) on an mbarrier given by its shared::cluster address
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}
// tiled TMA load into this CTA's shared memory for a cta_group::2 MMA; the
// completed bytes are counted on the mbarrier at `bar_cluster_addr`, which may
// belong to the peer CTA
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster_addr,
                                                 int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(smem_dst)),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(bar_cluster_addr)
      : "memory");
}
__device__ __forceinline__ void umma_i8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on the mbarrier at `bar_cluster_addr` when this thread's prior cta_group::2 tcgen05 ops complete
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster_addr)
               : "memory");
}
// collective with the peer CTA's warp of the same index (same slot offset in both CTAs)
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// 128-bit global accesses
__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
// Coherent 128-bit load, for data the same kernel may overwrite in place.
__device__ __forceinline__ uint4 ldg_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ void stg_v4(void* p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

}  // namespace h3
