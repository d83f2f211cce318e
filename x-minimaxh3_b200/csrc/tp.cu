// Tensor-parallel gated MLP over peer-mapped memory (one process per GPU, the other
// ranks' buffers mapped through CUDA IPC over NVLink). The int32 reduce-scatter of
// fc2's partial sums is fused into the GEMM itself (its epilogue stores each row into
// the owning rank's receive slot, gemm_i8.cu); this file holds the rest of the
// exchange:
//   * tp_push_u32_kernel: this rank's fc1 row absmax into its slot on every rank;
//   * tp_barrier_kernel: a cross-GPU barrier (release/acquire flags at system scope,
//     bounded wait);
//   * tp_max_u32_kernel: the global row absmax = max over the ranks' slots;
//   * tp_finish_kernel: the owner's rows: sum of the ranks' int32 partials, dequant +
//     gated residual (the fused MLP's fc2 epilogue arithmetic), rows pushed to every
//     rank's gather buffer (the all-gather, fused);
//   * tp_gather_rows_kernel: the other owners' rows from the gather buffer into out.
// Rows are owned block-cyclically (kernels.h: tp_owner / tp_local_row).
// Publication: a kernel's writes (to this GPU's or another GPU's memory) happen before
// the next kernel of the same stream; the barrier kernel that follows them issues a
// system-scope fence and a release store, so a rank that acquires the flag sees every
// write its peers made before their barrier. The data kernels themselves need no fence.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "quant_math.cuh"

namespace h3 {
namespace {

constexpr unsigned kErrTpBarrier = 0x201;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// dst.p[q][i] = src[i] for q < ndst
__global__ void tp_push_u32_kernel(const uint32_t* __restrict__ src, int64_t n, TpPtrs dst, int ndst) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t v = __ldcg(src + i);
    for (int q = 0; q < ndst; ++q) static_cast<uint32_t*>(dst.p[q])[i] = v;
  }
}

// Thread q < world stores `epoch` into this rank's flag on rank q (flag_out.p[q]),
// then waits until rank q's flag on this rank (my_flags[q]) has reached it. The wait
// is bounded (time and iterations); on expiry the kernel records kErrTpBarrier and
// returns.
__global__ void tp_barrier_kernel(TpPtrs flag_out, const uint32_t* my_flags, int world, uint32_t epoch,
                                  unsigned long long timeout_ns) {
  const int q = threadIdx.x;
  if (q >= world) return;
  __threadfence_system();
  st_release_sys(static_cast<uint32_t*>(flag_out.p[q]), epoch);
  const unsigned long long t0 = global_ns();
  const unsigned long long max_spins = timeout_ns / 16 + 1024;  // __nanosleep(32) per spin at least
  unsigned long long spins = 0;
  while ((int32_t)(ld_acquire_sys(my_flags + q) - epoch) < 0) {
    if (++spins > max_spins || ((spins & 63u) == 0u && global_ns() - t0 > timeout_ns)) {
      set_status(kErrTpBarrier);
      return;
    }
    __nanosleep(32);
  }
}

// out[i] = max over q < world of slots[q * stride + i] (fp32 absmax bit patterns: non-negative,
// so the unsigned order is the float order)
__global__ void tp_max_u32_kernel(const uint32_t* __restrict__ slots, int64_t stride, int world, int64_t n,
                                  uint32_t* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  uint32_t v = 0u;
  for (int q = 0; q < world; ++q) v = max(v, __ldcg(slots + q * stride + i));
  out[i] = v;
}

// Owner `owner`'s rows of a chunk of `rows` rows: local row lr < span (compact receive
// layout) is chunk row tp_chunk_row(lr); acc = sum over q < world of
// recv[q * slot + lr * n + c] (int32, exact); y = bf16(float(acc) * (xs * ws[c])), xs =
// row_scale(absmax[row]); out row = bf16(residual + y * gate[c]). 8 columns per thread. The
// row goes to out (this rank) and to gather.p[q] (row stride n) for every non-null q.
// WC: the world size at compile time (all loads issued before the first use), or 0.
template <int WC>
__global__ void tp_finish_kernel(const int32_t* recv, int64_t slot, int world_rt, int owner, int64_t rows, int64_t n,
                                 int64_t span, const uint32_t* __restrict__ absmax, const float* __restrict__ ws,
                                 const __nv_bfloat16* __restrict__ gate, const __nv_bfloat16* residual, int64_t ldr,
                                 __nv_bfloat16* out, int64_t ldo, TpPtrs gather) {
  const int world = WC > 0 ? WC : world_rt;
  const int64_t per_row = n / 8;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t lr = idx / per_row;
  if (lr >= span) return;
  const int64_t row = tp_chunk_row(lr, world, owner);
  if (row >= rows) return;
  const int64_t c = (idx - lr * per_row) * 8;
  const int32_t* src = recv + lr * n + c;
  int32_t av[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if constexpr (WC > 0) {
    int4 part[WC][2];
#pragma unroll
    for (int q = 0; q < WC; ++q) {
      part[q][0] = __ldcg(reinterpret_cast<const int4*>(src + q * slot));
      part[q][1] = __ldcg(reinterpret_cast<const int4*>(src + q * slot) + 1);
    }
#pragma unroll
    for (int q = 0; q < WC; ++q) {
      av[0] += part[q][0].x; av[1] += part[q][0].y; av[2] += part[q][0].z; av[3] += part[q][0].w;
      av[4] += part[q][1].x; av[5] += part[q][1].y; av[6] += part[q][1].z; av[7] += part[q][1].w;
    }
  } else {
    for (int q = 0; q < world; ++q) {
      const int4 a0 = __ldcg(reinterpret_cast<const int4*>(src + q * slot));
      const int4 a1 = __ldcg(reinterpret_cast<const int4*>(src + q * slot) + 1);
      av[0] += a0.x; av[1] += a0.y; av[2] += a0.z; av[3] += a0.w;
      av[4] += a1.x; av[5] += a1.y; av[6] += a1.z; av[7] += a1.w;
    }
  }
  const uint4 rv = ldg_v4(residual + row * ldr + c);
  const uint4 gv = ldg_nc_v4(gate + c);
  const float4 w0 = __ldg(reinterpret_cast<const float4*>(ws + c));
  const float4 w1 = __ldg(reinterpret_cast<const float4*>(ws + c + 4));
  const float x = row_scale(__uint_as_float(__ldcg(absmax + row)));
  const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
  const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float y0 = bf16_round(__fmul_rn(__int2float_rn(av[2 * e]), __fmul_rn(x, wv[2 * e])));
    const float y1 = bf16_round(__fmul_rn(__int2float_rn(av[2 * e + 1]), __fmul_rn(x, wv[2 * e + 1])));
    o[e] = pack_bf16(__fadd_rn(bf16_lo(rw[e]), __fmul_rn(y0, bf16_lo(gw[e]))),
                     __fadd_rn(bf16_hi(rw[e]), __fmul_rn(y1, bf16_hi(gw[e]))));
  }
  const uint4 ov = make_uint4(o[0], o[1], o[2], o[3]);
  stg_v4(out + row * ldo + c, ov);
#pragma unroll
  for (int q = 0; q < kTpMaxWorld; ++q)
    if (q < world && gather.p[q] != nullptr) stg_v4(static_cast<__nv_bfloat16*>(gather.p[q]) + row * n + c, ov);
}

// out[row] = gather[row] for the chunk rows that other ranks own (8 columns per thread)
__global__ void tp_gather_rows_kernel(const __nv_bfloat16* gather, int world, int owner, int64_t rows, int64_t n,
                                      __nv_bfloat16* out, int64_t ldo) {
  const int64_t per_row = n / 8;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * per_row) return;
  const int64_t row = idx / per_row;
  if (tp_owner(row, world) == owner) return;
  const int64_t c = (idx - row * per_row) * 8;
  stg_v4(out + row * ldo + c, __ldcg(reinterpret_cast<const uint4*>(gather + row * n + c)));
}

}  // namespace

cudaError_t launch_tp_push_u32(const uint32_t* src, int64_t n, const TpPtrs& dst, int ndst, cudaStream_t stream) {
  if (n <= 0 || ndst <= 0) return cudaSuccess;
  if (ndst > kTpMaxWorld) return cudaErrorNotSupported;
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 148);
  tp_push_u32_kernel<<<(unsigned)blocks, 256, 0, stream>>>(src, n, dst, ndst);
  return cudaGetLastError();
}

cudaError_t launch_tp_barrier(const TpPtrs& flag_out, const uint32_t* my_flags, int world, uint32_t epoch,
                              unsigned long long timeout_ns, cudaStream_t stream) {
  if (world <= 1) return cudaSuccess;
  if (world > kTpMaxWorld) return cudaErrorNotSupported;
  tp_barrier_kernel<<<1, 32, 0, stream>>>(flag_out, my_flags, world, epoch, timeout_ns);
  return cudaGetLastError();
}

cudaError_t launch_tp_max_u32(const uint32_t* slots, int64_t stride, int world, int64_t n, uint32_t* out,
                              cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  tp_max_u32_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(slots, stride, world, n, out);
  return cudaGetLastError();
}

cudaError_t launch_tp_finish(const int32_t* recv, int64_t slot, int world, int owner, int64_t rows, int64_t n,
                             const uint32_t* absmax, const float* ws, const void* gate, const void* residual,
                             int64_t ldr, void* out, int64_t ldo, const TpPtrs& gather, cudaStream_t stream) {
  const int64_t span = tp_owned_span(rows, world, owner);
  if (span <= 0) return cudaSuccess;
  if (n % 8 || ldr % 8 || ldo % 8 || slot % 8 || (reinterpret_cast<uintptr_t>(recv) & 15) ||
      (reinterpret_cast<uintptr_t>(residual) & 15) || (reinterpret_cast<uintptr_t>(out) & 15) ||
      (reinterpret_cast<uintptr_t>(gate) & 15) || (reinterpret_cast<uintptr_t>(ws) & 15))
    return cudaErrorNotSupported;
  for (int q = 0; q < kTpMaxWorld; ++q)
    if (reinterpret_cast<uintptr_t>(gather.p[q]) & 15) return cudaErrorNotSupported;
  const int64_t total = span * (n / 8);
  const unsigned grid = (unsigned)((total + 255) / 256);
  const auto* g = static_cast<const __nv_bfloat16*>(gate);
  const auto* r = static_cast<const __nv_bfloat16*>(residual);
  auto* o = static_cast<__nv_bfloat16*>(out);
  switch (world) {
    case 1: tp_finish_kernel<1><<<grid, 256, 0, stream>>>(recv, slot, world, owner, rows, n, span, absmax, ws, g, r, ldr, o, ldo, gather); break;
    case 2: tp_finish_kernel<2><<<grid, 256, 0, stream>>>(recv, slot, world, owner, rows, n, span, absmax, ws, g, r, ldr, o, ldo, gather); break;
    case 4: tp_finish_kernel<4><<<grid, 256, 0, stream>>>(recv, slot, world, owner, rows, n, span, absmax, ws, g, r, ldr, o, ldo, gather); break;
    case 8: tp_finish_kernel<8><<<grid, 256, 0, stream>>>(recv, slot, world, owner, rows, n, span, absmax, ws, g, r, ldr, o, ldo, gather); break;
    default: tp_finish_kernel<0><<<grid, 256, 0, stream>>>(recv, slot, world, owner, rows, n, span, absmax, ws, g, r, ldr, o, ldo, gather); break;
  }
  return cudaGetLastError();
}

cudaError_t launch_tp_gather_rows(const void* gather, int world, int owner, int64_t rows, int64_t n, void* out,
                                  int64_t ldo, cudaStream_t stream) {
  if (rows <= 0 || world <= 1) return cudaSuccess;
  if (n % 8 || ldo % 8 || (reinterpret_cast<uintptr_t>(gather) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
    return cudaErrorNotSupported;
  const int64_t total = rows * (n / 8);
  tp_gather_rows_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(gather), world, owner, rows, n, static_cast<__nv_bfloat16*>(out), ldo);
  return cudaGetLastError();
}

}  // namespace h3
