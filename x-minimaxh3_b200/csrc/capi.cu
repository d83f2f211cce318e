// extern "C" entry points: argument validation, workspace carving, launches.
// Errors are returned as status codes with a thread-local message; nothing
// falls back to another implementation.
#include <stdarg.h>
#include <stdio.h>

#include <string.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace {

thread_local std::string t_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int from_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return H3B200_OK;
  if (e == cudaErrorNotSupported) return fail(H3B200_ERR_UNSUPPORTED, "%s: shape, stride or alignment outside the kernel contract", what);
  return fail(H3B200_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
}

inline cudaStream_t S(h3b200_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }


inline int64_t round_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

// Carves consecutive 256-byte aligned regions out of a caller workspace.
struct Carver {
  uint8_t* base;
  int64_t size;
  int64_t off = 0;
  bool ok = true;
  void* take(int64_t bytes) {
    off = round_up(off, 256);
    void* p = base + off;
    off += bytes;
    if (off > size) ok = false;
    return p;
  }
};

// ---------------------------------------------------------------------------
// Host mirror of the device status word. A kernel whose bounded wait expires
// records a code in g_status (device memory) and, through g_status_host, in one
// word of mapped pinned host memory per device. Every launching entry point
// reads that word first (no synchronisation) and refuses with
// H3B200_ERR_DEVICE while it is set: outputs of kernels that ran after the
// failure are not valid, and they must not be mistaken for results. The mirror
// is set up by the first call on each device that is not under stream capture
// (it writes a device symbol); h3b200_device_status(.., clear = 1) resets both.
// ---------------------------------------------------------------------------
constexpr int kMaxDevices = 64;
std::mutex g_mirror_mu;
unsigned int* g_mirror = nullptr;  // kMaxDevices words, cudaHostAllocMapped | Portable
std::atomic<bool> g_mirror_ready[kMaxDevices];

void status_mirror_setup(int dev, cudaStream_t stream) {
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) return;
  std::lock_guard<std::mutex> lock(g_mirror_mu);
  if (g_mirror_ready[dev].load(std::memory_order_acquire)) return;
  if (g_mirror == nullptr) {
    void* p = nullptr;
    if (cudaHostAlloc(&p, kMaxDevices * sizeof(unsigned int), cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
      cudaGetLastError();
      return;  // no mirror: failures still show in h3b200_device_status
    }
    memset(p, 0, kMaxDevices * sizeof(unsigned int));
    g_mirror = static_cast<unsigned int*>(p);
  }
  void* dptr = nullptr;
  if (cudaHostGetDevicePointer(&dptr, g_mirror + dev, 0) != cudaSuccess ||
      cudaMemcpyToSymbol(h3::g_status_host, &dptr, sizeof(dptr)) != cudaSuccess) {
    cudaGetLastError();
    return;
  }
  g_mirror_ready[dev].store(true, std::memory_order_release);
}

unsigned int status_mirror_read(int dev) {
  if (g_mirror == nullptr || !g_mirror_ready[dev].load(std::memory_order_acquire)) return 0u;
  return *reinterpret_cast<volatile unsigned int*>(g_mirror + dev);
}

// First statement of every launching entry point.
int status_guard(const char* what, h3b200_stream_t stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return H3B200_OK;  // the launch itself reports the device error
  }
  if (!g_mirror_ready[dev].load(std::memory_order_acquire)) status_mirror_setup(dev, reinterpret_cast<cudaStream_t>(stream));
  const unsigned int code = status_mirror_read(dev);
  if (code != 0u)
    return fail(H3B200_ERR_DEVICE,
                "%s: refused: a bounded device wait on device %d expired earlier (status 0x%x); outputs of calls "
                "since then are not valid; read and clear it with h3b200_device_status(device, &status, 1)",
                what, dev, code);
  return H3B200_OK;
}

#define H3_GUARD(what, stream)                                        \
  do {                                                                \
    if (const int rc_ = status_guard(what, stream)) return rc_;       \
  } while (0)

// Test-only: one thread waits on a shared-memory mbarrier that nothing arrives
// at, with the given limit, so that the bounded wait expires and the kernel
// records kErrSelftest and returns. No copy or MMA is in flight.
constexpr unsigned kErrSelftest = 0x7E57u;
__global__ void selftest_expire_kernel(unsigned long long timeout_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  h3::mbar_init(&bar, 1);
  h3::fence_barrier_init();
  h3::mbar_wait(&bar, 0u, kErrSelftest, timeout_ns);
}

}  // namespace

// Raw input columns per activated column: 2 for SwiGLU ([gate | up] rows), else 1.
static int64_t act_width(int act) { return act == H3B200_ACT_SWIGLU ? 2 : 1; }

extern "C" {

const char* h3b200_version(void) { return "h3b200 0.1.0 (sm_100a)"; }

const char* h3b200_last_error(void) { return t_last_error.c_str(); }

int h3b200_device_status(int device, unsigned int* status, int clear) {
  if (status == nullptr) return fail(H3B200_ERR_INVALID, "device_status: status is NULL");
  int prev = 0;
  cudaGetDevice(&prev);
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(status, h3::g_status, sizeof(unsigned int));
  if (e == cudaSuccess && clear) {
    unsigned int zero = 0;
    e = cudaMemcpyToSymbol(h3::g_status, &zero, sizeof(unsigned int));
    if (e == cudaSuccess && device >= 0 && device < kMaxDevices && g_mirror != nullptr)
      *reinterpret_cast<volatile unsigned int*>(g_mirror + device) = 0u;
  }
  cudaSetDevice(prev);
  return from_cuda(e, "device_status");
}

int h3b200_device_status_nowait(int device, unsigned int* status) {
  if (status == nullptr) return fail(H3B200_ERR_INVALID, "device_status_nowait: status is NULL");
  if (device < 0 || device >= kMaxDevices) return fail(H3B200_ERR_INVALID, "device_status_nowait: bad device %d", device);
  *status = status_mirror_read(device);
  return H3B200_OK;
}

int h3b200_selftest_expire_wait(int64_t timeout_ns, h3b200_stream_t stream) {
  H3_GUARD("selftest_expire_wait", stream);
  if (timeout_ns < 1000 || timeout_ns > 1000000000) return fail(H3B200_ERR_INVALID, "selftest_expire_wait: timeout must be within [1 us, 1 s]");
  selftest_expire_kernel<<<1, 32, 0, S(stream)>>>((unsigned long long)timeout_ns);
  return from_cuda(cudaGetLastError(), "selftest_expire_wait");
}

int h3b200_apply_input_act(const void* x, void* y, int64_t n, int act, h3b200_stream_t stream) {
  H3_GUARD("apply_input_act", stream);
  if (n < 0) return fail(H3B200_ERR_INVALID, "apply_input_act: negative size");
  if (act == H3B200_ACT_SWIGLU) return fail(H3B200_ERR_INVALID, "apply_input_act: swiglu halves each row; use h3b200_swiglu");
  if (act != H3B200_ACT_NONE && act != H3B200_ACT_GELU_TANH) return fail(H3B200_ERR_INVALID, "apply_input_act: unsupported act code %d", act);
  if (n > 0 && (x == nullptr || y == nullptr)) return fail(H3B200_ERR_INVALID, "apply_input_act: NULL pointer");
  if (n > (1ll << 40)) return fail(H3B200_ERR_UNSUPPORTED, "apply_input_act: n too large");
  return from_cuda(h3::launch_apply_act(x, y, n, act, S(stream)), "apply_input_act");
}

int h3b200_swiglu(const void* x, int64_t ldx, void* y, int64_t ldy, int64_t m, int64_t k, h3b200_stream_t stream) {
  H3_GUARD("swiglu", stream);
  if (m < 0 || k < 0 || ldx < 2 * k || ldy < k) return fail(H3B200_ERR_INVALID, "swiglu: bad shape m=%lld k=%lld ldx=%lld ldy=%lld (ldx >= 2k, ldy >= k)", (long long)m, (long long)k, (long long)ldx, (long long)ldy);
  if (m == 0 || k == 0) return H3B200_OK;
  if (x == nullptr || y == nullptr) return fail(H3B200_ERR_INVALID, "swiglu: NULL pointer");
  if (m * k > (1ll << 40)) return fail(H3B200_ERR_UNSUPPORTED, "swiglu: too large");
  return from_cuda(h3::launch_swiglu_rows(x, ldx, y, ldy, m, k, S(stream)), "swiglu");
}

int h3b200_quantize_int8_rowwise(const void* x, int64_t m, int64_t k, int64_t ldx, int act, int8_t* q, float* scale,
                                 h3b200_stream_t stream) {
  H3_GUARD("quantize_int8_rowwise", stream);
  if (act != H3B200_ACT_NONE && act != H3B200_ACT_GELU_TANH && act != H3B200_ACT_SWIGLU) return fail(H3B200_ERR_INVALID, "quantize_int8_rowwise: unsupported act code %d", act);
  if (m < 0 || k < 0 || ldx < k * act_width(act)) return fail(H3B200_ERR_INVALID, "quantize_int8_rowwise: bad shape m=%lld k=%lld ldx=%lld (act %d reads %lld columns)", (long long)m, (long long)k, (long long)ldx, act, (long long)(k * act_width(act)));
  if (m > 0 && (x == nullptr || q == nullptr || scale == nullptr)) return fail(H3B200_ERR_INVALID, "quantize_int8_rowwise: NULL pointer");
  if (m > 0x7fffffffll) return fail(H3B200_ERR_UNSUPPORTED, "quantize_int8_rowwise: m too large");
  return from_cuda(h3::launch_quantize_rows(x, ldx, m, k, act, nullptr, q, scale, S(stream)), "quantize_int8_rowwise");
}

int h3b200_quantize_int8_rowwise_f16(const void* x, int64_t m, int64_t k, int64_t ldx, int8_t* q, float* scale,
                                     h3b200_stream_t stream) {
  H3_GUARD("quantize_int8_rowwise_f16", stream);
  if (m < 0 || k < 0 || ldx < k) return fail(H3B200_ERR_INVALID, "quantize_int8_rowwise_f16: bad shape m=%lld k=%lld ldx=%lld", (long long)m, (long long)k, (long long)ldx);
  if (m > 0 && (x == nullptr || q == nullptr || scale == nullptr)) return fail(H3B200_ERR_INVALID, "quantize_int8_rowwise_f16: NULL pointer");
  if (m > 0x7fffffffll) return fail(H3B200_ERR_UNSUPPORTED, "quantize_int8_rowwise_f16: m too large");
  return from_cuda(h3::launch_quantize_rows_f16(x, ldx, m, k, q, scale, S(stream)), "quantize_int8_rowwise_f16");
}

int h3b200_quantize_int8_rowwise_stochastic(const void* x, int64_t m, int64_t k, int64_t ldx, int act,
                                            int64_t seed, int8_t* q, float* scale, h3b200_stream_t stream) {
  H3_GUARD("quantize_int8_rowwise_stochastic", stream);
  if (seed <= 0) return fail(H3B200_ERR_INVALID, "quantize_int8_rowwise_stochastic: seed must be > 0 (got %lld)", (long long)seed);
  if (act != H3B200_ACT_NONE && act != H3B200_ACT_GELU_TANH && act != H3B200_ACT_SWIGLU) return fail(H3B200_ERR_INVALID, "quantize_int8_rowwise_stochastic: unsupported act code %d", act);
  if (m < 0 || k < 0 || ldx < k * act_width(act)) return fail(H3B200_ERR_INVALID, "quantize_int8_rowwise_stochastic: bad shape");
  if (m > 0 && (x == nullptr || q == nullptr || scale == nullptr)) return fail(H3B200_ERR_INVALID, "quantize_int8_rowwise_stochastic: NULL pointer");
  if (m > 0x7fffffffll) return fail(H3B200_ERR_UNSUPPORTED, "quantize_int8_rowwise_stochastic: m too large");
  return from_cuda(h3::launch_quantize_rows_stochastic(x, ldx, m, k, act, (uint64_t)seed, q, scale, S(stream)), "quantize_int8_rowwise_stochastic");
}

int h3b200_quantize_int8_rowwise_absmax(const void* x, const float* absmax, int64_t m, int64_t k, int64_t ldx,
                                        int8_t* q, float* scale, h3b200_stream_t stream) {
  H3_GUARD("quantize_int8_rowwise_absmax", stream);
  if (m < 0 || k < 0 || ldx < k) return fail(H3B200_ERR_INVALID, "quantize_int8_rowwise_absmax: bad shape");
  if (m > 0 && (x == nullptr || q == nullptr || scale == nullptr || absmax == nullptr)) return fail(H3B200_ERR_INVALID, "quantize_int8_rowwise_absmax: NULL pointer");
  if (m > 0x7fffffffll) return fail(H3B200_ERR_UNSUPPORTED, "quantize_int8_rowwise_absmax: m too large");
  return from_cuda(h3::launch_quantize_rows(x, ldx, m, k, H3B200_ACT_NONE, absmax, q, scale, S(stream)), "quantize_int8_rowwise_absmax");
}

int h3b200_int8_mm(const int8_t* a, const int8_t* w, int64_t m, int64_t n, int64_t k, int32_t* out,
                   h3b200_stream_t stream) {
  H3_GUARD("int8_mm", stream);
  if (m < 0 || n < 0 || k < 0) return fail(H3B200_ERR_INVALID, "int8_mm: negative shape");
  if (m == 0 || n == 0) return H3B200_OK;
  if (a == nullptr || w == nullptr || out == nullptr) return fail(H3B200_ERR_INVALID, "int8_mm: NULL pointer");
  if (k % 16 || n % 8) return fail(H3B200_ERR_UNSUPPORTED, "int8_mm: needs k %% 16 == 0 and n %% 8 == 0 (k=%lld n=%lld)", (long long)k, (long long)n);
  h3::GemmArgs g;
  g.a = a; g.w = w; g.m = m; g.n = n; g.k = k; g.lda = k; g.ldw = k;
  g.epilogue = h3::kEpiI32; g.out = out; g.ldo = n;
  return from_cuda(h3::launch_gemm_i8(g, S(stream)), "int8_mm");
}

int h3b200_int8_linear_prequantized(const int8_t* xq, const float* x_scale, const int8_t* w, const float* w_scale,
                                    int64_t w_scale_numel, const void* bias, int out_dtype, void* out, int64_t m,
                                    int64_t n, int64_t k, h3b200_stream_t stream) {
  H3_GUARD("int8_linear_prequantized", stream);
  if (m < 0 || n < 0 || k < 0) return fail(H3B200_ERR_INVALID, "int8_linear_prequantized: negative shape");
  if (out_dtype != H3B200_DTYPE_BF16 && out_dtype != H3B200_DTYPE_F16) return fail(H3B200_ERR_UNSUPPORTED, "int8_linear_prequantized: bf16 or fp16 output (got code %d)", out_dtype);
  if (w_scale_numel != 1 && w_scale_numel != n) return fail(H3B200_ERR_INVALID, "int8_linear_prequantized: weight scale must be scalar or per-output-channel, got %lld for n=%lld", (long long)w_scale_numel, (long long)n);
  if (m == 0 || n == 0) return H3B200_OK;
  if (!xq || !x_scale || !w || !w_scale || !out) return fail(H3B200_ERR_INVALID, "int8_linear_prequantized: NULL pointer");
  if (k % 16 || n % 8) return fail(H3B200_ERR_UNSUPPORTED, "int8_linear_prequantized: needs k %% 16 == 0 and n %% 8 == 0");
  h3::GemmArgs g;
  g.a = xq; g.w = w; g.m = m; g.n = n; g.k = k; g.lda = k; g.ldw = k;
  g.epilogue = h3::kEpiBF16; g.a_scale = x_scale; g.w_scale = w_scale; g.w_scale_per_channel = w_scale_numel == n && n != 1 ? 1 : 0;
  if (w_scale_numel == n && n == 1) g.w_scale_per_channel = 0;
  g.bias = bias; g.out = out; g.ldo = n;
  g.out_f16 = out_dtype == H3B200_DTYPE_F16 ? 1 : 0;
  return from_cuda(h3::launch_gemm_i8(g, S(stream)), "int8_linear_prequantized");
}

int h3b200_int8_gemm_fused(const int8_t* a, int64_t lda, const int8_t* w, int64_t ldw, int64_t m, int64_t n,
                           int64_t k, int epilogue, const float* a_scale, const float* w_scale,
                           int64_t w_scale_numel, const void* bias, const void* gate, const void* residual,
                           int64_t ldr, void* out, int64_t ldo, float* row_absmax, h3b200_stream_t stream) {
  H3_GUARD("int8_gemm_fused", stream);
  if (m < 0 || n < 0 || k < 0 || lda < k || ldw < k || ldo < n) return fail(H3B200_ERR_INVALID, "int8_gemm_fused: bad shape");
  if (epilogue < h3::kEpiI32 || epilogue > h3::kEpiGatedResidual) return fail(H3B200_ERR_INVALID, "int8_gemm_fused: unknown epilogue %d", epilogue);
  if (m == 0 || n == 0) return H3B200_OK;
  if (!a || !w || !out) return fail(H3B200_ERR_INVALID, "int8_gemm_fused: NULL pointer");
  if (epilogue != h3::kEpiI32) {
    if (!a_scale || !w_scale) return fail(H3B200_ERR_INVALID, "int8_gemm_fused: scales required");
    if (w_scale_numel != 1 && w_scale_numel != n) return fail(H3B200_ERR_INVALID, "int8_gemm_fused: weight scale must be scalar or per-output-channel");
  }
  if (epilogue == h3::kEpiGeluAbsmax && !row_absmax) return fail(H3B200_ERR_INVALID, "int8_gemm_fused: row_absmax required");
  if (epilogue == h3::kEpiGatedResidual && (!gate || !residual || ldr < n)) return fail(H3B200_ERR_INVALID, "int8_gemm_fused: gate and residual required");
  h3::GemmArgs g;
  g.a = a; g.w = w; g.m = m; g.n = n; g.k = k; g.lda = lda; g.ldw = ldw;
  g.epilogue = epilogue; g.a_scale = a_scale; g.w_scale = w_scale; g.w_scale_per_channel = (w_scale_numel == n && n > 1) ? 1 : 0;
  g.bias = bias; g.gate = gate; g.residual = residual; g.ldr = ldr; g.out = out; g.ldo = ldo; g.row_absmax = row_absmax;
  return from_cuda(h3::launch_gemm_i8(g, S(stream)), "int8_gemm_fused");
}

int64_t h3b200_requant_gemm_workspace_bytes(int64_t m, int64_t k) {
  return round_up(m * k, 256) + round_up(h3::requant_ready_count(m) * 4, 256) + 256;
}

int h3b200_requant_gemm_gated_residual(const void* h, int64_t ldh, const float* h_absmax, const int8_t* w,
                                       const float* w_scale, int64_t w_scale_numel, const void* bias,
                                       const void* gate, int64_t ldg, const int32_t* row_map, const void* residual,
                                       int64_t ldr, void* out, int64_t ldo, int64_t m, int64_t n, int64_t k,
                                       void* workspace, int64_t workspace_bytes, h3b200_stream_t stream) {
  H3_GUARD("requant_gemm_gated_residual", stream);
  if (m < 0 || n < 0 || k < 0 || ldh < k || ldr < n || ldo < n) return fail(H3B200_ERR_INVALID, "requant_gemm_gated_residual: bad shape");
  if (w_scale_numel != 1 && w_scale_numel != n) return fail(H3B200_ERR_INVALID, "requant_gemm_gated_residual: weight scale must be scalar or per-output-channel");
  if (m == 0 || n == 0) return H3B200_OK;
  if (!h || !h_absmax || !w || !w_scale || !gate || !residual || !out) return fail(H3B200_ERR_INVALID, "requant_gemm_gated_residual: NULL pointer");
  if (row_map != nullptr && (ldg < n || ldg % 8)) return fail(H3B200_ERR_INVALID, "requant_gemm_gated_residual: gate row stride %lld must be >= n and a multiple of 8", (long long)ldg);
  if (k % 16 || n % 8 || ldh % 8) return fail(H3B200_ERR_UNSUPPORTED, "requant_gemm_gated_residual: needs k %% 16 == 0, n %% 8 == 0 and ldh %% 8 == 0");
  if (workspace == nullptr || workspace_bytes < h3b200_requant_gemm_workspace_bytes(m, k)) return fail(H3B200_ERR_INVALID, "requant_gemm_gated_residual: workspace too small (need %lld bytes)", (long long)h3b200_requant_gemm_workspace_bytes(m, k));
  Carver c{static_cast<uint8_t*>(workspace), workspace_bytes};
  int8_t* q = static_cast<int8_t*>(c.take(m * k));
  unsigned int* ready = static_cast<unsigned int*>(c.take(h3::requant_ready_count(m) * 4));
  if (!c.ok) return fail(H3B200_ERR_INVALID, "requant_gemm_gated_residual: workspace too small");
  cudaStream_t st = S(stream);
  cudaError_t e = cudaMemsetAsync(ready, 0, (size_t)(h3::requant_ready_count(m) * 4), st);
  if (e != cudaSuccess) return from_cuda(e, "requant_gemm_gated_residual: memset");
  h3::GemmArgs g;
  g.a = q; g.w = w; g.m = m; g.n = n; g.k = k; g.lda = k; g.ldw = k;
  g.epilogue = h3::kEpiGatedResidual; g.w_scale = w_scale; g.w_scale_per_channel = (w_scale_numel == n && n > 1) ? 1 : 0;
  g.requant_src = h; g.requant_lds = ldh; g.requant_ready = ready; g.row_absmax = const_cast<float*>(h_absmax);
  g.bias = bias; g.gate = gate; g.row_map = row_map; g.ldg = row_map != nullptr ? ldg : 0;
  g.residual = residual; g.ldr = ldr; g.out = out; g.ldo = ldo;
  return from_cuda(h3::launch_gemm_i8(g, st), "requant_gemm_gated_residual");
}

int h3b200_dequant_gated_residual(const int32_t* acc, const float* x_scale, const float* w_scale, const void* gate,
                                  const void* residual, int64_t ldr, void* out, int64_t ldo, int64_t m, int64_t n,
                                  h3b200_stream_t stream) {
  H3_GUARD("dequant_gated_residual", stream);
  if (m < 0 || n < 0 || ldr < n || ldo < n) return fail(H3B200_ERR_INVALID, "dequant_gated_residual: bad shape");
  if (m == 0 || n == 0) return H3B200_OK;
  if (!acc || !x_scale || !w_scale || !gate || !residual || !out) return fail(H3B200_ERR_INVALID, "dequant_gated_residual: NULL pointer");
  return from_cuda(h3::launch_dequant_gated_residual(acc, x_scale, w_scale, gate, residual, ldr, out, ldo, m, n, S(stream)), "dequant_gated_residual");
}

int64_t h3b200_int8_linear_workspace_bytes(int64_t m, int64_t k) {
  return round_up(m * k, 256) + round_up(m * 4, 256) + 512;
}

int h3b200_int8_linear(const void* x, int64_t ldx, const int8_t* w, const float* w_scale, int64_t w_scale_numel,
                       const void* bias, int act, void* out, int64_t m, int64_t n, int64_t k, void* workspace,
                       int64_t workspace_bytes, h3b200_stream_t stream) {
  H3_GUARD("int8_linear", stream);
  if (m < 0 || n < 0 || k < 0 || ldx < k * act_width(act)) return fail(H3B200_ERR_INVALID, "int8_linear: bad shape");
  if (m == 0 || n == 0) return H3B200_OK;
  if (workspace == nullptr || workspace_bytes < h3b200_int8_linear_workspace_bytes(m, k)) return fail(H3B200_ERR_INVALID, "int8_linear: workspace too small (need %lld bytes)", (long long)h3b200_int8_linear_workspace_bytes(m, k));
  Carver c{static_cast<uint8_t*>(workspace), workspace_bytes};
  int8_t* xq = static_cast<int8_t*>(c.take(m * k));
  float* xs = static_cast<float*>(c.take(m * 4));
  if (!c.ok) return fail(H3B200_ERR_INVALID, "int8_linear: workspace too small");
  int st = h3b200_quantize_int8_rowwise(x, m, k, ldx, act, xq, xs, stream);
  if (st != H3B200_OK) return st;
  return h3b200_int8_linear_prequantized(xq, xs, w, w_scale, w_scale_numel, bias, H3B200_DTYPE_BF16, out, m, n, k, stream);
}

int64_t h3b200_fused_gated_mlp_workspace_bytes(int64_t m, int64_t d, int64_t ffn) {
  return round_up(m * d, 256) + round_up(m * 4, 256) * 3 + round_up(m * ffn * 2, 256) + round_up(m * ffn, 256) + 1024;
}

}  // extern "C"

// The W8A8 MLP of h3b200_fused_gated_mlp(_segmented): gate is one row [d] (row_map
// nullptr) or rows at stride ldg selected per token by row_map.
static int fused_gated_mlp_impl(const char* what, const void* x, int64_t ldx, const int8_t* w1, const float* s1,
                                const int8_t* w2, const float* s2, const void* gate, int64_t ldg,
                                const int32_t* row_map, const void* residual, int64_t ldr, void* out, int64_t ldo,
                                int64_t m, int64_t d, int64_t ffn, int act, void* workspace, int64_t workspace_bytes,
                                h3b200_stream_t stream) {
  if (m < 0 || d <= 0 || ffn <= 0 || ldx < d || ldr < d || ldo < d) return fail(H3B200_ERR_INVALID, "%s: bad shape m=%lld d=%lld ffn=%lld", what, (long long)m, (long long)d, (long long)ffn);
  if (act != H3B200_ACT_GELU_TANH) return fail(H3B200_ERR_UNSUPPORTED, "%s: only act=gelu_tanh (1) is built, got %d", what, act);
  if (row_map != nullptr && (ldg < d || ldg % 8)) return fail(H3B200_ERR_INVALID, "%s: gate row stride %lld must be >= d and a multiple of 8", what, (long long)ldg);
  if (m == 0) return H3B200_OK;
  if (!x || !w1 || !s1 || !w2 || !s2 || !gate || !residual || !out) return fail(H3B200_ERR_INVALID, "%s: NULL pointer", what);
  if (d % 16 || ffn % 16) return fail(H3B200_ERR_UNSUPPORTED, "%s: needs d %% 16 == 0 and ffn %% 16 == 0", what);
  if (workspace == nullptr || workspace_bytes < h3b200_fused_gated_mlp_workspace_bytes(m, d, ffn)) return fail(H3B200_ERR_INVALID, "%s: workspace too small (need %lld bytes)", what, (long long)h3b200_fused_gated_mlp_workspace_bytes(m, d, ffn));
  Carver c{static_cast<uint8_t*>(workspace), workspace_bytes};
  int8_t* xq = static_cast<int8_t*>(c.take(m * d));
  float* xs = static_cast<float*>(c.take(m * 4));
  float* amax = static_cast<float*>(c.take(m * 4));
  // the fc2 kernel requantizes fc1's output itself; this slot holds its block counters
  unsigned int* ready = static_cast<unsigned int*>(c.take(m * 4));
  void* a = c.take(m * ffn * 2);
  int8_t* q2 = static_cast<int8_t*>(c.take(m * ffn));
  if (!c.ok) return fail(H3B200_ERR_INVALID, "%s: workspace too small", what);
  cudaStream_t st = S(stream);
  cudaError_t e = h3::launch_quantize_rows(x, ldx, m, d, H3B200_ACT_NONE, nullptr, xq, xs, st);
  if (e != cudaSuccess) return from_cuda(e, "fused_gated_mlp: quantize x");
  // one memset zeroes the row absmax and the counters that follow it
  const int64_t zero_bytes = reinterpret_cast<uint8_t*>(ready + h3::requant_ready_count(m)) -
                             reinterpret_cast<uint8_t*>(amax);
  e = cudaMemsetAsync(amax, 0, (size_t)zero_bytes, st);
  if (e != cudaSuccess) return from_cuda(e, "fused_gated_mlp: memset");
  h3::GemmArgs g1;
  g1.a = xq; g1.w = w1; g1.m = m; g1.n = ffn; g1.k = d; g1.lda = d; g1.ldw = d;
  g1.epilogue = h3::kEpiGeluAbsmax; g1.a_scale = xs; g1.w_scale = s1; g1.w_scale_per_channel = 1;
  g1.out = a; g1.ldo = ffn; g1.row_absmax = amax;
  e = h3::launch_gemm_i8(g1, st);
  if (e != cudaSuccess) return from_cuda(e, "fused_gated_mlp: fc1");
  h3::GemmArgs g2;
  g2.a = q2; g2.w = w2; g2.m = m; g2.n = d; g2.k = ffn; g2.lda = ffn; g2.ldw = ffn;
  g2.epilogue = h3::kEpiGatedResidual; g2.w_scale = s2; g2.w_scale_per_channel = 1;
  g2.requant_src = a; g2.requant_lds = ffn; g2.requant_ready = ready; g2.row_absmax = amax;
  g2.gate = gate; g2.row_map = row_map; g2.ldg = row_map != nullptr ? ldg : 0;
  g2.residual = residual; g2.ldr = ldr; g2.out = out; g2.ldo = ldo;
  e = h3::launch_gemm_i8(g2, st);
  return from_cuda(e, "fused_gated_mlp: fc2 (with the requantization of its input)");
}

extern "C" {

int h3b200_fused_gated_mlp(const void* x, int64_t ldx, const int8_t* w1, const float* s1, const int8_t* w2,
                           const float* s2, const void* gate, const void* residual, int64_t ldr, void* out,
                           int64_t ldo, int64_t m, int64_t d, int64_t ffn, int act, void* workspace,
                           int64_t workspace_bytes, h3b200_stream_t stream) {
  H3_GUARD("fused_gated_mlp", stream);
  return fused_gated_mlp_impl("fused_gated_mlp", x, ldx, w1, s1, w2, s2, gate, 0, nullptr, residual, ldr, out, ldo,
                              m, d, ffn, act, workspace, workspace_bytes, stream);
}

int h3b200_fused_gated_mlp_segmented(const void* x, int64_t ldx, const int8_t* w1, const float* s1,
                                     const int8_t* w2, const float* s2, const void* gate_rows, int64_t ldg,
                                     const int32_t* row_map, const void* residual, int64_t ldr, void* out,
                                     int64_t ldo, int64_t m, int64_t d, int64_t ffn, int act, void* workspace,
                                     int64_t workspace_bytes, h3b200_stream_t stream) {
  H3_GUARD("fused_gated_mlp_segmented", stream);
  if (m > 0 && row_map == nullptr) return fail(H3B200_ERR_INVALID, "fused_gated_mlp_segmented: row_map is NULL");
  return fused_gated_mlp_impl("fused_gated_mlp_segmented", x, ldx, w1, s1, w2, s2, gate_rows, ldg, row_map, residual,
                              ldr, out, ldo, m, d, ffn, act, workspace, workspace_bytes, stream);
}

int h3b200_rms_adaln(const void* x, int64_t ldx, const void* norm_weight, const void* scale, int64_t ld_scale,
                     const void* shift, int64_t ld_shift, int64_t mod_rows, const int32_t* row_map,
                     int64_t tokens_per_row, float eps, void* out, int64_t ldo, int64_t m, int64_t d,
                     h3b200_stream_t stream) {
  H3_GUARD("rms_adaln", stream);
  if (m < 0 || d <= 0 || ldx < d || ldo < d) return fail(H3B200_ERR_INVALID, "rms_adaln: bad shape m=%lld d=%lld ldx=%lld ldo=%lld", (long long)m, (long long)d, (long long)ldx, (long long)ldo);
  if ((scale == nullptr) != (shift == nullptr)) return fail(H3B200_ERR_INVALID, "rms_adaln: scale and shift must be given together");
  if (scale != nullptr && (mod_rows <= 0 || ld_scale < d || ld_shift < d)) return fail(H3B200_ERR_INVALID, "rms_adaln: modulation needs mod_rows >= 1 and row strides >= d");
  if (!(eps >= 0.0f)) return fail(H3B200_ERR_INVALID, "rms_adaln: eps must be >= 0");
  if (m == 0) return H3B200_OK;
  if (x == nullptr || out == nullptr) return fail(H3B200_ERR_INVALID, "rms_adaln: NULL pointer");
  if (d % 8 || d > 8192 || ldx % 8 || ldo % 8 || (scale != nullptr && (ld_scale % 8 || ld_shift % 8)))
    return fail(H3B200_ERR_UNSUPPORTED, "rms_adaln: needs d %% 8 == 0, d <= 8192 and row strides that are multiples of 8 elements");
  h3::RmsAdalnArgs a;
  a.x = x; a.ldx = ldx; a.y = out; a.ldy = ldo; a.weight = norm_weight;
  a.scale = scale; a.lds = ld_scale; a.shift = shift; a.ldh = ld_shift;
  a.row_map = row_map; a.tokens_per_row = tokens_per_row; a.rows = scale != nullptr ? mod_rows : 0;
  a.m = m; a.d = d; a.eps = eps;
  return from_cuda(h3::launch_rms_adaln(a, S(stream)), "rms_adaln");
}

int h3b200_adaln_rms_rope(const void* q, int64_t ldq, const void* k, int64_t ldk, void* q_out, int64_t ldqo,
                          void* k_out, int64_t ldko, const float* freqs, const void* q_weight, const void* k_weight,
                          const void* scale, const void* shift, int64_t m, int64_t heads, int64_t head_dim,
                          int64_t rot_dim, int norm_span, float eps, h3b200_stream_t stream) {
  H3_GUARD("adaln_rms_rope", stream);
  if (m < 0 || heads <= 0 || head_dim <= 0) return fail(H3B200_ERR_INVALID, "adaln_rms_rope: bad shape");
  if (norm_span != 0 && norm_span != 1) return fail(H3B200_ERR_INVALID, "adaln_rms_rope: norm_span must be 0 (row) or 1 (head)");
  const int64_t rot = rot_dim == 0 ? head_dim : rot_dim;
  if (rot < 0 || rot > head_dim || rot % 2) return fail(H3B200_ERR_INVALID, "adaln_rms_rope: rot_dim %lld invalid for head_dim %lld", (long long)rot_dim, (long long)head_dim);
  if ((scale == nullptr) != (shift == nullptr)) return fail(H3B200_ERR_INVALID, "adaln_rms_rope: scale and shift must both be given or both be NULL");
  if (ldq < heads * head_dim || ldk < heads * head_dim || ldqo < heads * head_dim || ldko < heads * head_dim) return fail(H3B200_ERR_INVALID, "adaln_rms_rope: token stride smaller than a row");
  if (m == 0) return H3B200_OK;
  h3::NormRopeArgs a;
  a.q = q; a.k = k; a.q_out = q_out; a.k_out = k_out; a.ldq = ldq; a.ldk = ldk; a.ldqo = ldqo; a.ldko = ldko;
  a.freqs = freqs; a.q_weight = q_weight; a.k_weight = k_weight; a.scale = scale; a.shift = shift;
  a.m = m; a.heads = heads; a.head_dim = head_dim; a.rot_dim = rot; a.norm_span = norm_span; a.eps = eps;
  return from_cuda(h3::launch_adaln_rms_rope(a, S(stream)), "adaln_rms_rope");
}

int h3b200_adaln_rms_rope_segmented(const void* q, int64_t ldq, const void* k, int64_t ldk, void* q_out,
                                    int64_t ldqo, void* k_out, int64_t ldko, const float* freqs,
                                    const void* q_weight, const void* k_weight, const void* scale,
                                    int64_t ld_scale, const void* shift, int64_t ld_shift, int64_t mod_rows,
                                    const int32_t* row_map, int64_t tokens_per_row, int64_t m, int64_t heads,
                                    int64_t head_dim, int64_t rot_dim, float eps, h3b200_stream_t stream) {
  H3_GUARD("adaln_rms_rope_segmented", stream);
  if (m < 0 || heads <= 0 || head_dim <= 0) return fail(H3B200_ERR_INVALID, "adaln_rms_rope_segmented: bad shape");
  const int64_t rot = rot_dim == 0 ? head_dim : rot_dim;
  if (rot < 0 || rot > head_dim || rot % 2) return fail(H3B200_ERR_INVALID, "adaln_rms_rope_segmented: rot_dim %lld invalid for head_dim %lld", (long long)rot_dim, (long long)head_dim);
  if (scale == nullptr || shift == nullptr || mod_rows < 1) return fail(H3B200_ERR_INVALID, "adaln_rms_rope_segmented: scale, shift and mod_rows >= 1 are required");
  const int64_t w = heads * head_dim;
  if (ld_scale < w || ld_shift < w) return fail(H3B200_ERR_INVALID, "adaln_rms_rope_segmented: modulation row strides must be >= heads * head_dim");
  if (ldq < w || ldk < w || ldqo < w || ldko < w) return fail(H3B200_ERR_INVALID, "adaln_rms_rope_segmented: token stride smaller than a row");
  if (m == 0) return H3B200_OK;
  h3::NormRopeArgs a;
  a.q = q; a.k = k; a.q_out = q_out; a.k_out = k_out; a.ldq = ldq; a.ldk = ldk; a.ldqo = ldqo; a.ldko = ldko;
  a.freqs = freqs; a.q_weight = q_weight; a.k_weight = k_weight; a.scale = scale; a.shift = shift;
  a.row_map = row_map; a.tokens_per_row = tokens_per_row; a.mod_rows = mod_rows; a.lds = ld_scale; a.ldh = ld_shift;
  a.m = m; a.heads = heads; a.head_dim = head_dim; a.rot_dim = rot; a.norm_span = 0; a.eps = eps;
  return from_cuda(h3::launch_adaln_rms_rope(a, S(stream)), "adaln_rms_rope_segmented");
}

int h3b200_qknorm_rope_strided(const void* q, int64_t q_st, int64_t q_sh, void* q_out, int64_t qo_st,
                               int64_t qo_sh, const void* q_weight, const void* k, int64_t k_st, int64_t k_sh,
                               void* k_out, int64_t ko_st, int64_t ko_sh, const void* k_weight, const void* freqs,
                               int freqs_dtype, int64_t f_st, int64_t f_sh, int64_t m, int64_t heads,
                               int64_t head_dim, int64_t rot_dim, float eps, h3b200_stream_t stream) {
  H3_GUARD("qknorm_rope_strided", stream);
  const char* who = "qknorm_rope_strided";
  if (m < 0 || heads <= 0 || head_dim <= 0) return fail(H3B200_ERR_INVALID, "%s: bad shape", who);
  const int64_t rot = rot_dim == 0 ? head_dim : rot_dim;
  if (rot < 0 || rot > head_dim || rot % 4) return fail(H3B200_ERR_INVALID, "%s: rot_dim %lld invalid for head_dim %lld", who, (long long)rot_dim, (long long)head_dim);
  if (head_dim != 128 || rot % 16) return fail(H3B200_ERR_UNSUPPORTED, "%s: head_dim 128 with rot_dim a multiple of 16 is built (got %lld, %lld)", who, (long long)head_dim, (long long)rot);
  if (freqs_dtype != H3B200_DTYPE_F32 && freqs_dtype != H3B200_DTYPE_BF16 && freqs_dtype != H3B200_DTYPE_F16)
    return fail(H3B200_ERR_INVALID, "%s: freqs dtype code must be 0 (float32), 1 (float16) or 2 (bfloat16), got %d", who, freqs_dtype);
  if (f_st < 0 || f_sh < 0) return fail(H3B200_ERR_INVALID, "%s: negative table stride", who);
  if (m == 0) return H3B200_OK;
  if (!q || !q_out || !q_weight || (k && (!k_out || !k_weight))) return fail(H3B200_ERR_INVALID, "%s: NULL pointer", who);
  h3::QKNormRopeArgs a;
  a.x[0] = q; a.y[0] = q_out; a.w[0] = q_weight; a.xs_t[0] = q_st; a.xs_h[0] = q_sh; a.ys_t[0] = qo_st; a.ys_h[0] = qo_sh;
  a.tensors = k ? 2 : 1;
  if (k) {
    a.x[1] = k; a.y[1] = k_out; a.w[1] = k_weight; a.xs_t[1] = k_st; a.xs_h[1] = k_sh; a.ys_t[1] = ko_st; a.ys_h[1] = ko_sh;
  }
  a.freqs = freqs;
  a.table_dtype = freqs_dtype == H3B200_DTYPE_F32 ? 0 : (freqs_dtype == H3B200_DTYPE_BF16 ? 1 : 2);
  a.fs_t = f_st; a.fs_h = f_sh;
  a.m = m; a.heads = heads; a.head_dim = head_dim; a.rot_dim = rot; a.eps = eps;
  return from_cuda(h3::launch_qk_rms_rope(a, S(stream)), who);
}

int64_t h3b200_qkv_qknorm_rope_workspace_bytes(int64_t m, int64_t heads, int64_t head_dim, int sec_begin,
                                              int sec_end) {
  if (m < 0 || heads <= 0 || head_dim <= 0 || sec_begin < 0 || sec_end > 3 || sec_begin >= sec_end) return 0;
  // the larger of the projection buffer (three-kernel path) and the transposed
  // rotation table (fused path: at most head_dim / 2 pairs x 16 bytes per token)
  return std::max(round_up(m * (sec_end - sec_begin) * heads * head_dim * 2, 256),
                  round_up(m * (head_dim / 2) * 16, 256)) + 256;
}

int h3b200_qkv_qknorm_rope(const int8_t* xq, const float* x_scale, int64_t m, int64_t k, const int8_t* w_qkv,
                           const float* w_scale, int64_t w_scale_numel, const void* bias, int64_t heads,
                           int64_t head_dim, int sec_begin, int sec_end, const void* q_norm_weight,
                           const void* k_norm_weight, const void* freqs, int freqs_dtype, int64_t f_st, int64_t f_sh,
                           int64_t rot_dim, float eps, void* q_out, int64_t q_st, int64_t q_sh, void* k_out,
                           int64_t k_st, int64_t k_sh, void* v_out, int64_t v_st, int64_t v_sh, void* workspace,
                           int64_t workspace_bytes, h3b200_stream_t stream) {
  H3_GUARD("qkv_qknorm_rope", stream);
  const char* who = "qkv_qknorm_rope";
  if (m < 0 || k <= 0 || heads <= 0 || head_dim != 128) return fail(H3B200_ERR_INVALID, "%s: bad shape (head_dim must be 128)", who);
  if (sec_begin < 0 || sec_end > 3 || sec_begin >= sec_end) return fail(H3B200_ERR_INVALID, "%s: section range [%d, %d) is not a non-empty part of Q|K|V", who, sec_begin, sec_end);
  const int64_t inner = heads * head_dim;
  if (w_scale_numel != 1 && w_scale_numel != 3 * inner) return fail(H3B200_ERR_INVALID, "%s: weight scale must be scalar or [3 * heads * head_dim]", who);
  const bool has_q = sec_begin == 0, has_k = sec_begin <= 1 && sec_end >= 2, has_v = sec_end == 3;
  if ((has_q && (!q_out || !q_norm_weight)) || (has_k && (!k_out || !k_norm_weight)) || (has_v && !v_out))
    return fail(H3B200_ERR_INVALID, "%s: an output or norm weight of a requested section is NULL", who);
  if (m == 0) return H3B200_OK;
  if (!xq || !x_scale || !w_qkv || !w_scale) return fail(H3B200_ERR_INVALID, "%s: NULL pointer", who);
  if (k % 16) return fail(H3B200_ERR_UNSUPPORTED, "%s: needs k %% 16 == 0", who);
  const int64_t need = h3b200_qkv_qknorm_rope_workspace_bytes(m, heads, head_dim, sec_begin, sec_end);
  if (workspace == nullptr || workspace_bytes < need) return fail(H3B200_ERR_INVALID, "%s: workspace too small (need %lld bytes)", who, (long long)need);
  cudaStream_t st = S(stream);
  const int64_t n = (sec_end - sec_begin) * inner;
  // Fused path: one GEMM whose epilogue normalises, rotates and stores every head
  // straight into the caller's views (per-token table, rotation a multiple of 32 dims).
  const int64_t rot = freqs ? (rot_dim == 0 ? head_dim : rot_dim) : 0;
  void* const outs[3] = {q_out, k_out, v_out};
  const int64_t sts[3] = {q_st, k_st, v_st}, shs[3] = {q_sh, k_sh, v_sh};
  bool fused = (freqs == nullptr || (f_sh == 0 && rot % 32 == 0 && rot >= 32 && rot <= 128)) && !(k % 16);
  for (int s = sec_begin; s < sec_end; ++s)
    fused = fused && !(reinterpret_cast<uintptr_t>(outs[s]) & 15) && sts[s] > 0 && shs[s] > 0 && sts[s] % 8 == 0 &&
            shs[s] % 8 == 0;
  if (fused) {
    float4* rope_t = nullptr;
    if (freqs) {
      if (freqs_dtype != H3B200_DTYPE_F32 && freqs_dtype != H3B200_DTYPE_BF16 && freqs_dtype != H3B200_DTYPE_F16)
        return fail(H3B200_ERR_INVALID, "%s: freqs dtype code must be 0, 1 or 2, got %d", who, freqs_dtype);
      rope_t = static_cast<float4*>(workspace);
      const int tab = freqs_dtype == H3B200_DTYPE_F32 ? 0 : (freqs_dtype == H3B200_DTYPE_BF16 ? 1 : 2);
      cudaError_t e = h3::launch_rope_table_transpose(freqs, tab, f_st, m, (int)(rot / 2), rope_t, st);
      if (e != cudaSuccess) return from_cuda(e, "qkv_qknorm_rope: rotation table");
    }
    h3::GemmArgs g;
    g.a = xq; g.w = w_qkv + sec_begin * inner * k; g.m = m; g.n = n; g.k = k; g.lda = k; g.ldw = k;
    g.epilogue = h3::kEpiQKV; g.a_scale = x_scale;
    g.w_scale = w_scale_numel == 1 ? w_scale : w_scale + sec_begin * inner;
    g.w_scale_per_channel = w_scale_numel == 1 ? 0 : 1;
    g.bias = bias ? static_cast<const __nv_bfloat16*>(bias) + sec_begin * inner : nullptr;
    g.qkv_heads = heads; g.qkv_sec0 = sec_begin; g.qkv_rot = (int)rot; g.rope_t = rope_t; g.qk_eps = eps;
    g.qk_w[0] = q_norm_weight; g.qk_w[1] = k_norm_weight;
    for (int s = 0; s < 3; ++s) {
      g.qkv_out[s] = outs[s]; g.qkv_st[s] = sts[s]; g.qkv_sh[s] = shs[s];
    }
    return from_cuda(h3::launch_gemm_i8(g, st), "qkv_qknorm_rope: fused projection");
  }
  auto* proj = static_cast<__nv_bfloat16*>(workspace);
  // the requested Q/K/V rows of the projection: dequant (+ bias) into [m, n] bf16
  h3::GemmArgs g;
  g.a = xq; g.w = w_qkv + sec_begin * inner * k; g.m = m; g.n = n; g.k = k; g.lda = k; g.ldw = k;
  g.epilogue = h3::kEpiBF16; g.a_scale = x_scale;
  g.w_scale = w_scale_numel == 1 ? w_scale : w_scale + sec_begin * inner;
  g.w_scale_per_channel = w_scale_numel == 1 ? 0 : 1;
  g.bias = bias ? static_cast<const __nv_bfloat16*>(bias) + sec_begin * inner : nullptr;
  g.out = proj; g.ldo = n;
  cudaError_t e = h3::launch_gemm_i8(g, st);
  if (e != cudaSuccess) return from_cuda(e, "qkv_qknorm_rope: projection");
  // QK-norm + RoPE of the Q and K sections (one launch for both) into the caller's views
  if (has_q || has_k) {
    const int rc = h3b200_qknorm_rope_strided(
        has_q ? proj : proj + (1 - sec_begin) * inner, n, head_dim, has_q ? q_out : k_out, has_q ? q_st : k_st,
        has_q ? q_sh : k_sh, has_q ? q_norm_weight : k_norm_weight, has_q && has_k ? proj + inner : nullptr, n,
        head_dim, has_q && has_k ? k_out : nullptr, k_st, k_sh, k_norm_weight, freqs, freqs_dtype, f_st, f_sh, m,
        heads, head_dim, rot_dim, eps, stream);
    if (rc != H3B200_OK) return rc;
  }
  if (has_v) {
    e = h3::launch_copy_heads(proj + (2 - sec_begin) * inner, n, head_dim, v_out, v_st, v_sh, m, heads, st);
    if (e != cudaSuccess) return from_cuda(e, "qkv_qknorm_rope: V layout");
  }
  return H3B200_OK;
}

int h3b200_dequant_int4_grouped_to_int8_ex(const int8_t* qdata, const void* s_rel, int s_rel_dtype,
                                           const float* codebook, int64_t n, int64_t k, int64_t group_size,
                                           int8_t* out, h3b200_stream_t stream) {
  H3_GUARD("dequant_int4_grouped_to_int8_ex", stream);
  if (n < 0 || k < 0) return fail(H3B200_ERR_INVALID, "dequant_int4_grouped_to_int8: negative shape");
  if (group_size < 4 || k % 16 || k % group_size || (16 % group_size && group_size % 16))
    return fail(H3B200_ERR_INVALID, "dequant_int4_grouped_to_int8: K=%lld must be divisible by 16 and group_size=%lld; group_size must be >=4 and divide 16 or be a multiple of 16", (long long)k, (long long)group_size);
  if (s_rel_dtype != H3B200_DTYPE_F32 && s_rel_dtype != H3B200_DTYPE_E4M3)
    return fail(H3B200_ERR_INVALID, "dequant_int4_grouped_to_int8: s_rel dtype code must be 0 (float32) or 5 (float8_e4m3fn), got %d", s_rel_dtype);
  if (n == 0 || k == 0) return H3B200_OK;
  if (!qdata || !s_rel || !out) return fail(H3B200_ERR_INVALID, "dequant_int4_grouped_to_int8: NULL pointer");
  return from_cuda(h3::launch_dequant_int4(qdata, s_rel, s_rel_dtype == H3B200_DTYPE_E4M3, codebook, n, k, group_size,
                                           out, S(stream)),
                   "dequant_int4_grouped_to_int8");
}

int h3b200_dequant_int4_grouped_to_int8(const int8_t* qdata, const float* s_rel, int64_t n, int64_t k,
                                        int64_t group_size, int8_t* out, h3b200_stream_t stream) {
  H3_GUARD("dequant_int4_grouped_to_int8", stream);
  return h3b200_dequant_int4_grouped_to_int8_ex(qdata, s_rel, H3B200_DTYPE_F32, nullptr, n, k, group_size, out,
                                                stream);
}

int h3b200_quantize_int8_rowwise_convrot(const void* x, int64_t m, int64_t k, int64_t ldx, int64_t group_size,
                                         int act, int8_t* q, float* scale, h3b200_stream_t stream) {
  H3_GUARD("quantize_int8_rowwise_convrot", stream);
  if (act != H3B200_ACT_NONE && act != H3B200_ACT_GELU_TANH && act != H3B200_ACT_SWIGLU) return fail(H3B200_ERR_INVALID, "quantize_int8_rowwise_convrot: unsupported act %d", act);
  if (m < 0 || k < 0 || ldx < k * act_width(act)) return fail(H3B200_ERR_INVALID, "quantize_int8_rowwise_convrot: bad shape");
  if (group_size != 256) return fail(H3B200_ERR_UNSUPPORTED, "quantize_int8_rowwise_convrot: only group_size 256 is built (got %lld)", (long long)group_size);
  if (k % 256) return fail(H3B200_ERR_INVALID, "quantize_int8_rowwise_convrot: ConvRot group size 256 does not divide input features %lld", (long long)k);
  if (m == 0) return H3B200_OK;
  if (!x || !q || !scale) return fail(H3B200_ERR_INVALID, "quantize_int8_rowwise_convrot: NULL pointer");
  return from_cuda(h3::launch_quantize_convrot(x, ldx, m, k, act, q, scale, nullptr, 0, 0, S(stream)), "quantize_int8_rowwise_convrot");
}

int64_t h3b200_w4a8_linear_workspace_bytes(int64_t m, int64_t n, int64_t k, int64_t group_size) {
  const int64_t kp = group_size > 0 ? h3::correction_kpad(k / group_size) : 0;
  return round_up(m * k, 256) + round_up(m * 4, 256) + round_up(m * kp * 2, 256) + round_up(n * kp * 2, 256) + 1024;
}

int h3b200_w4a8_int8_linear(const void* x, int64_t ldx, const int8_t* grid, const float* s_channel,
                            const void* correction, const void* bias, int64_t group_size, int64_t convrot_group,
                            int act, void* out,
                            int64_t m, int64_t n, int64_t k, void* workspace, int64_t workspace_bytes,
                            h3b200_stream_t stream) {
  H3_GUARD("w4a8_int8_linear", stream);
  if (act != H3B200_ACT_NONE && act != H3B200_ACT_GELU_TANH && act != H3B200_ACT_SWIGLU) return fail(H3B200_ERR_INVALID, "w4a8_int8_linear: unsupported act code %d", act);
  if (m < 0 || n < 0 || k < 0 || ldx < k * act_width(act)) return fail(H3B200_ERR_INVALID, "w4a8_int8_linear: bad shape");
  if (group_size < 4 || k % 16 || k % group_size || k % convrot_group || (16 % group_size && group_size % 16))
    return fail(H3B200_ERR_INVALID, "w4a8_int8_linear: K=%lld must be divisible by 16, group_size=%lld, and convrot_groupsize=%lld", (long long)k, (long long)group_size, (long long)convrot_group);
  if (convrot_group != 256) return fail(H3B200_ERR_UNSUPPORTED, "w4a8_int8_linear: only convrot_groupsize 256 is built");
  if (correction != nullptr && (group_size % 8 || 256 % group_size)) return fail(H3B200_ERR_UNSUPPORTED, "w4a8_int8_linear: asymmetric correction needs group_size dividing 256");
  if (m == 0 || n == 0) return H3B200_OK;
  if (!x || !grid || !s_channel || !out) return fail(H3B200_ERR_INVALID, "w4a8_int8_linear: NULL pointer");
  if (n % 8) return fail(H3B200_ERR_UNSUPPORTED, "w4a8_int8_linear: needs n %% 8 == 0");
  if (workspace == nullptr || workspace_bytes < h3b200_w4a8_linear_workspace_bytes(m, n, k, group_size)) return fail(H3B200_ERR_INVALID, "w4a8_int8_linear: workspace too small (need %lld bytes)", (long long)h3b200_w4a8_linear_workspace_bytes(m, n, k, group_size));
  const int64_t groups = k / group_size, kp = h3::correction_kpad(groups);
  if (correction != nullptr && kp > 128) return fail(H3B200_ERR_UNSUPPORTED, "w4a8_int8_linear: at most 128 correction groups are built (K / group_size = %lld)", (long long)groups);
  Carver c{static_cast<uint8_t*>(workspace), workspace_bytes};
  int8_t* xq = static_cast<int8_t*>(c.take(m * k));
  float* xs = static_cast<float*>(c.take(m * 4));
  void* sx = c.take(m * kp * 2);
  void* corr_t = c.take(n * kp * 2);
  if (!c.ok) return fail(H3B200_ERR_INVALID, "w4a8_int8_linear: workspace too small");
  cudaStream_t st = S(stream);
  cudaError_t e = h3::launch_quantize_convrot(x, ldx, m, k, act, xq, xs, correction ? sx : nullptr, group_size, kp, st);
  if (e != cudaSuccess) return from_cuda(e, "w4a8_int8_linear: convrot quantize");
  if (correction != nullptr) {
    e = h3::launch_correction_transpose(correction, groups, n, kp, corr_t, st);
    if (e != cudaSuccess) return from_cuda(e, "w4a8_int8_linear: correction layout");
  }
  // GEMM with the dequant epilogue; the asymmetric correction is fused into it
  h3::GemmArgs g;
  g.a = xq; g.w = grid; g.m = m; g.n = n; g.k = k; g.lda = k; g.ldw = k;
  g.epilogue = correction ? h3::kEpiBF16Corr : h3::kEpiBF16;
  g.a_scale = xs; g.w_scale = s_channel; g.w_scale_per_channel = 1;
  g.bias = bias; g.out = out; g.ldo = n;
  g.sx = sx; g.corr_t = corr_t; g.kp = kp;
  e = h3::launch_gemm_i8(g, st);
  return from_cuda(e, "w4a8_int8_linear: gemm");
}


int64_t h3b200_w4a8_linear_packed_workspace_bytes(int64_t m, int64_t n, int64_t k, int64_t group_size) {
  // large m: the decoded int8 grid in front of the grid path's own workspace; small m: the
  // split-K int32 sums [m, n] and one counter per output tile after the quantized activation
  if (!h3::gemm_w4_smallm_supported(m, n, k, group_size, 0))
    return round_up(n * k, 256) + h3b200_w4a8_linear_workspace_bytes(m, n, k, group_size);
  const int64_t tiles = ((n + 255) / 256) * ((m + 127) / 128);
  int dev = 0;
  cudaGetDevice(&dev);
  const int64_t splits = h3::gemm_w4_smallm_splits(m, n, k, h3::num_sms(dev));
  (void)splits;
  return h3b200_w4a8_linear_workspace_bytes(m, n, k, group_size) + round_up(m * n * 4, 256) + round_up(tiles * 4, 256);
}

int h3b200_w4a8_int8_linear_packed(const void* x, int64_t ldx, const uint8_t* qdata, const void* s_rel,
                                   int s_rel_dtype, const float* codebook, const float* s_channel,
                                   const void* correction, const void* bias, int64_t group_size,
                                   int64_t convrot_group, int act, void* out, int64_t m, int64_t n, int64_t k,
                                   void* workspace, int64_t workspace_bytes, h3b200_stream_t stream) {
  H3_GUARD("w4a8_int8_linear_packed", stream);
  if (s_rel_dtype != H3B200_DTYPE_F32 && s_rel_dtype != H3B200_DTYPE_E4M3) return fail(H3B200_ERR_INVALID, "w4a8_int8_linear_packed: s_rel dtype code must be 0 (float32) or 5 (float8_e4m3fn), got %d", s_rel_dtype);
  if (act != H3B200_ACT_NONE && act != H3B200_ACT_GELU_TANH && act != H3B200_ACT_SWIGLU) return fail(H3B200_ERR_INVALID, "w4a8_int8_linear_packed: unsupported act code %d", act);
  if (m < 0 || n < 0 || k < 0 || ldx < k * act_width(act)) return fail(H3B200_ERR_INVALID, "w4a8_int8_linear_packed: bad shape");
  if (group_size < 4 || k % 16 || k % group_size || k % convrot_group || (16 % group_size && group_size % 16))
    return fail(H3B200_ERR_INVALID, "w4a8_int8_linear_packed: K=%lld must be divisible by 16, group_size=%lld, and convrot_groupsize=%lld", (long long)k, (long long)group_size, (long long)convrot_group);
  if (convrot_group != 256) return fail(H3B200_ERR_UNSUPPORTED, "w4a8_int8_linear_packed: only convrot_groupsize 256 is built");
  if (m == 0 || n == 0) return H3B200_OK;
  if (!x || !qdata || !s_rel || !s_channel || !out) return fail(H3B200_ERR_INVALID, "w4a8_int8_linear_packed: NULL pointer");
  if (n % 8) return fail(H3B200_ERR_UNSUPPORTED, "w4a8_int8_linear_packed: needs n %% 8 == 0");
  const int64_t need = h3b200_w4a8_linear_packed_workspace_bytes(m, n, k, group_size);
  if (workspace == nullptr || workspace_bytes < need) return fail(H3B200_ERR_INVALID, "w4a8_int8_linear_packed: workspace too small (need %lld bytes)", (long long)need);
  const int64_t groups = k / group_size;
  if (h3::gemm_w4_smallm_supported(m, n, k, group_size, correction ? groups : 0) &&
      !(reinterpret_cast<uintptr_t>(qdata) & 15)) {
    // few rows: the GEMM unpacks the int4 weight in shared memory
    if (correction != nullptr && (group_size % 8 || 256 % group_size)) return fail(H3B200_ERR_UNSUPPORTED, "w4a8_int8_linear_packed: asymmetric correction needs group_size dividing 256");
    const int64_t kp = h3::correction_kpad(groups);
    Carver c{static_cast<uint8_t*>(workspace), workspace_bytes};
    int8_t* xq = static_cast<int8_t*>(c.take(m * k));
    float* xs = static_cast<float*>(c.take(m * 4));
    void* sx = c.take(m * kp * 2);
    const int64_t tiles = ((n + 255) / 256) * ((m + 127) / 128);
    int dev = 0;
    cudaGetDevice(&dev);
    const int splits = h3::gemm_w4_smallm_splits(m, n, k, h3::num_sms(dev));
    int32_t* acc_ws = static_cast<int32_t*>(c.take(m * n * 4));  // the splits' int32 sums
    unsigned int* tile_cnt = static_cast<unsigned int*>(c.take(tiles * 4));
    if (!c.ok) return fail(H3B200_ERR_INVALID, "w4a8_int8_linear_packed: workspace too small");
    cudaStream_t st = S(stream);
    // the sums and the tile counters start at zero (contiguous in the workspace)
    cudaError_t e = cudaMemsetAsync(acc_ws, 0, (size_t)(reinterpret_cast<uint8_t*>(tile_cnt + tiles) -
                                                        reinterpret_cast<uint8_t*>(acc_ws)), st);
    if (e != cudaSuccess) return from_cuda(e, "w4a8_int8_linear_packed: memset");
    e = h3::launch_quantize_convrot(x, ldx, m, k, act, xq, xs, correction ? sx : nullptr, group_size, kp, st);
    if (e != cudaSuccess) return from_cuda(e, "w4a8_int8_linear_packed: convrot quantize");
    h3::W4SmallMArgs a;
    a.xq = xq; a.xs = xs; a.qdata = qdata; a.s_rel = s_rel; a.s_rel_e4m3 = s_rel_dtype == H3B200_DTYPE_E4M3;
    a.codebook = codebook; a.s_channel = s_channel; a.bias = bias;
    a.sx = correction ? sx : nullptr; a.kp = kp; a.corr = correction;
    a.out = out; a.ldo = n; a.m = m; a.n = n; a.k = k; a.group = group_size;
    a.splits = splits; a.acc_ws = acc_ws; a.tile_cnt = tile_cnt;
    return from_cuda(h3::launch_gemm_w4_smallm(a, st), "w4a8_int8_linear_packed: small-M W4 GEMM");
  }
  // many rows: decode the grid once into the workspace, then the INT8 GEMM path
  Carver c{static_cast<uint8_t*>(workspace), workspace_bytes};
  int8_t* grid = static_cast<int8_t*>(c.take(n * k));
  if (!c.ok) return fail(H3B200_ERR_INVALID, "w4a8_int8_linear_packed: workspace too small");
  uint8_t* rest = static_cast<uint8_t*>(workspace) + round_up(n * k, 256);
  int stc = h3b200_dequant_int4_grouped_to_int8_ex(reinterpret_cast<const int8_t*>(qdata), s_rel, s_rel_dtype, codebook,
                                                   n, k, group_size, grid, stream);
  if (stc != H3B200_OK) return stc;
  return h3b200_w4a8_int8_linear(x, ldx, grid, s_channel, correction, bias, group_size, convrot_group, act, out, m, n,
                                 k, rest, workspace_bytes - round_up(n * k, 256), stream);
}

int64_t h3b200_fused_gated_mlp_swiglu_workspace_bytes(int64_t chunk_tokens, int64_t d, int64_t ffn) {
  if (chunk_tokens <= 0 || d <= 0 || ffn <= 0) return 0;
  const int64_t c = chunk_tokens;
  // xq, xs, h = silu(gate) * up (bf16 [c, ffn], written by fc1's epilogue), q2, xs2
  return round_up(c * d, 256) + round_up(c * 4, 256) * 2 + round_up(c * ffn * 2, 256) + round_up(c * ffn, 256) +
         1024;
}

}  // extern "C"

namespace {

struct SwiGLUMlp {
  const void* x; int64_t ldx;
  const int8_t* w1; const float* s1; int64_t s1_numel; const void* b1;
  const int8_t* w2; const float* s2; int64_t s2_numel; const void* b2;
  const void* gate; int64_t ldg; const int32_t* row_map;
  const void* residual; int64_t ldr; void* out; int64_t ldo;
  int64_t m, d, ffn, fc1_convrot_group, chunk_tokens;
};

// Shape and pointer checks shared by the INT8 and W4A8 SwiGLU MLPs (the weight
// pointers are checked by the callers).
int check_swiglu_mlp(const SwiGLUMlp& a, const char* who) {
  if (a.m < 0 || a.d <= 0 || a.ffn <= 0 || a.ldx < a.d || a.ldr < a.d || a.ldo < a.d || a.chunk_tokens <= 0)
    return fail(H3B200_ERR_INVALID, "%s: bad shape m=%lld d=%lld ffn=%lld chunk=%lld", who, (long long)a.m, (long long)a.d, (long long)a.ffn, (long long)a.chunk_tokens);
  if (a.fc1_convrot_group != 0 && a.fc1_convrot_group != 256) return fail(H3B200_ERR_UNSUPPORTED, "%s: fc1 ConvRot group must be 0 (off) or 256, got %lld", who, (long long)a.fc1_convrot_group);
  if (a.d % 256 && a.fc1_convrot_group) return fail(H3B200_ERR_INVALID, "%s: ConvRot group 256 does not divide d=%lld", who, (long long)a.d);
  if (a.ffn % 256) return fail(H3B200_ERR_INVALID, "%s: fc2 ConvRot group 256 does not divide ffn=%lld", who, (long long)a.ffn);
  if (a.d % 16) return fail(H3B200_ERR_UNSUPPORTED, "%s: needs d %% 16 == 0", who);
  if (a.s1_numel != 1 && a.s1_numel != 2 * a.ffn) return fail(H3B200_ERR_INVALID, "%s: fc1 scale must be scalar or [2*ffn]", who);
  if (a.s2_numel != 1 && a.s2_numel != a.d) return fail(H3B200_ERR_INVALID, "%s: fc2 scale must be scalar or [d]", who);
  if (a.row_map != nullptr && a.ldg < a.d) return fail(H3B200_ERR_INVALID, "%s: gate row stride %lld < d", who, (long long)a.ldg);
  if (a.m > 0 && (!a.x || !a.gate || !a.residual || !a.out)) return fail(H3B200_ERR_INVALID, "%s: NULL pointer", who);
  return H3B200_OK;
}

// Per chunk of tokens: (ConvRot-)quantize x -> fc1 GEMM (dequant + bias) ->
// SwiGLU + ConvRot-256 + quantize -> fc2 GEMM (dequant + bias + gated residual
// by modulation row). `work` holds at least
// h3b200_fused_gated_mlp_swiglu_workspace_bytes(min(chunk, m), d, ffn) bytes.
int run_swiglu_mlp(const SwiGLUMlp& a, void* work, int64_t work_bytes, cudaStream_t st, const char* who) {
  const int64_t m = a.m, d = a.d, ffn = a.ffn;
  const int64_t chunk = std::min(a.chunk_tokens, m);
  Carver c{static_cast<uint8_t*>(work), work_bytes};
  int8_t* xq = static_cast<int8_t*>(c.take(chunk * d));
  float* xs = static_cast<float*>(c.take(chunk * 4));
  void* hbuf = c.take(chunk * ffn * 2);
  int8_t* q2 = static_cast<int8_t*>(c.take(chunk * ffn));
  float* xs2 = static_cast<float*>(c.take(chunk * 4));
  if (!c.ok) return fail(H3B200_ERR_INVALID, "%s: workspace too small", who);
  const auto* xb = static_cast<const __nv_bfloat16*>(a.x);
  const auto* rb = static_cast<const __nv_bfloat16*>(a.residual);
  auto* ob = static_cast<__nv_bfloat16*>(a.out);
  for (int64_t s0 = 0; s0 < m; s0 += chunk) {
    const int64_t mc = std::min(chunk, m - s0);
    // fc1: (ConvRot-)quantize x, GEMM with the SwiGLU epilogue: the gate and up halves
    // of each output column are dequantized (+ bias) and combined in the same tile,
    // h [mc, ffn] = bf16(silu(gate) * up)
    cudaError_t e = a.fc1_convrot_group
                        ? h3::launch_quantize_convrot(xb + s0 * a.ldx, a.ldx, mc, d, H3B200_ACT_NONE, xq, xs, nullptr, 0, 0, st)
                        : h3::launch_quantize_rows(xb + s0 * a.ldx, a.ldx, mc, d, H3B200_ACT_NONE, nullptr, xq, xs, st);
    if (e != cudaSuccess) return from_cuda(e, "swiglu mlp: quantize x");
    h3::GemmArgs g1;
    g1.a = xq; g1.w = a.w1; g1.m = mc; g1.n = 2 * ffn; g1.k = d; g1.lda = d; g1.ldw = d;
    g1.epilogue = h3::kEpiSwiGLU; g1.a_scale = xs; g1.w_scale = a.s1; g1.w_scale_per_channel = a.s1_numel > 1 ? 1 : 0;
    g1.bias = a.b1; g1.out = hbuf; g1.ldo = ffn;
    e = h3::launch_gemm_i8(g1, st);
    if (e != cudaSuccess) return from_cuda(e, "swiglu mlp: fc1");
    // fc2: ConvRot-256 + quantize h, GEMM, dequant (+ bias), gated residual per modulation row
    e = h3::launch_quantize_convrot(hbuf, ffn, mc, ffn, H3B200_ACT_NONE, q2, xs2, nullptr, 0, 0, st);
    if (e != cudaSuccess) return from_cuda(e, "swiglu mlp: quantize h");
    h3::GemmArgs g2;
    g2.a = q2; g2.w = a.w2; g2.m = mc; g2.n = d; g2.k = ffn; g2.lda = ffn; g2.ldw = ffn;
    g2.epilogue = h3::kEpiGatedResidual; g2.a_scale = xs2; g2.w_scale = a.s2; g2.w_scale_per_channel = a.s2_numel > 1 ? 1 : 0;
    g2.bias = a.b2; g2.gate = a.gate; g2.row_map = a.row_map ? a.row_map + s0 : nullptr; g2.ldg = a.ldg;
    g2.residual = rb + s0 * a.ldr; g2.ldr = a.ldr; g2.out = ob + s0 * a.ldo; g2.ldo = a.ldo;
    e = h3::launch_gemm_i8(g2, st);
    if (e != cudaSuccess) return from_cuda(e, "swiglu mlp: fc2");
  }
  return H3B200_OK;
}

}  // namespace

extern "C" {

int h3b200_fused_gated_mlp_swiglu(const void* x, int64_t ldx, const int8_t* w1, const float* s1, int64_t s1_numel,
                                  const void* b1, const int8_t* w2, const float* s2, int64_t s2_numel, const void* b2,
                                  const void* gate, int64_t ldg, const int32_t* row_map, const void* residual,
                                  int64_t ldr, void* out, int64_t ldo, int64_t m, int64_t d, int64_t ffn,
                                  int64_t fc1_convrot_group, int64_t chunk_tokens, void* workspace,
                                  int64_t workspace_bytes, h3b200_stream_t stream) {
  H3_GUARD("fused_gated_mlp_swiglu", stream);
  const SwiGLUMlp a{x, ldx, w1, s1, s1_numel, b1, w2, s2, s2_numel, b2, gate, ldg, row_map, residual, ldr, out, ldo,
                    m, d, ffn, fc1_convrot_group, chunk_tokens};
  if (int rc = check_swiglu_mlp(a, "fused_gated_mlp_swiglu")) return rc;
  if (m == 0) return H3B200_OK;
  if (!w1 || !s1 || !w2 || !s2) return fail(H3B200_ERR_INVALID, "fused_gated_mlp_swiglu: NULL pointer");
  const int64_t chunk = std::min(chunk_tokens, m);
  const int64_t need = h3b200_fused_gated_mlp_swiglu_workspace_bytes(chunk, d, ffn);
  if (workspace == nullptr || workspace_bytes < need) return fail(H3B200_ERR_INVALID, "fused_gated_mlp_swiglu: workspace too small (need %lld bytes for %lld-token chunks)", (long long)need, (long long)chunk);
  return run_swiglu_mlp(a, workspace, workspace_bytes, S(stream), "fused_gated_mlp_swiglu");
}

int64_t h3b200_fused_gated_mlp_swiglu_w4a8_workspace_bytes(int64_t chunk_tokens, int64_t d, int64_t ffn) {
  if (chunk_tokens <= 0 || d <= 0 || ffn <= 0) return 0;
  return round_up(2 * ffn * d, 256) + round_up(d * ffn, 256) +
         h3b200_fused_gated_mlp_swiglu_workspace_bytes(chunk_tokens, d, ffn) + 256;
}

int h3b200_fused_gated_mlp_swiglu_w4a8(const void* x, int64_t ldx, const int8_t* qdata1, const void* s_rel1,
                                       const float* s_channel1, const float* codebook1, const void* b1,
                                       const int8_t* qdata2, const void* s_rel2, const float* s_channel2,
                                       const float* codebook2, const void* b2, int s_rel_dtype, int64_t group_size,
                                       const void* gate, int64_t ldg, const int32_t* row_map, const void* residual,
                                       int64_t ldr, void* out, int64_t ldo, int64_t m, int64_t d, int64_t ffn,
                                       int64_t chunk_tokens, void* workspace, int64_t workspace_bytes,
                                       h3b200_stream_t stream) {
  H3_GUARD("fused_gated_mlp_swiglu_w4a8", stream);
  const char* who = "fused_gated_mlp_swiglu_w4a8";
  if (group_size < 4 || (16 % group_size && group_size % 16) || d % group_size || ffn % group_size)
    return fail(H3B200_ERR_INVALID, "%s: group_size=%lld must be >=4, divide 16 or be a multiple of 16, and divide d and ffn", who, (long long)group_size);
  if (s_rel_dtype != H3B200_DTYPE_F32 && s_rel_dtype != H3B200_DTYPE_E4M3)
    return fail(H3B200_ERR_INVALID, "%s: s_rel dtype code must be 0 (float32) or 5 (float8_e4m3fn), got %d", who, s_rel_dtype);
  const SwiGLUMlp a0{x, ldx, nullptr, s_channel1, 2 * ffn, b1, nullptr, s_channel2, d, b2, gate, ldg, row_map,
                     residual, ldr, out, ldo, m, d, ffn, 256, chunk_tokens};
  if (int rc = check_swiglu_mlp(a0, who)) return rc;
  if (m == 0) return H3B200_OK;
  if (!qdata1 || !s_rel1 || !s_channel1 || !qdata2 || !s_rel2 || !s_channel2) return fail(H3B200_ERR_INVALID, "%s: NULL pointer", who);
  const int64_t chunk = std::min(chunk_tokens, m);
  const int64_t need = h3b200_fused_gated_mlp_swiglu_w4a8_workspace_bytes(chunk, d, ffn);
  if (workspace == nullptr || workspace_bytes < need) return fail(H3B200_ERR_INVALID, "%s: workspace too small (need %lld bytes for %lld-token chunks)", who, (long long)need, (long long)chunk);
  Carver c{static_cast<uint8_t*>(workspace), workspace_bytes};
  int8_t* grid1 = static_cast<int8_t*>(c.take(2 * ffn * d));
  int8_t* grid2 = static_cast<int8_t*>(c.take(d * ffn));
  c.off = round_up(c.off, 256);
  if (!c.ok) return fail(H3B200_ERR_INVALID, "%s: workspace too small", who);
  cudaStream_t st = S(stream);
  const bool e4m3 = s_rel_dtype == H3B200_DTYPE_E4M3;
  // the int4 weights are decoded once per call; every token chunk's GEMMs read the grids
  cudaError_t e = h3::launch_dequant_int4(qdata1, s_rel1, e4m3, codebook1, 2 * ffn, d, group_size, grid1, st);
  if (e != cudaSuccess) return from_cuda(e, "fused_gated_mlp_swiglu_w4a8: decode W1");
  e = h3::launch_dequant_int4(qdata2, s_rel2, e4m3, codebook2, d, ffn, group_size, grid2, st);
  if (e != cudaSuccess) return from_cuda(e, "fused_gated_mlp_swiglu_w4a8: decode W2");
  SwiGLUMlp a = a0;
  a.w1 = grid1; a.w2 = grid2;
  return run_swiglu_mlp(a, static_cast<uint8_t*>(workspace) + c.off, workspace_bytes - c.off, st, who);
}

int64_t h3b200_fused_gated_mlp_w4a8_workspace_bytes(int64_t m, int64_t d, int64_t ffn, int64_t group_size) {
  if (m < 0 || d <= 0 || ffn <= 0 || group_size <= 0) return 0;
  const int64_t kp1 = h3::correction_kpad(d / group_size), kp2 = h3::correction_kpad(ffn / group_size);
  return round_up(ffn * d, 256) * 2 + round_up(m * d, 256) + round_up(m * 4, 256) * 2 +
         round_up(m * kp1 * 2, 256) + round_up(ffn * kp1 * 2, 256) + round_up(m * ffn * 2, 256) +
         round_up(m * ffn, 256) + round_up(m * kp2 * 2, 256) + round_up(d * kp2 * 2, 256) + 4096;
}

int h3b200_fused_gated_mlp_w4a8(const void* x, int64_t ldx, const int8_t* qdata1, const float* s_rel1,
                                const float* s_channel1, const void* correction1, const int8_t* qdata2,
                                const float* s_rel2, const float* s_channel2, const void* correction2,
                                const void* gate, const void* residual, int64_t ldr, void* out, int64_t ldo,
                                int64_t m, int64_t d, int64_t ffn, int64_t group_size, int act, void* workspace,
                                int64_t workspace_bytes, h3b200_stream_t stream) {
  H3_GUARD("fused_gated_mlp_w4a8", stream);
  if (m < 0 || d <= 0 || ffn <= 0 || ldx < d || ldr < d || ldo < d) return fail(H3B200_ERR_INVALID, "fused_gated_mlp_w4a8: bad shape m=%lld d=%lld ffn=%lld", (long long)m, (long long)d, (long long)ffn);
  if (act != H3B200_ACT_GELU_TANH) return fail(H3B200_ERR_UNSUPPORTED, "fused_gated_mlp_w4a8: only act=gelu_tanh (1) is built, got %d", act);
  if (group_size < 16 || group_size % 16 || 256 % group_size) return fail(H3B200_ERR_UNSUPPORTED, "fused_gated_mlp_w4a8: group_size must be 16..256 and divide 256, got %lld", (long long)group_size);
  if (d % 256 || ffn % 256) return fail(H3B200_ERR_UNSUPPORTED, "fused_gated_mlp_w4a8: d and ffn must be multiples of 256 (ConvRot-256)");
  if (m == 0) return H3B200_OK;
  if (!x || !qdata1 || !s_rel1 || !s_channel1 || !qdata2 || !s_rel2 || !s_channel2 || !gate || !residual || !out) return fail(H3B200_ERR_INVALID, "fused_gated_mlp_w4a8: NULL pointer");
  const int64_t need = h3b200_fused_gated_mlp_w4a8_workspace_bytes(m, d, ffn, group_size);
  if (workspace == nullptr || workspace_bytes < need) return fail(H3B200_ERR_INVALID, "fused_gated_mlp_w4a8: workspace too small (need %lld bytes)", (long long)need);
  const int64_t ng1 = d / group_size, ng2 = ffn / group_size;
  const int64_t kp1 = h3::correction_kpad(ng1), kp2 = h3::correction_kpad(ng2);
  if (kp1 > 128 || kp2 > 128) return fail(H3B200_ERR_UNSUPPORTED, "fused_gated_mlp_w4a8: at most 128 correction groups are built");
  Carver c{static_cast<uint8_t*>(workspace), workspace_bytes};
  int8_t* grid1 = static_cast<int8_t*>(c.take(ffn * d));
  int8_t* grid2 = static_cast<int8_t*>(c.take(d * ffn));
  int8_t* xq = static_cast<int8_t*>(c.take(m * d));
  float* xs = static_cast<float*>(c.take(m * 4));
  void* sx1 = c.take(m * kp1 * 2);
  void* ct1 = c.take(ffn * kp1 * 2);
  void* h = c.take(m * ffn * 2);
  int8_t* q2 = static_cast<int8_t*>(c.take(m * ffn));
  float* xs2 = static_cast<float*>(c.take(m * 4));
  void* sx2 = c.take(m * kp2 * 2);
  void* ct2 = c.take(d * kp2 * 2);
  if (!c.ok) return fail(H3B200_ERR_INVALID, "fused_gated_mlp_w4a8: workspace too small");
  cudaStream_t st = S(stream);
  cudaError_t e = h3::launch_dequant_int4(qdata1, s_rel1, false, nullptr, ffn, d, group_size, grid1, st);
  if (e != cudaSuccess) return from_cuda(e, "fused_gated_mlp_w4a8: decode W1");
  e = h3::launch_dequant_int4(qdata2, s_rel2, false, nullptr, d, ffn, group_size, grid2, st);
  if (e != cudaSuccess) return from_cuda(e, "fused_gated_mlp_w4a8: decode W2");
  // fc1: ConvRot-quantize x, GEMM, asymmetric correction
  e = h3::launch_quantize_convrot(x, ldx, m, d, H3B200_ACT_NONE, xq, xs, correction1 ? sx1 : nullptr, group_size, kp1, st);
  if (e != cudaSuccess) return from_cuda(e, "fused_gated_mlp_w4a8: quantize x");
  if (correction1) {
    e = h3::launch_correction_transpose(correction1, ng1, ffn, kp1, ct1, st);
    if (e != cudaSuccess) return from_cuda(e, "fused_gated_mlp_w4a8: fc1 correction layout");
  }
  // fc1 GEMM: dequant, asymmetric correction and GELU in the epilogue (without
  // a correction the plain dequant epilogue runs and the fc2 quantizer applies the GELU)
  h3::GemmArgs g1;
  g1.a = xq; g1.w = grid1; g1.m = m; g1.n = ffn; g1.k = d; g1.lda = d; g1.ldw = d;
  g1.epilogue = correction1 ? h3::kEpiBF16CorrGelu : h3::kEpiBF16;
  g1.a_scale = xs; g1.w_scale = s_channel1; g1.w_scale_per_channel = 1;
  g1.out = h; g1.ldo = ffn;
  g1.sx = sx1; g1.corr_t = ct1; g1.kp = kp1;
  e = h3::launch_gemm_i8(g1, st);
  if (e != cudaSuccess) return from_cuda(e, "fused_gated_mlp_w4a8: fc1");
  // fc2: ConvRot-quantize gelu(h); GEMM with dequant, correction and gated residual in the epilogue
  e = h3::launch_quantize_convrot(h, ffn, m, ffn, correction1 ? H3B200_ACT_NONE : H3B200_ACT_GELU_TANH, q2, xs2,
                                  correction2 ? sx2 : nullptr, group_size, kp2, st);
  if (e != cudaSuccess) return from_cuda(e, "fused_gated_mlp_w4a8: quantize gelu(h)");
  if (correction2) {
    e = h3::launch_correction_transpose(correction2, ng2, d, kp2, ct2, st);
    if (e != cudaSuccess) return from_cuda(e, "fused_gated_mlp_w4a8: fc2 correction layout");
  }
  h3::GemmArgs g2;
  g2.a = q2; g2.w = grid2; g2.m = m; g2.n = d; g2.k = ffn; g2.lda = ffn; g2.ldw = ffn;
  g2.epilogue = correction2 ? h3::kEpiGatedResidualCorr : h3::kEpiGatedResidual;
  g2.a_scale = xs2; g2.w_scale = s_channel2; g2.w_scale_per_channel = 1;
  g2.gate = gate; g2.residual = residual; g2.ldr = ldr;
  g2.out = out; g2.ldo = ldo;
  g2.sx = sx2; g2.corr_t = ct2; g2.kp = kp2;
  e = h3::launch_gemm_i8(g2, st);
  return from_cuda(e, "fused_gated_mlp_w4a8: fc2");
}
}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free INT8 linear.
//
// Some callers cannot allocate device memory for a call: a host runtime that
// hands this library only the input and output buffers it owns, or a serving
// loop that forbids allocation after start-up so that its memory use stays
// fixed. For them, h3b200_int8_linear_noalloc keeps the quantized activation
// (int8 [m, k]) and its row scales (fp32 [m]) in the static device array below
// instead of a caller workspace. Every GPU that loads this library holds the
// array until the process exits. All calls share it and it keeps the last
// call's contents; both parts are fully rewritten by every call, so nothing
// has to start at zero. Calls whose executions overlap on the GPU (different
// streams, or different host threads on one device) race on it.
// ---------------------------------------------------------------------------
namespace {

constexpr int64_t kNoAllocScratchBytes = 8ll << 20;  // 8 MiB per device
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {nullptr};

// Device address of the scratch array on the current device `device`. The first
// call on a device looks it up (cudaGetSymbolAddress, with that device current)
// and also fills the device's exact tanh-GELU table, which synchronises
// `stream` once; later calls use the cached address and launch only. Host code
// must never pass g_noalloc_scratch itself to a kernel: on the host that name is
// only a stand-in, not a device address.
cudaError_t noalloc_scratch(int device, cudaStream_t stream, void** out) {
  if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[device] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    if ((e = h3::ensure_act_table(H3B200_ACT_GELU_TANH, stream)) != cudaSuccess) return e;
    g_noalloc_ptr[device] = p;
  }
  *out = g_noalloc_ptr[device];
  return cudaSuccess;
}

}  // namespace

extern "C" {

int64_t h3b200_int8_linear_noalloc_max_scratch_bytes(void) { return kNoAllocScratchBytes; }

int h3b200_int8_linear_noalloc(const void* x, int64_t ldx, const int8_t* w, const float* w_scale,
                               int64_t w_scale_numel, const void* bias, int act, void* out, int64_t m, int64_t n,
                               int64_t k, h3b200_stream_t stream) {
  H3_GUARD("int8_linear_noalloc", stream);
  if (m < 0 || n < 0 || k < 0 || ldx < k) return fail(H3B200_ERR_INVALID, "int8_linear_noalloc: bad shape");
  if (act != H3B200_ACT_NONE && act != H3B200_ACT_GELU_TANH) return fail(H3B200_ERR_INVALID, "int8_linear_noalloc: unsupported act code %d", act);
  if (w_scale_numel != 1 && w_scale_numel != n) return fail(H3B200_ERR_INVALID, "int8_linear_noalloc: weight scale must be scalar or per-output-channel");
  if (m == 0 || n == 0) return H3B200_OK;
  if (!x || !w || !w_scale || !out) return fail(H3B200_ERR_INVALID, "int8_linear_noalloc: NULL pointer");
  if (k % 16 || n % 8) return fail(H3B200_ERR_UNSUPPORTED, "int8_linear_noalloc: needs k %% 16 == 0 and n %% 8 == 0");
  if (m > (1ll << 30) || k > (1ll << 30)) return fail(H3B200_ERR_INVALID, "int8_linear_noalloc: m or k too large");
  const int64_t q_bytes = round_up(m * k, 256);
  const int64_t need = q_bytes + m * 4;
  if (need > kNoAllocScratchBytes)
    return fail(H3B200_ERR_INVALID,
                "int8_linear_noalloc: m=%lld, k=%lld needs %lld bytes of scratch (int8 activations + fp32 row "
                "scales) but the static scratch holds %lld; split the rows or use h3b200_int8_linear",
                (long long)m, (long long)k, (long long)need, (long long)kNoAllocScratchBytes);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  void* base = nullptr;
  if (e == cudaSuccess) e = noalloc_scratch(dev, S(stream), &base);
  if (e != cudaSuccess) return from_cuda(e, "int8_linear_noalloc: scratch set-up");
  int8_t* xq = static_cast<int8_t*>(base);
  float* xs = reinterpret_cast<float*>(static_cast<unsigned char*>(base) + q_bytes);
  cudaStream_t st = S(stream);
  e = h3::launch_quantize_rows(x, ldx, m, k, act, nullptr, xq, xs, st);
  if (e != cudaSuccess) return from_cuda(e, "int8_linear_noalloc: quantize");
  h3::GemmArgs g;
  g.a = xq; g.w = w; g.m = m; g.n = n; g.k = k; g.lda = k; g.ldw = k;
  g.epilogue = h3::kEpiBF16; g.a_scale = xs; g.w_scale = w_scale; g.w_scale_per_channel = (w_scale_numel == n && n > 1) ? 1 : 0;
  g.bias = bias; g.out = out; g.ldo = n;
  return from_cuda(h3::launch_gemm_i8(g, st), "int8_linear_noalloc: gemm");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Tensor-parallel MLP communicator. Each rank owns one cudaMalloc'd region, exported
// through CUDA IPC and mapped by every other rank, laid out identically on all ranks:
//   flags   u32 [kTpMaxWorld]                      flag q: last barrier epoch from rank q
//   amax    u32 [2][world][max_rows]               slot q: rank q's fc1 row absmax (chunk parity)
//   recv    i32 [2][world][per_max][d]             slot q: rank q's fc2 partial rows owned here
//                                                  (compact: tp_local_row of the block-cyclic owner)
//   gather  bf16 [2][max_rows][d]                  finished rows of the other owners
// Chunk parity double-buffers every slot; the two barriers per chunk order each
// reuse after the last read of the same parity (see h3b200_tp_gated_mlp).
// ---------------------------------------------------------------------------
namespace {

struct TpHandle {
  char magic[8];
  int32_t rank, world;
  int64_t max_rows, d, ffn;
  uint64_t shared_bytes;
  cudaIpcMemHandle_t ipc;
};
static_assert(sizeof(TpHandle) <= H3B200_TP_HANDLE_BYTES, "TP handle does not fit H3B200_TP_HANDLE_BYTES");
constexpr char kTpMagic[8] = {'h', '3', 'b', '2', 'T', 'P', 'v', '1'};
constexpr unsigned long long kTpDefaultTimeoutNs = 5000000000ull;

struct TpComm {
  int rank = 0, world = 1, device = 0;
  bool linked_local = false;
  int64_t max_rows = 0, d = 0, ffn = 0, per_max = 0;
  unsigned long long timeout_ns = kTpDefaultTimeoutNs;
  uint8_t* shared = nullptr;
  size_t shared_bytes = 0, off_amax = 0, off_recv = 0, off_gather = 0;
  uint8_t* peer[h3::kTpMaxWorld] = {};
  bool ipc_open[h3::kTpMaxWorld] = {};
  uint8_t* work = nullptr;
  int8_t* xq = nullptr;
  float* xs = nullptr;
  uint32_t* amax = nullptr;
  unsigned int* ready = nullptr;
  void* a = nullptr;
  int8_t* q2 = nullptr;
  uint32_t epoch = 0;

  uint32_t* flags(int q) const { return reinterpret_cast<uint32_t*>(peer[q]); }
  uint32_t* amax_slot(int q, int parity, int slot) const {
    return reinterpret_cast<uint32_t*>(peer[q] + off_amax) + ((int64_t)parity * world + slot) * max_rows;
  }
  int32_t* recv_slot(int q, int parity, int slot) const {
    return reinterpret_cast<int32_t*>(peer[q] + off_recv) + ((int64_t)parity * world + slot) * per_max * d;
  }
  uint16_t* gather(int q, int parity) const {
    return reinterpret_cast<uint16_t*>(peer[q] + off_gather) + (int64_t)parity * max_rows * d;
  }
  bool connected() const {
    for (int q = 0; q < world; ++q)
      if (peer[q] == nullptr) return false;
    return true;
  }
};

void tp_release(TpComm* c) {
  for (int q = 0; q < h3::kTpMaxWorld; ++q)
    if (c->ipc_open[q]) cudaIpcCloseMemHandle(c->peer[q]);
  if (c->shared) cudaFree(c->shared);
  if (c->work) cudaFree(c->work);
  delete c;
}

int tp_barrier_impl(TpComm* c, cudaStream_t st) {
  if (c->world == 1 || c->linked_local) return H3B200_OK;
  ++c->epoch;
  h3::TpPtrs out{};
  for (int q = 0; q < c->world; ++q) out.p[q] = c->flags(q) + c->rank;
  return from_cuda(h3::launch_tp_barrier(out, c->flags(c->rank), c->world, c->epoch, c->timeout_ns, st), "tp_barrier");
}

int tp_stage_impl(TpComm* c, int stage, int64_t chunk, const void* x, int64_t ldx, const void* residual, int64_t ldr,
                  const void* gate, const int8_t* w1q, const float* s1, const int8_t* w2q, const float* s2, void* out,
                  int64_t ldo, int64_t lo, int64_t hi, cudaStream_t st) {
  const int64_t rows = hi - lo, d = c->d, ffn = c->ffn;
  const int parity = (int)(chunk & 1), me = c->rank, W = c->world;
  cudaError_t e = cudaSuccess;
  switch (stage) {
    case 1: {  // quantize x, fc1 + GELU + row absmax, absmax into every rank's slot
      e = h3::launch_quantize_rows(static_cast<const uint16_t*>(x) + lo * ldx, ldx, rows, d, H3B200_ACT_NONE, nullptr,
                                   c->xq, c->xs, st);
      if (e != cudaSuccess) return from_cuda(e, "tp_stage 1: quantize x");
      const int64_t zero_bytes = reinterpret_cast<uint8_t*>(c->ready + h3::requant_ready_count(rows)) -
                                 reinterpret_cast<uint8_t*>(c->amax);
      if ((e = cudaMemsetAsync(c->amax, 0, (size_t)zero_bytes, st)) != cudaSuccess) return from_cuda(e, "tp_stage 1: memset");
      h3::GemmArgs g1;
      g1.a = c->xq; g1.w = w1q; g1.m = rows; g1.n = ffn; g1.k = d; g1.lda = d; g1.ldw = d;
      g1.epilogue = h3::kEpiGeluAbsmax; g1.a_scale = c->xs; g1.w_scale = s1; g1.w_scale_per_channel = 1;
      g1.out = c->a; g1.ldo = ffn; g1.row_absmax = reinterpret_cast<float*>(c->amax);
      if ((e = h3::launch_gemm_i8(g1, st)) != cudaSuccess) return from_cuda(e, "tp_stage 1: fc1");
      if (W > 1) {
        h3::TpPtrs dst{};
        for (int q = 0; q < W; ++q) dst.p[q] = c->amax_slot(q, parity, me);
        e = h3::launch_tp_push_u32(c->amax, rows, dst, W, st);
      }
      return from_cuda(e, "tp_stage 1: absmax push");
    }
    case 2: {  // global absmax, fc2 (own requant) with every int32 row stored at its owner
      if (W > 1 && (e = h3::launch_tp_max_u32(c->amax_slot(me, parity, 0), c->max_rows, W, rows, c->amax, st)) != cudaSuccess)
        return from_cuda(e, "tp_stage 2: absmax max");
      h3::GemmArgs g2;
      g2.a = c->q2; g2.w = w2q; g2.m = rows; g2.n = d; g2.k = ffn; g2.lda = ffn; g2.ldw = ffn;
      g2.epilogue = h3::kEpiI32;
      g2.requant_src = c->a; g2.requant_lds = ffn; g2.requant_ready = c->ready;
      g2.row_absmax = reinterpret_cast<float*>(c->amax);
      g2.out = c->recv_slot(me, parity, me); g2.ldo = d;
      g2.peer_world = W;
      for (int q = 0; q < W; ++q) g2.peer_out[q] = c->recv_slot(q, parity, me);
      return from_cuda(h3::launch_gemm_i8(g2, st), "tp_stage 2: fc2 (requant, rows to their owners)");
    }
    case 3: {  // this rank's rows: sum of partials, dequant + gated residual, rows to every rank
      h3::TpPtrs g{};
      for (int q = 0; q < W; ++q)
        if (q != me) g.p[q] = c->gather(q, parity);
      e = h3::launch_tp_finish(c->recv_slot(me, parity, 0), c->per_max * d, W, me, rows, d, c->amax, s2, gate,
                               static_cast<const uint16_t*>(residual) + lo * ldr, ldr,
                               static_cast<uint16_t*>(out) + lo * ldo, ldo, g, st);
      return from_cuda(e, "tp_stage 3: owner rows");
    }
    case 4:  // the other owners' rows of this chunk, from the gather buffer into out
      return from_cuda(h3::launch_tp_gather_rows(c->gather(me, parity), W, me, rows, d,
                                                 static_cast<uint16_t*>(out) + lo * ldo, ldo, st),
                       "tp_stage 4: gathered rows");
    default:
      return fail(H3B200_ERR_INVALID, "tp_stage: stage must be 1..4, got %d", stage);
  }
}

int tp_check_args(const char* what, TpComm* c, const void* x, int64_t ldx, const void* residual, int64_t ldr,
                  const void* gate, const int8_t* w1q, const float* s1, const int8_t* w2q, const float* s2,
                  const void* out, int64_t ldo) {
  if (c == nullptr) return fail(H3B200_ERR_INVALID, "%s: NULL communicator", what);
  if (!c->connected()) return fail(H3B200_ERR_INVALID, "%s: communicator not connected (h3b200_tp_comm_open or h3b200_tp_comm_link_local first)", what);
  int dev = -1;
  cudaGetDevice(&dev);
  if (dev != c->device) return fail(H3B200_ERR_INVALID, "%s: current device %d is not the communicator's device %d", what, dev, c->device);
  if (!x || !residual || !gate || !w1q || !s1 || !w2q || !s2 || !out) return fail(H3B200_ERR_INVALID, "%s: NULL pointer", what);
  if (ldx < c->d || ldr < c->d || ldo < c->d || ldr % 8 || ldo % 8)
    return fail(H3B200_ERR_INVALID, "%s: row strides must be >= d (residual and out: multiples of 8 elements)", what);
  if ((reinterpret_cast<uintptr_t>(residual) & 15) || (reinterpret_cast<uintptr_t>(out) & 15) ||
      (reinterpret_cast<uintptr_t>(gate) & 15) || (reinterpret_cast<uintptr_t>(w1q) & 15) ||
      (reinterpret_cast<uintptr_t>(w2q) & 15))
    return fail(H3B200_ERR_UNSUPPORTED, "%s: residual, out, gate and weights must be 16-byte aligned", what);
  return H3B200_OK;
}

}  // namespace

extern "C" {

int h3b200_tp_comm_create(int rank, int world, int64_t max_rows, int64_t d, int64_t ffn_shard,
                          int64_t barrier_timeout_ns, void** comm, uint8_t* handle) {
  if (comm == nullptr || handle == nullptr) return fail(H3B200_ERR_INVALID, "tp_comm_create: NULL output");
  *comm = nullptr;
  if (world < 1 || world > h3::kTpMaxWorld || rank < 0 || rank >= world)
    return fail(H3B200_ERR_INVALID, "tp_comm_create: rank %d of world %d (1..%d ranks)", rank, world, h3::kTpMaxWorld);
  if (max_rows <= 0 || d <= 0 || ffn_shard <= 0 || d % 16 || ffn_shard % 16 || max_rows > (1ll << 24))
    return fail(H3B200_ERR_INVALID, "tp_comm_create: needs 0 < max_rows <= 2^24 and d, ffn_shard positive multiples of 16");
  if (barrier_timeout_ns < 0) return fail(H3B200_ERR_INVALID, "tp_comm_create: negative barrier timeout");
  TpComm* c = new TpComm();
  c->rank = rank;
  c->world = world;
  c->max_rows = max_rows;
  c->d = d;
  c->ffn = ffn_shard;
  c->per_max = h3::tp_owned_span(max_rows, world, 0);  // rank 0 owns the most rows
  c->timeout_ns = barrier_timeout_ns > 0 ? (unsigned long long)barrier_timeout_ns : kTpDefaultTimeoutNs;
  cudaError_t e = cudaGetDevice(&c->device);
  size_t off = 256;  // flags
  c->off_amax = off;
  off += (size_t)round_up(2 * world * max_rows * 4, 256);
  c->off_recv = off;
  off += (size_t)round_up(2 * world * c->per_max * d * 4, 256);
  c->off_gather = off;
  off += (size_t)round_up(2 * max_rows * d * 2, 256);
  c->shared_bytes = off;
  if (e == cudaSuccess) e = cudaMalloc(&c->shared, c->shared_bytes);
  if (e == cudaSuccess) e = cudaMemset(c->shared, 0, c->shared_bytes);
  const int64_t work_bytes = round_up(max_rows * d, 256) + round_up(max_rows * 4, 256) +
                             round_up((max_rows + h3::requant_ready_count(max_rows)) * 4, 256) +
                             round_up(max_rows * ffn_shard * 2, 256) + round_up(max_rows * ffn_shard, 256) + 1024;
  if (e == cudaSuccess) e = cudaMalloc(&c->work, (size_t)work_bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();  // flags are zero before any rank can map them
  if (e != cudaSuccess) {
    tp_release(c);
    return from_cuda(e, "tp_comm_create");
  }
  Carver w{c->work, work_bytes};
  c->xq = static_cast<int8_t*>(w.take(max_rows * d));
  c->xs = static_cast<float*>(w.take(max_rows * 4));
  c->amax = static_cast<uint32_t*>(w.take((max_rows + h3::requant_ready_count(max_rows)) * 4));
  c->ready = reinterpret_cast<unsigned int*>(c->amax + max_rows);  // the requant counters follow the absmax
  c->a = w.take(max_rows * ffn_shard * 2);
  c->q2 = static_cast<int8_t*>(w.take(max_rows * ffn_shard));
  if (!w.ok) {
    tp_release(c);
    return fail(H3B200_ERR_INVALID, "tp_comm_create: internal workspace layout");
  }
  c->peer[rank] = c->shared;
  TpHandle h;
  memset(&h, 0, sizeof(h));
  memcpy(h.magic, kTpMagic, sizeof(kTpMagic));
  h.rank = rank;
  h.world = world;
  h.max_rows = max_rows;
  h.d = d;
  h.ffn = ffn_shard;
  h.shared_bytes = c->shared_bytes;
  if (world > 1 && (e = cudaIpcGetMemHandle(&h.ipc, c->shared)) != cudaSuccess) {
    tp_release(c);
    return from_cuda(e, "tp_comm_create: cudaIpcGetMemHandle");
  }
  memset(handle, 0, H3B200_TP_HANDLE_BYTES);
  memcpy(handle, &h, sizeof(h));
  *comm = c;
  return H3B200_OK;
}

int h3b200_tp_comm_open(void* comm, const uint8_t* handles) {
  TpComm* c = static_cast<TpComm*>(comm);
  if (c == nullptr || handles == nullptr) return fail(H3B200_ERR_INVALID, "tp_comm_open: NULL argument");
  if (c->linked_local) return fail(H3B200_ERR_INVALID, "tp_comm_open: communicator is linked locally");
  TpHandle hs[h3::kTpMaxWorld];
  for (int q = 0; q < c->world; ++q) {
    memcpy(&hs[q], handles + (size_t)q * H3B200_TP_HANDLE_BYTES, sizeof(TpHandle));
    const TpHandle& h = hs[q];
    if (memcmp(h.magic, kTpMagic, sizeof(kTpMagic)) != 0 || h.rank != q || h.world != c->world ||
        h.max_rows != c->max_rows || h.d != c->d || h.ffn != c->ffn || h.shared_bytes != c->shared_bytes)
      return fail(H3B200_ERR_INVALID, "tp_comm_open: handle %d does not match this communicator (rank order, world, max_rows, d, ffn_shard)", q);
    if (q != c->rank && c->ipc_open[q]) return fail(H3B200_ERR_INVALID, "tp_comm_open: already open");
  }
  int dev = -1;
  cudaGetDevice(&dev);
  if (dev != c->device) return fail(H3B200_ERR_INVALID, "tp_comm_open: current device %d is not the communicator's device %d", dev, c->device);
  for (int q = 0; q < c->world; ++q) {
    if (q == c->rank) continue;
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, hs[q].ipc, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int r = 0; r < c->world; ++r)
        if (c->ipc_open[r]) {
          cudaIpcCloseMemHandle(c->peer[r]);
          c->ipc_open[r] = false;
          c->peer[r] = nullptr;
        }
      return from_cuda(e, "tp_comm_open: cudaIpcOpenMemHandle");
    }
    c->peer[q] = static_cast<uint8_t*>(p);
    c->ipc_open[q] = true;
  }
  return H3B200_OK;
}

int h3b200_tp_comm_link_local(void* const* comms, int world) {
  if (comms == nullptr || world < 1 || world > h3::kTpMaxWorld) return fail(H3B200_ERR_INVALID, "tp_comm_link_local: bad arguments");
  TpComm* cs[h3::kTpMaxWorld];
  for (int q = 0; q < world; ++q) {
    cs[q] = static_cast<TpComm*>(comms[q]);
    if (cs[q] == nullptr || cs[q]->world != world || cs[q]->rank != q || cs[q]->max_rows != cs[0]->max_rows ||
        cs[q]->d != cs[0]->d || cs[q]->ffn != cs[0]->ffn || cs[q]->device != cs[0]->device)
      return fail(H3B200_ERR_INVALID, "tp_comm_link_local: communicator %d is not rank %d of the same group on the same device", q, q);
    for (int r = 0; r < world; ++r)
      if (cs[q]->ipc_open[r]) return fail(H3B200_ERR_INVALID, "tp_comm_link_local: communicator %d is IPC-connected", q);
  }
  for (int q = 0; q < world; ++q) {
    for (int r = 0; r < world; ++r) cs[q]->peer[r] = cs[r]->shared;
    cs[q]->linked_local = true;
  }
  return H3B200_OK;
}

int h3b200_tp_comm_destroy(void* comm) {
  if (comm != nullptr) tp_release(static_cast<TpComm*>(comm));
  return H3B200_OK;
}

int h3b200_tp_barrier(void* comm, h3b200_stream_t stream) {
  H3_GUARD("tp_barrier", stream);
  TpComm* c = static_cast<TpComm*>(comm);
  if (c == nullptr || !c->connected()) return fail(H3B200_ERR_INVALID, "tp_barrier: communicator not connected");
  return tp_barrier_impl(c, S(stream));
}

int h3b200_tp_stage(void* comm, int stage, int64_t chunk, const void* x, int64_t ldx, const void* residual,
                    int64_t ldr, const void* gate, const int8_t* w1q, const float* s1, const int8_t* w2q,
                    const float* s2, void* out, int64_t ldo, int64_t lo, int64_t hi, h3b200_stream_t stream) {
  H3_GUARD("tp_stage", stream);
  TpComm* c = static_cast<TpComm*>(comm);
  if (const int rc = tp_check_args("tp_stage", c, x, ldx, residual, ldr, gate, w1q, s1, w2q, s2, out, ldo)) return rc;
  if (chunk < 0 || lo < 0 || hi <= lo || hi - lo > c->max_rows)
    return fail(H3B200_ERR_INVALID, "tp_stage: chunk rows [%lld, %lld) must be non-empty and at most max_rows", (long long)lo, (long long)hi);
  return tp_stage_impl(c, stage, chunk, x, ldx, residual, ldr, gate, w1q, s1, w2q, s2, out, ldo, lo, hi, S(stream));
}

int h3b200_tp_gated_mlp(void* comm, const void* x, int64_t ldx, const void* residual, int64_t ldr, const void* gate,
                        const int8_t* w1q, const float* s1, const int8_t* w2q, const float* s2, void* out,
                        int64_t ldo, int64_t m, int64_t chunk_rows, h3b200_stream_t stream) {
  H3_GUARD("tp_gated_mlp", stream);
  TpComm* c = static_cast<TpComm*>(comm);
  if (m < 0) return fail(H3B200_ERR_INVALID, "tp_gated_mlp: m < 0");
  if (m == 0) return H3B200_OK;
  if (const int rc = tp_check_args("tp_gated_mlp", c, x, ldx, residual, ldr, gate, w1q, s1, w2q, s2, out, ldo)) return rc;
  if (c->linked_local) return fail(H3B200_ERR_UNSUPPORTED, "tp_gated_mlp: locally linked communicators run stage by stage (h3b200_tp_stage)");
  const int64_t chunk = chunk_rows > 0 ? std::min(chunk_rows, c->max_rows) : c->max_rows;
  const cudaStream_t st = S(stream);
  int rc = H3B200_OK;
  int64_t prev_lo = 0, prev_hi = 0;
  for (int64_t i = 0, lo = 0; lo < m; ++i, lo += chunk) {
    const int64_t hi = std::min(m, lo + chunk);
    // barrier A(i): every rank's owner rows of chunk i-1 are in the gather buffers
    if ((rc = tp_stage_impl(c, 1, i, x, ldx, residual, ldr, gate, w1q, s1, w2q, s2, out, ldo, lo, hi, st)) ||
        (rc = tp_barrier_impl(c, st)))
      return rc;
    if (i > 0 && (rc = tp_stage_impl(c, 4, i - 1, x, ldx, residual, ldr, gate, w1q, s1, w2q, s2, out, ldo, prev_lo,
                                     prev_hi, st)))
      return rc;
    // barrier B(i): every rank's fc2 rows of chunk i are in their owners' receive slots
    if ((rc = tp_stage_impl(c, 2, i, x, ldx, residual, ldr, gate, w1q, s1, w2q, s2, out, ldo, lo, hi, st)) ||
        (rc = tp_barrier_impl(c, st)) ||
        (rc = tp_stage_impl(c, 3, i, x, ldx, residual, ldr, gate, w1q, s1, w2q, s2, out, ldo, lo, hi, st)))
      return rc;
    prev_lo = lo;
    prev_hi = hi;
  }
  const int64_t last = (m + chunk - 1) / chunk - 1;
  if ((rc = tp_barrier_impl(c, st))) return rc;
  return tp_stage_impl(c, 4, last, x, ldx, residual, ldr, gate, w1q, s1, w2q, s2, out, ldo, prev_lo, prev_hi, st);
}

}  // extern "C"

