// Internal launchers shared between the kernel files and the C-ABI layer.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace h3 {

// Epilogue variants of the tcgen05 INT8 GEMM.
enum GemmEpilogue : int {
  kEpiI32 = 0,             // raw int32 accumulators
  kEpiBF16 = 1,            // bf16(acc * (xs * ws)) (+ bf16 bias)
  kEpiGeluAbsmax = 2,      // a = gelu(bf16(acc * (xs * ws))) stored bf16, row absmax of |a| via atomicMax
  kEpiGatedResidual = 3,   // out = bf16(residual + y * gate), y = bf16(acc * (xs * ws)) (+ bias, rounded)
  // W4A8 linears with the asymmetric correction fused into the INT8 GEMM:
  //   y = bf16(bf16(acc * (xs * ws)) + sum_g sx[m, g] * corr_t[n, g])   (fp32 sum, one rounding)
  kEpiBF16Corr = 4,          // out = y
  kEpiBF16CorrGelu = 5,      // out = tanh-GELU(y) (exact bf16)
  kEpiGatedResidualCorr = 6, // out = bf16(residual + y * gate)
  // Q/K/V projection into attention layouts: y = bf16(bf16(acc * (xs * ws)) + bias);
  // Q and K heads get per-head RMSNorm and partial split-half RoPE, V is stored as is.
  kEpiQKV = 7,
  // kEpiSwiGLU: W holds n = 2 f rows, gate rows [0, f) then up rows [f, 2 f);
  // out [m, f] = bf16(silu(g) * u) with g, u = bf16(acc * (xs * ws)) (+ bf16 bias,
  // rounded), the reference's fc1 -> silu(gate).mul_(up) in one pass
  kEpiSwiGLU = 8,
  // internal: kEpiGatedResidual whose A operand the kernel quantizes itself
  // (GemmArgs::requant_src); chosen by launch_gemm_i8, not by callers
  kEpiGatedResidualRq = 9,
  // internal: kEpiI32 on an A operand the kernel quantizes itself (requant_src set)
  kEpiI32Rq = 10,
};

// Largest tensor-parallel group whose int32 rows one GEMM routes to their owners.
constexpr int kTpMaxWorld = 8;
// Row ownership in the tensor-parallel MLP: blocks of kTpBlockRows rows go round-robin
// over the ranks (block b belongs to rank b % world), so the two CTAs of a 256-row GEMM
// tile write to different owners and the NVLink traffic of the routed rows spreads over
// the whole GEMM. An owner keeps its rows compact: block b is its local block b / world.
constexpr int kTpBlockRows = 128;
__host__ __device__ inline int tp_owner(int64_t row, int world) { return (int)((row / kTpBlockRows) % world); }
__host__ __device__ inline int64_t tp_local_row(int64_t row, int world) {
  return (row / kTpBlockRows / world) * kTpBlockRows + row % kTpBlockRows;
}
// rows [0, tp_owned_span(c, world, o)) of owner o's compact buffer cover its rows of a
// c-row chunk (the last block may be partial; local rows past it map to rows >= c)
__host__ __device__ inline int64_t tp_owned_span(int64_t c, int world, int o) {
  const int64_t nb = (c + kTpBlockRows - 1) / kTpBlockRows;
  return (o < nb ? (nb - o + world - 1) / world : 0) * kTpBlockRows;
}
__host__ __device__ inline int64_t tp_chunk_row(int64_t local, int world, int o) {
  return ((local / kTpBlockRows) * world + o) * kTpBlockRows + local % kTpBlockRows;
}

struct GemmArgs {
  const int8_t* a = nullptr;  // [m, k] int8, row stride lda bytes
  const int8_t* w = nullptr;  // [n, k] int8, row stride ldw bytes
  int64_t m = 0, n = 0, k = 0;
  int64_t lda = 0, ldw = 0;
  int epilogue = kEpiBF16;
  const float* a_scale = nullptr;  // [m]
  const float* w_scale = nullptr;  // [n] or [1]
  int w_scale_per_channel = 1;
  const void* bias = nullptr;      // bf16 [n]
  const void* gate = nullptr;      // bf16 [n], or [rows, ldg] with row_map
  const int32_t* row_map = nullptr;  // kEpiGatedResidual: gate row of each output row [m] (modulation segments)
  int64_t ldg = 0;
  const void* residual = nullptr;  // bf16 [m, ldr]
  int64_t ldr = 0;
  void* out = nullptr;  // bf16 or int32 [m, ldo]
  int64_t ldo = 0;
  float* row_absmax = nullptr;              // fp32 [m], must start at 0 (values are non-negative)
  // W4A8 correction operands (kEpi*Corr): sx bf16 [m, kp], corr_t bf16 [n, kp],
  // both zero for group index >= groups; kp a multiple of 64, at most 128.
  const void* sx = nullptr;
  const void* corr_t = nullptr;
  int64_t kp = 0;
  // kEpiQKV: GEMM column c is dim c % 128 of head (c % inner) / 128 of section
  // sec0 + c / inner (0 Q, 1 K, 2 V), inner = heads * 128. Section s writes
  // [m, heads, 128] bf16 at qkv_out[s] with element strides token qkv_st[s] and
  // head qkv_sh[s] (16-byte multiples). qk_w: bf16 [128] RMSNorm weights of Q and
  // K; rope_t: the rotation rows transposed to [qkv_rot / 2][m] x {t00, t01, t10, t11}
  // fp32 (nullptr: RMSNorm only); qkv_rot a multiple of 32, at most 128.
  int64_t qkv_heads = 0;
  int qkv_sec0 = 0;
  int qkv_rot = 0;
  void* qkv_out[3] = {nullptr, nullptr, nullptr};
  int64_t qkv_st[3] = {0, 0, 0}, qkv_sh[3] = {0, 0, 0};
  const void* qk_w[2] = {nullptr, nullptr};
  const float4* rope_t = nullptr;
  float qk_eps = 1e-6f;
  // kEpiGatedResidual with requant_src set: A is not an input but is produced by the
  // same kernel. Its rows are quantize_int8_rowwise of the bf16 rows requant_src
  // [m, k] (row stride requant_lds) with the row absmax given in row_absmax (fc1's
  // epilogue atomics), written into a (lda == k); requant_ready holds one counter per
  // block of tile rows and must be zero at launch. a_scale is not read: the epilogue
  // takes the row scale from row_absmax.
  const void* requant_src = nullptr;
  int64_t requant_lds = 0;
  unsigned int* requant_ready = nullptr;
  // kEpiI32 with peer_world > 0: output row r goes to its owner's buffer
  // peer_out[tp_owner(r, peer_world)] at row tp_local_row(r, peer_world) (row stride
  // ldo), instead of to out. The destinations may be other GPUs' memory (peer-mapped):
  // the epilogue writes them with plain 16-byte stores, published by a stream-ordered
  // cross-GPU barrier after the kernel (a system-scope release).
  int32_t* peer_out[kTpMaxWorld] = {};
  int peer_world = 0;
  // kEpiBF16 only: out and bias are fp16 (y = fp16(acc * (xs * ws)), + bias in fp16)
  int out_f16 = 0;
};

// One pointer per rank of a tensor-parallel group (by value in kernel parameters).
struct TpPtrs {
  void* p[kTpMaxWorld];
};

// Tensor-parallel MLP exchange kernels (tp.cu); see that file for the protocol.
cudaError_t launch_tp_push_u32(const uint32_t* src, int64_t n, const TpPtrs& dst, int ndst, cudaStream_t stream);
cudaError_t launch_tp_barrier(const TpPtrs& flag_out, const uint32_t* my_flags, int world, uint32_t epoch,
                              unsigned long long timeout_ns, cudaStream_t stream);
cudaError_t launch_tp_max_u32(const uint32_t* slots, int64_t stride, int world, int64_t n, uint32_t* out,
                              cudaStream_t stream);
cudaError_t launch_tp_finish(const int32_t* recv, int64_t slot, int world, int owner, int64_t rows, int64_t n,
                             const uint32_t* absmax, const float* ws, const void* gate, const void* residual,
                             int64_t ldr, void* out, int64_t ldo, const TpPtrs& gather, cudaStream_t stream);
cudaError_t launch_tp_gather_rows(const void* gather, int world, int owner, int64_t rows, int64_t n, void* out,
                                  int64_t ldo, cudaStream_t stream);

// 32-bit words requant_ready needs for m rows: one counter per 128-row block (enough
// for both tile shapes), then the progress word of the tiles.
inline int64_t requant_ready_count(int64_t m) { return (m + 127) / 128 + 1; }

// rope_t[p, t] = {t00, t01, t10, t11} of pair p < pairs of token t, fp32, from
// table rows [pairs, 2, 2] at element stride fs_t (table dtype 0 fp32, 1 bf16, 2 fp16)
cudaError_t launch_rope_table_transpose(const void* freqs, int table_dtype, int64_t fs_t, int64_t m, int pairs,
                                        float4* rope_t, cudaStream_t stream);

cudaError_t launch_dequant_gated_residual(const int32_t* acc, const float* xs, const float* ws, const void* gate,
                                          const void* residual, int64_t ldr, void* out, int64_t ldo, int64_t m,
                                          int64_t n, cudaStream_t stream);
cudaError_t launch_apply_act(const void* x, void* y, int64_t n, int act, cudaStream_t stream);
// Row quantizer of the activated row (width k; for act = SwiGLU the raw row is
// [gate | up], 2 k wide, at stride ldx >= 2 k).
cudaError_t launch_quantize_rows(const void* x, int64_t ldx, int64_t m, int64_t k, int act, const float* absmax_in,
                                 int8_t* q, float* scale, cudaStream_t stream);

// Row quantizer of fp16 rows (no input activation): the reference's fp16 semantics (quantize.cu).
cudaError_t launch_quantize_rows_f16(const void* x, int64_t ldx, int64_t m, int64_t k, int8_t* q, float* scale,
                                     cudaStream_t stream);

// Stochastic rounding (seed > 0): the reference CUDA kernel's counter-based noise added
// to the bf16 quotient, then floor (quantize.cu).
cudaError_t launch_quantize_rows_stochastic(const void* x, int64_t ldx, int64_t m, int64_t k, int act,
                                            uint64_t seed, int8_t* q, float* scale, cudaStream_t stream);

// Returns cudaErrorNotSupported when the shape is outside the kernel's contract.
cudaError_t launch_gemm_i8(const GemmArgs& args, cudaStream_t stream);

// Small-M W4A8 linear with the int4 weight unpacked in shared memory (gemm_w4.cu):
// xq int8 [m, k] (contiguous), xs fp32 [m]; qdata packed [n, k / 2]; s_rel fp32 or
// fp8-e4m3 [n, k / group]; codebook 16 fp32 levels or null; s_channel fp32 [n];
// bias bf16 [n] or null; sx bf16 [m, kp] and corr bf16 [k / group, n] (both or neither);
// out bf16 [m, ldo].
struct W4SmallMArgs {
  const int8_t* xq = nullptr;
  const float* xs = nullptr;
  const uint8_t* qdata = nullptr;
  const void* s_rel = nullptr;
  bool s_rel_e4m3 = false;
  const float* codebook = nullptr;
  const float* s_channel = nullptr;
  const void* bias = nullptr;
  const void* sx = nullptr;
  int64_t kp = 0;
  const void* corr = nullptr;
  void* out = nullptr;
  int64_t ldo = 0;
  int64_t m = 0, n = 0, k = 0, group = 0;
  // split-K over `splits` CTAs per tile (gemm_w4_smallm_splits): acc_ws int32 [m, n] and
  // tile_cnt [tiles] must be zero at launch
  int64_t splits = 1;
  int32_t* acc_ws = nullptr;
  unsigned int* tile_cnt = nullptr;
};
bool gemm_w4_smallm_supported(int64_t m, int64_t n, int64_t k, int64_t group, int64_t groups_corr);
int gemm_w4_smallm_splits(int64_t m, int64_t n, int64_t k, int sms);
cudaError_t launch_gemm_w4_smallm(const W4SmallMArgs& args, cudaStream_t stream);

struct NormRopeArgs {
  const void* q = nullptr;
  const void* k = nullptr;
  void* q_out = nullptr;
  void* k_out = nullptr;
  int64_t ldq = 0, ldk = 0, ldqo = 0, ldko = 0;
  const float* freqs = nullptr;
  const void* q_weight = nullptr;
  const void* k_weight = nullptr;
  const void* scale = nullptr;
  const void* shift = nullptr;
  // Per-token modulation rows (row span only): with row_map (int32 [m]), tokens_per_row > 0 or
  // mod_rows > 1, token t uses row row_map[t] (clamped) or t / tokens_per_row of scale / shift
  // at row strides lds / ldh; otherwise scale / shift are one row.
  const int32_t* row_map = nullptr;
  int64_t tokens_per_row = 0, mod_rows = 1, lds = 0, ldh = 0;
  int64_t m = 0, heads = 0, head_dim = 0, rot_dim = 0;
  int norm_span = 0;
  float eps = 1e-6f;
};
cudaError_t launch_adaln_rms_rope(const NormRopeArgs& a, cudaStream_t stream);

// Per-head RMSNorm + partial split-half RoPE over strided [m, heads, 128] bf16
// views (x[t] -> y[t], t < tensors; in place when x == y). Table rows
// [rot/2, 2, 2] of fp32 (0), bf16 (1) or fp16 (2) at token stride fs_t and
// head stride fs_h (0: one row per token) in elements.
struct QKNormRopeArgs {
  const void* x[2] = {nullptr, nullptr};
  void* y[2] = {nullptr, nullptr};
  const void* w[2] = {nullptr, nullptr};
  int64_t xs_t[2] = {0, 0}, xs_h[2] = {0, 0}, ys_t[2] = {0, 0}, ys_h[2] = {0, 0};
  const void* freqs = nullptr;
  int table_dtype = 0;
  int64_t fs_t = 0, fs_h = 0;
  int64_t m = 0, heads = 0, head_dim = 128, rot_dim = 0;
  int tensors = 1;
  float eps = 1e-6f;
};
cudaError_t launch_qk_rms_rope(const QKNormRopeArgs& a, cudaStream_t stream);
// y[t, h, :] = x[t, h, :] over strided [m, heads, 128] bf16 views
cudaError_t launch_copy_heads(const void* x, int64_t xs_t, int64_t xs_h, void* y, int64_t ys_t, int64_t ys_h,
                              int64_t m, int64_t heads, cudaStream_t stream);

// int4 -> int8 grid; s_rel fp32 or (s_rel_e4m3) fp8-e4m3 bytes; codebook: 16 fp32 levels or nullptr (u - 8)
cudaError_t launch_dequant_int4(const int8_t* qdata, const void* s_rel, bool s_rel_e4m3, const float* codebook,
                                int64_t n, int64_t k, int64_t group, int8_t* out, cudaStream_t stream);
// ConvRot-256 + row quantization with the rotation correctly rounded (convrot.cu);
// with sx != nullptr also writes the correction operand sx (bf16 [m, kp], zero
// beyond k / sum_group). k a multiple of 256, at most convrot_max_k(act).
int64_t convrot_max_k(int act);
cudaError_t launch_quantize_convrot(const void* x, int64_t ldx, int64_t m, int64_t k, int act, int8_t* q,
                                    float* scale, void* sx, int64_t sum_group, int64_t kp, cudaStream_t stream);
// corr_t[n, kp] (bf16) = correction[g, n] transposed, zero for g >= groups
cudaError_t launch_correction_transpose(const void* corr, int64_t groups, int64_t n, int64_t kp, void* corr_t,
                                        cudaStream_t stream);
// K padding of the correction operands: groups rounded up to 64 (one 128-byte bf16 k-block)
inline int64_t correction_kpad(int64_t groups) { return (groups + 63) / 64 * 64; }

int num_sms(int device);

// Fills the device's exact bf16 tanh-GELU table on first use (once per device,
// synchronously on `stream`); cudaErrorStreamCaptureUnsupported if that first
// use happens inside a stream capture.
cudaError_t ensure_gelu_table(cudaStream_t stream);
// The same for the table of `act` (GELU or SiLU; no-op for other codes).
cudaError_t ensure_act_table(int act, cudaStream_t stream);

// Standalone RMS-AdaLN (adaln.cu): y = bf16(bf16(bf16((x * rstd) * w) * bf16(1 + scale[r])) + shift[r]),
// r = row_map[t] (clamped to [0, rows)), else t / tokens_per_row (<= 0: 0). weight may be nullptr
// (no affine weight); scale == shift == nullptr is a plain RMSNorm. y may alias x.
struct RmsAdalnArgs {
  const void* x = nullptr;
  int64_t ldx = 0;
  void* y = nullptr;
  int64_t ldy = 0;
  const void* weight = nullptr;
  const void* scale = nullptr;
  int64_t lds = 0;
  const void* shift = nullptr;
  int64_t ldh = 0;
  const int32_t* row_map = nullptr;
  int64_t tokens_per_row = 0;
  int64_t rows = 0;
  int64_t m = 0, d = 0;
  float eps = 1e-6f;
};
cudaError_t launch_rms_adaln(const RmsAdalnArgs& a, cudaStream_t stream);
// y[m, k] = silu(x[:, :k]) * x[:, k:2k] per row (bf16)
cudaError_t launch_swiglu_rows(const void* x, int64_t ldx, void* y, int64_t ldy, int64_t m, int64_t k,
                               cudaStream_t stream);

// 2-D tiled TMA descriptor (no interleave, 256-byte L2 promotion, no OOB fill);
// false when the driver's encoder is unavailable or rejects the layout.
bool encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t rows,
                    uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swizzle);

}  // namespace h3
