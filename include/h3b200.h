/*
 * h3b200 -- B200-native (sm_100a) kernels for X-MinimaxH3's quantized DiT-block
 * hot path, exported through a plain C ABI.
 *
 * Conventions (mirroring comfy_kitchen's CUDA backend launchers):
 *  - Pointers are device pointers unless stated; the caller allocates every
 *    output and workspace. Nothing here frees or keeps caller memory.
 *  - Launches are asynchronous on `stream` (a cudaStream_t, e.g. torch's
 *    current stream). No entry point synchronises the device except
 *    h3b200_device_status().
 *  - bf16 tensors are 16-bit storage; int8 tensors are signed bytes.
 *  - Every entry point returns an int status (H3B200_OK on success). A
 *    non-zero status leaves a message in h3b200_last_error(). No C++
 *    exception crosses this boundary and nothing falls back to another path.
 *  - Every wait inside a kernel is bounded. A wait that expires records a code
 *    in the device status word and in a mapped host copy of it; from then on
 *    every launching entry point on that device returns H3B200_ERR_DEVICE
 *    without launching, until h3b200_device_status(device, &s, 1) clears it.
 *    Errors are reported asynchronously, like CUDA's: calls queued before the
 *    failure became visible return H3B200_OK but their outputs are not valid.
 *    The host copy is set up by the first call on each device that is not
 *    made under stream capture.
 *  - Activation codes follow comfy_kitchen backends/cuda/input_act_codes.h:13
 *    (0 none, 1 gelu_tanh, 2 swiglu); dtype codes follow eager/quantization.py:34-40
 *    (0 fp32, 1 fp16, 2 bf16).
 */
#ifndef H3B200_H_
#define H3B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define H3B200_API __attribute__((visibility("default")))
#else
#define H3B200_API
#endif

typedef void* h3b200_stream_t; /* cudaStream_t */

enum {
  H3B200_OK = 0,
  H3B200_ERR_INVALID = 1,     /* shape / stride / alignment / code outside the contract */
  H3B200_ERR_UNSUPPORTED = 2, /* valid request this build does not implement */
  H3B200_ERR_LAUNCH = 3,      /* CUDA runtime error at launch */
  H3B200_ERR_DEVICE = 4       /* a kernel recorded a device-side failure (bounded wait expired); refused until cleared */
};

enum { H3B200_ACT_NONE = 0, H3B200_ACT_GELU_TANH = 1, H3B200_ACT_SWIGLU = 2 };
enum { H3B200_DTYPE_F32 = 0, H3B200_DTYPE_F16 = 1, H3B200_DTYPE_BF16 = 2, H3B200_DTYPE_I32 = 3, H3B200_DTYPE_E4M3 = 5 };

/* Library identification and diagnostics. */
H3B200_API const char* h3b200_version(void);
/* Message for the last non-zero status returned on the calling thread. */
H3B200_API const char* h3b200_last_error(void);
/* Reads (and optionally clears) the device status word of `device`, where
 * kernels record bounded-wait timeouts. Synchronises that device. */
H3B200_API int h3b200_device_status(int device, unsigned int* status, int clear);
/* Reads the mapped host copy of the status word of `device` without
 * synchronising (0 until a failure has become visible to the host). No
 * counterpart in the reference, whose kernels have no bounded waits. */
H3B200_API int h3b200_device_status_nowait(int device, unsigned int* status);
/* Test hook: launches one thread that waits, with limit timeout_ns (1 us to
 * 1 s), on a barrier nothing arrives at, so the wait expires and the kernel
 * records status 0x7E57 and returns. Exercises the failure reporting above
 * without a fault or a hang. No counterpart in the reference. */
H3B200_API int h3b200_selftest_expire_wait(int64_t timeout_ns, h3b200_stream_t stream);

/*
 * Elementwise pre-quantization activation on bf16 (y may alias x).
 * Replaces apply_input_act (backends/_activations.py:40-53; gelu_tanh =
 * torch.nn.functional.gelu(approximate="tanh")); bit-identical to the
 * reference's CPU result for every bf16 input. act = H3B200_ACT_SWIGLU is
 * row-structured and goes through h3b200_swiglu.
 */
H3B200_API int h3b200_apply_input_act(const void* x, void* y, int64_t n, int act, h3b200_stream_t stream);

/*
 * SwiGLU input activation: y[m, k] = silu(x[:, :k]) * x[:, k:2k] (bf16).
 * Replaces apply_input_act(x, "swiglu") (backends/_activations.py:40-53:
 * gate, up = x.chunk(2, -1); silu(gate).mul_(up)); bit-identical to the
 * reference's CPU result (silu exact on every bf16 input, the product rounded
 * once). x rows are [gate | up] at stride ldx >= 2k; y rows at stride ldy >= k.
 */
H3B200_API int h3b200_swiglu(const void* x, int64_t ldx, void* y, int64_t ldy, int64_t m, int64_t k,
                             h3b200_stream_t stream);

/*
 * Per-token absmax INT8 quantizer.
 * Replaces comfy_kitchen quantize_int8_rowwise: eager/quantization.py:857-875,
 * CUDA _C.quantize_int8_rowwise (backends/cuda/dlpack_bindings.cpp:2623,
 * kernel backends/cuda/ops/int8_linear.cu:157-200).
 * x: bf16 [m, k] with row stride ldx elements; act applied to x first
 * (backends/_activations.py:40-53). q: int8 [m, k] contiguous; scale: fp32 [m].
 * For act = H3B200_ACT_SWIGLU the rows of x are [gate | up], 2k wide
 * (ldx >= 2k), and the activated k-wide row is quantized; the same holds for
 * every entry point below that takes an act code, except the fused MLPs.
 */
H3B200_API int h3b200_quantize_int8_rowwise(const void* x, int64_t m, int64_t k, int64_t ldx, int act, int8_t* q,
                                 float* scale, h3b200_stream_t stream);

/*
 * quantize_int8_rowwise(x, stochastic_rounding=seed) with seed > 0: the same row
 * scale, then q = clamp(floor(bf16(bf16(x / bf16(scale)) + u)), -128, 127) with the
 * counter-based noise of the reference's CUDA kernel (backends/cuda/ops/int8_linear.cu:
 * 78-90, 186-193): u = bf16(float(pcg_hash(lo32(i + seed) ^ hi32(i + seed)) >> 8) * 2^-24)
 * for element i = row * k + col. Replaces the stochastic branch of _round_int8
 * (backends/eager/quantization.py:821-826), whose eager noise comes from torch.rand
 * and is generator-specific. Arguments as h3b200_quantize_int8_rowwise.
 */
H3B200_API int h3b200_quantize_int8_rowwise_stochastic(const void* x, int64_t m, int64_t k, int64_t ldx, int act,
                                                       int64_t seed, int8_t* q, float* scale,
                                                       h3b200_stream_t stream);

/*
 * quantize_int8_rowwise of an fp16 activation (no input activation): the
 * reference's arithmetic in fp16 (eager/quantization.py:815-826, 857-875): fp16 row
 * absmax, scale = max(absmax / 127, 1e-30) in fp32 (stored), divisor fp16(scale)
 * (2^-14 when that is zero), q = clamp(rne(fp16(x / divisor)), -128, 127).
 * x: fp16 [m, k] at row stride ldx elements; q int8 [m, k]; scale fp32 [m].
 */
H3B200_API int h3b200_quantize_int8_rowwise_f16(const void* x, int64_t m, int64_t k, int64_t ldx, int8_t* q,
                                                float* scale, h3b200_stream_t stream);

/*
 * Quantizer body with a precomputed per-row absmax (fp32 [m]); same arithmetic
 * as h3b200_quantize_int8_rowwise. Used for fc2's input after the fc1 epilogue
 * has reduced the row absmax (the reference quantizes the activated fc1 output
 * with quantize_int8_rowwise inside int8_linear, eager/quantization.py:1024).
 */
H3B200_API int h3b200_quantize_int8_rowwise_absmax(const void* x, const float* absmax, int64_t m, int64_t k, int64_t ldx,
                                        int8_t* q, float* scale, h3b200_stream_t stream);

/*
 * INT8 GEMM with int32 accumulators: out[m, n] = a[m, k] . w[n, k]^T.
 * Replaces comfy_kitchen mm_int8 / _int8_matmul_accumulate
 * (eager/quantization.py:749-800; CUDA cublas_gemm_int8.cu:204).
 * a, w: int8, rows contiguous along k (k % 16 == 0); out: int32 [m, n], n % 8 == 0.
 */
H3B200_API int h3b200_int8_mm(const int8_t* a, const int8_t* w, int64_t m, int64_t n, int64_t k, int32_t* out,
                   h3b200_stream_t stream);

/*
 * Dequantizing INT8 linear from an already quantized activation:
 * out = bf16(float(acc) * (x_scale[row] * w_scale[col])) (+ bf16 bias).
 * Replaces int8_linear_prequantized (backends/cuda/__init__.py:1934-1957) /
 * _C.cutlass_int8_dequant (dlpack_bindings.cpp:2713, cutlass_gemm_int8.cu:613),
 * with the eager epilogue association (eager/quantization.py:1044-1048).
 * w_scale_numel is 1 (tensor-wise) or n (per channel). bias may be NULL.
 * out_dtype H3B200_DTYPE_BF16 or H3B200_DTYPE_F16 (the reference's out_dtype,
 * eager/quantization.py:1044-1053): with F16, out = fp16(float(acc) * (x_scale *
 * w_scale)) and then fp16(out + bias), bias fp16 [n] (the reference converts the
 * bias to the output dtype before adding).
 */
H3B200_API int h3b200_int8_linear_prequantized(const int8_t* xq, const float* x_scale, const int8_t* w, const float* w_scale,
                                    int64_t w_scale_numel, const void* bias, int out_dtype, void* out, int64_t m,
                                    int64_t n, int64_t k, h3b200_stream_t stream);

/*
 * One INT8 GEMM with a fused epilogue -- the building block of the fused MLP,
 * exposed so each stage can be launched and timed on its own.
 * epilogue: 0 int32 out; 1 bf16 dequant (+bias); 2 dequant -> tanh-GELU -> bf16
 * out with the per-row absmax of |out| atomically max-reduced into row_absmax
 * (fp32 [m], caller zero-fills); 3 out = bf16(residual + y * gate) with
 * y = dequant, or bf16(dequant + bias) when bias is given.
 * Arithmetic as h3b200_int8_linear_prequantized / h3b200_fused_gated_mlp.
 * Replaces the reference's CUTLASS EVT GEMM (backends/cuda/ops/cutlass_gemm_int8.cu:242-324)
 * and the experimental fc2 + dequant + gate + residual Triton epilogue
 * (h3serve/native_engine/model/fused_mlp.py:58-143).
 */
H3B200_API int h3b200_int8_gemm_fused(const int8_t* a, int64_t lda, const int8_t* w, int64_t ldw, int64_t m,
                                      int64_t n, int64_t k, int epilogue, const float* a_scale,
                                      const float* w_scale, int64_t w_scale_numel, const void* bias,
                                      const void* gate, const void* residual, int64_t ldr, void* out, int64_t ldo,
                                      float* row_absmax, h3b200_stream_t stream);

/*
 * fc2 of the fused MLP with the requantization of its input inside the GEMM:
 *   q, xs = quantize_int8_rowwise(h)   with max |h[row, :]| given in h_absmax[row]
 *   out   = bf16(residual + bf16(bf16(float(q . W^T) * (xs * w_scale)) (+ bias)) * gate)
 * the requant -> int8_linear -> addcmul_ chain of the reference's fused MLP
 * (h3serve/native_engine/model/fused_mlp.py:414-425; quantize_int8_rowwise
 * backends/eager/quantization.py:857-875). h_absmax is what epilogue 2 of
 * h3b200_int8_gemm_fused reduces. The GEMM's spare warps quantize h's rows into
 * the workspace in row order while the tensor cores run; tiles wait (bounded)
 * for their rows. gate is one row [n] (row_map NULL) or rows at stride ldg
 * selected per output row by row_map. Bit-identical to
 * h3b200_quantize_int8_rowwise_absmax followed by epilogue 3.
 * workspace: h3b200_requant_gemm_workspace_bytes(m, k) bytes, 256-byte aligned.
 * k % 16 == 0, n % 8 == 0, ldh % 8 == 0, h 16-byte aligned; out may alias residual.
 */
H3B200_API int64_t h3b200_requant_gemm_workspace_bytes(int64_t m, int64_t k);
H3B200_API int h3b200_requant_gemm_gated_residual(const void* h, int64_t ldh, const float* h_absmax,
                                                  const int8_t* w, const float* w_scale, int64_t w_scale_numel,
                                                  const void* bias, const void* gate, int64_t ldg,
                                                  const int32_t* row_map, const void* residual, int64_t ldr,
                                                  void* out, int64_t ldo, int64_t m, int64_t n, int64_t k,
                                                  void* workspace, int64_t workspace_bytes,
                                                  h3b200_stream_t stream);

/*
 * Dequant + gated residual on reduced int32 accumulators (tensor-parallel fc2):
 * out = bf16(residual + bf16(float(acc) * (x_scale[row] * w_scale[col])) * gate[col]).
 * The same arithmetic as epilogue 3 of h3b200_int8_gemm_fused, for when the
 * accumulators of a row-split fc2 were summed across ranks first (the
 * reference's addcmul_ gated residual, h3serve/native_engine/model/fused_mlp.py:414-425).
 * acc: int32 [m, n] contiguous; n % 8 == 0; out may alias residual.
 */
H3B200_API int h3b200_dequant_gated_residual(const int32_t* acc, const float* x_scale, const float* w_scale,
                                             const void* gate, const void* residual, int64_t ldr, void* out,
                                             int64_t ldo, int64_t m, int64_t n, h3b200_stream_t stream);

/*
 * Full dynamically quantized INT8 linear: act -> per-row quantize -> GEMM ->
 * dequant (+ bias). Replaces comfy_kitchen int8_linear(x, weight, weight_scale,
 * bias, out_dtype, convrot=False, input_act) (__init__.py:722-764; CUDA
 * backends/cuda/__init__.py:1960-2081; eager eager/quantization.py:971-1056).
 * workspace: at least h3b200_int8_linear_workspace_bytes(m, k) bytes, 256-byte aligned.
 */
H3B200_API int64_t h3b200_int8_linear_workspace_bytes(int64_t m, int64_t k);
H3B200_API int h3b200_int8_linear(const void* x, int64_t ldx, const int8_t* w, const float* w_scale, int64_t w_scale_numel,
                       const void* bias, int act, void* out, int64_t m, int64_t n, int64_t k, void* workspace,
                       int64_t workspace_bytes, h3b200_stream_t stream);

/*
 * Allocation-free variant of h3b200_int8_linear. It has no counterpart in the
 * reference. It is for callers that cannot allocate device memory per call
 * (a runtime that owns all device memory and passes only inputs and outputs,
 * or a serving loop that must not allocate after start-up): the quantized
 * activation and its row scales live in a static device array of
 * h3b200_int8_linear_noalloc_max_scratch_bytes() bytes (8 MiB) that every GPU
 * loading the library holds until exit, and no memory is allocated.
 * Limit: round_up(m * k, 256) + 4 * m must fit in that array (e.g. m <= 2600 at
 * k = 3072); larger calls are rejected with H3B200_ERR_INVALID. The first call
 * on a device looks up the array's device address with that device current and
 * fills the device's tanh-GELU table (synchronising `stream` once), whatever
 * `act` it asks for; make that first call before any stream capture. All calls
 * share the array: calls that overlap on the GPU race on it. The cached address
 * belongs to the device's current context: after cudaDeviceReset this library's
 * per-device state (this address, its activation tables, the status mirror) is
 * stale, so do not call it again in that process. Same arithmetic and result as
 * h3b200_int8_linear; the caller still passes x, w, scales, bias and out.
 */
H3B200_API int64_t h3b200_int8_linear_noalloc_max_scratch_bytes(void);
H3B200_API int h3b200_int8_linear_noalloc(const void* x, int64_t ldx, const int8_t* w, const float* w_scale,
                                          int64_t w_scale_numel, const void* bias, int act, void* out, int64_t m,
                                          int64_t n, int64_t k, h3b200_stream_t stream);

/*
 * Fused gated W8A8 MLP on a token chunk:
 *   h = int8_linear(x, w1, s1); a = act(h); y = int8_linear(a, w2, s2);
 *   out = residual + y * gate   (bf16 addcmul)
 * Replaces try_fused_gated_mlp (h3serve/native_engine/model/fused_mlp.py:269-426,
 * fc1 -> fused-act fc2 -> addcmul_ :393-425) and the original backend's
 * resident_weight_chunked_gated_mlp (backends/original/native_acceleration.py:79-126)
 * for the tanh-GELU activation (act must be H3B200_ACT_GELU_TANH).
 * x, residual, out: bf16 [m, d] (row strides ldx / ldr / ldo elements; out may
 * alias residual); w1: int8 [ffn, d]; s1: fp32 [ffn]; w2: int8 [d, ffn];
 * s2: fp32 [d]; gate: bf16 [d]. d % 16 == 0 and ffn % 16 == 0.
 */
H3B200_API int64_t h3b200_fused_gated_mlp_workspace_bytes(int64_t m, int64_t d, int64_t ffn);
H3B200_API int h3b200_fused_gated_mlp(const void* x, int64_t ldx, const int8_t* w1, const float* s1, const int8_t* w2,
                           const float* s2, const void* gate, const void* residual, int64_t ldr, void* out,
                           int64_t ldo, int64_t m, int64_t d, int64_t ffn, int act, void* workspace,
                           int64_t workspace_bytes, h3b200_stream_t stream);
/*
 * The same MLP with per-token gate rows: out[t] = residual[t] + y[t] * gate_rows[row_map[t]]
 * -- the per-modulation-segment addcmul_ of try_fused_gated_mlp
 * (h3serve/native_engine/model/fused_mlp.py:414-425 via _segment_row_map :34-55;
 * _gated_residual layers.py:937-953). gate_rows: bf16 rows at stride ldg
 * (>= d, a multiple of 8); row_map: int32 [m] on the device, every value a
 * valid row. Same workspace as h3b200_fused_gated_mlp.
 */
H3B200_API int h3b200_fused_gated_mlp_segmented(const void* x, int64_t ldx, const int8_t* w1, const float* s1,
                                                const int8_t* w2, const float* s2, const void* gate_rows,
                                                int64_t ldg, const int32_t* row_map, const void* residual,
                                                int64_t ldr, void* out, int64_t ldo, int64_t m, int64_t d,
                                                int64_t ffn, int act, void* workspace, int64_t workspace_bytes,
                                                h3b200_stream_t stream);

/*
 * RMS-AdaLN on the hidden stream, with per-token modulation rows:
 *   h   = bf16((x / sqrt(mean(x^2) + eps)) * w)   (no weight: bf16(x / sqrt(..)))
 *   out = bf16(bf16(h * bf16(1 + scale[r])) + shift[r])
 * r = row_map[t] (int32 [m] on the device; values outside [0, mod_rows) are
 * clamped), or, with row_map NULL, t / tokens_per_row (tokens_per_row <= 0:
 * row 0 for every token). scale == shift == NULL gives the plain RMSNorm.
 * Replaces H3's rms_adaln(value, norm, shift, scale, segments)
 * (h3serve/native_engine/model/kernels.py:7586-7634: F.rms_norm with the
 * module weight, then per segment mul_(1 + scale[row]).add_(shift[row]) in bf16;
 * its Triton _segmented_rms_adaln_kernel, backends/original/kernels/
 * fused_norm_rope.py:12-44, keeps the same three bf16 steps) and comfy_kitchen's
 * rms_adaln(x, scale, shift, eps) (__init__.py:130-150; eager
 * backends/eager/adaln.py:17-20, no weight; per-sample [B, 1, D] modulation is
 * tokens_per_row = T, like its CUDA kernel's scale_group, cuda/ops/adaln.cu:104-199).
 * x, out: bf16 [m, d] at row strides ldx / ldo (out may alias x); norm_weight:
 * bf16 [d] or NULL; scale / shift: bf16 [mod_rows, d] at row strides
 * ld_scale / ld_shift. d % 8 == 0, d <= 8192, 16-byte aligned rows.
 */
H3B200_API int h3b200_rms_adaln(const void* x, int64_t ldx, const void* norm_weight, const void* scale,
                                int64_t ld_scale, const void* shift, int64_t ld_shift, int64_t mod_rows,
                                const int32_t* row_map, int64_t tokens_per_row, float eps, void* out, int64_t ldo,
                                int64_t m, int64_t d, h3b200_stream_t stream);

/*
 * Fused (AdaLN-modulate +) RMSNorm + split-half RoPE on Q and K.
 * Q/K: bf16 [m, heads, head_dim] with token strides ldq/ldk (elements; rows of
 * heads*head_dim contiguous); outputs may alias inputs.
 * norm_span 0 = row: RMSNorm over heads*head_dim with q_weight/k_weight [heads*head_dim],
 *   then h*(1+scale) and +shift ([heads*head_dim] bf16, bf16 after each step)
 *   -- rms_adaln (h3serve/native_engine/model/kernels.py:7586-7634, eager order
 *   :7623-7631; comfy rms_adaln eager/adaln.py:132) fused with the rope below.
 * norm_span 1 = head: per-head RMSNorm with [head_dim] weights
 *   -- rms_rope_split_half(_) (__init__.py:549-580; eager/rope.py:67-143;
 *   CUDA backends/cuda/ops/rms_rope.cu:36-229, launcher :353-384). scale/shift,
 *   when non-NULL, are applied per row after the norm.
 * RoPE: freqs fp32 [m, rot_dim/2, 2, 2] packed [[cos,-sin],[sin,cos]]
 *   (h3serve/native_engine/model/layers.py:61-69); pair i couples element i and
 *   i + rot_dim/2 of each head (eager/rope.py:39-42); rot_dim 0 means head_dim;
 *   dims >= rot_dim pass through.
 * Supported: head_dim == 128, rot_dim % 16 == 0, heads <= 32, 16-byte aligned rows.
 */
H3B200_API int h3b200_adaln_rms_rope(const void* q, int64_t ldq, const void* k, int64_t ldk, void* q_out, int64_t ldqo,
                          void* k_out, int64_t ldko, const float* freqs, const void* q_weight, const void* k_weight,
                          const void* scale, const void* shift, int64_t m, int64_t heads, int64_t head_dim,
                          int64_t rot_dim, int norm_span, float eps, h3b200_stream_t stream);
/*
 * h3b200_adaln_rms_rope (row span) with a modulation row per token: token t
 * uses scale / shift row row_map[t] (int32 [m] on the device, clamped to
 * [0, mod_rows)), or t / tokens_per_row when row_map is NULL -- H3's segmented
 * rms_adaln (kernels.py:7586-7634, per-segment scale[row] / shift[row],
 * layers.py:909-934 _scale_shift) fused with the RoPE. scale / shift: bf16
 * [mod_rows, heads*head_dim] at row strides ld_scale / ld_shift (multiples of 8).
 */
H3B200_API int h3b200_adaln_rms_rope_segmented(const void* q, int64_t ldq, const void* k, int64_t ldk, void* q_out,
                                               int64_t ldqo, void* k_out, int64_t ldko, const float* freqs,
                                               const void* q_weight, const void* k_weight, const void* scale,
                                               int64_t ld_scale, const void* shift, int64_t ld_shift,
                                               int64_t mod_rows, const int32_t* row_map, int64_t tokens_per_row,
                                               int64_t m, int64_t heads, int64_t head_dim, int64_t rot_dim,
                                               float eps, h3b200_stream_t stream);

/*
 * Per-head RMSNorm + partial split-half RoPE on one tensor (k == NULL) or two,
 * over strided bf16 [m, heads, head_dim] views: element strides token (_st)
 * and head (_sh), unit stride on head_dim. Outputs may alias the inputs (in
 * place) or be other views, e.g. an HND-backed NHD view of an attention
 * buffer [heads, tokens, head_dim] (qo_st = head_dim, qo_sh = tokens * head_dim).
 *   h = bf16((x / sqrt(mean(x^2) + eps)) * w)   (w: bf16 [head_dim] per tensor)
 *   y[i] = t00 h[i] + t01 h[i + r/2], y[i + r/2] = t10 h[i] + t11 h[i + r/2]  (i < r/2)
 *   y[i] = h[i] for i >= r = rot_dim (0: head_dim)
 * freqs: rows of [r/2, 2, 2] values, dtype code 0 (float32), 1 (float16) or
 * 2 (bfloat16; widened to fp32), at element stride f_st per token and f_sh
 * per head (0 = one row shared by all heads); freqs NULL: RMSNorm only (the
 * reference's q_norm / k_norm without frequencies). head_dim 128, rot_dim a
 * multiple of 16; pointers 16-byte aligned, strides multiples of 8 elements.
 * Replaces launch_rms_rope_kernel with split_half = true and has_k = false
 * (single side) or true (backends/cuda/ops/rms_rope.cu:36-229, launcher
 * :353-384), as bound by h3serve/native_engine/model/single_qknorm_rope.py:
 * 37-63 (_try_apply_single_qknorm_rope_out :69-181, the HND target :209-236);
 * eager semantics backends/eager/rope.py:67-92.
 */
H3B200_API int h3b200_qknorm_rope_strided(const void* q, int64_t q_st, int64_t q_sh, void* q_out, int64_t qo_st,
                                          int64_t qo_sh, const void* q_weight, const void* k, int64_t k_st,
                                          int64_t k_sh, void* k_out, int64_t ko_st, int64_t ko_sh,
                                          const void* k_weight, const void* freqs, int freqs_dtype, int64_t f_st,
                                          int64_t f_sh, int64_t m, int64_t heads, int64_t head_dim,
                                          int64_t rot_dim, float eps, h3b200_stream_t stream);

/*
 * Q/K/V projection of one token chunk with QK-norm + partial RoPE into the
 * attention layout, from an activation quantized once (ConvRot or plain,
 * h3b200_quantize_int8_rowwise_convrot / h3b200_quantize_int8_rowwise):
 *   proj = int8_linear_prequantized(xq, x_scale, W[rows of sections], w_scale, bias)
 *   Q -> q_out, K -> k_out: per-head RMSNorm (q/k norm weight, bf16 [head_dim])
 *        and split-half RoPE as h3b200_qknorm_rope_strided (freqs NULL: RMSNorm only)
 *   V -> v_out unchanged
 * Sections [sec_begin, sec_end) of {0: Q, 1: K, 2: V}: (0, 3) all three,
 * (1, 3) the K/V build, (0, 1) a query chunk. w_qkv: int8 [3 heads head_dim, k]
 * (rows Q | K | V), w_scale fp32 [3 heads head_dim] or [1], bias bf16
 * [3 heads head_dim] or NULL; xq int8 [m, k], x_scale fp32 [m]. Outputs are
 * [m, heads, head_dim] views with element strides token (_st) and head (_sh),
 * e.g. HND buffers (st = head_dim, sh = tokens * head_dim). workspace:
 * h3b200_qkv_qknorm_rope_workspace_bytes(m, heads, head_dim, sec_begin, sec_end).
 * Replaces the H3 long-sequence attention build
 * (h3serve/native_engine/model/layers.py:445-641: prepare_output_slices /
 * forward_prepared_output_slice, quantization.py:340-415, with
 * try_apply_single_qknorm_rope_to_hnd for K and Q and the V copy into HND).
 */
H3B200_API int64_t h3b200_qkv_qknorm_rope_workspace_bytes(int64_t m, int64_t heads, int64_t head_dim, int sec_begin,
                                                         int sec_end);
H3B200_API int h3b200_qkv_qknorm_rope(const int8_t* xq, const float* x_scale, int64_t m, int64_t k,
                                      const int8_t* w_qkv, const float* w_scale, int64_t w_scale_numel,
                                      const void* bias, int64_t heads, int64_t head_dim, int sec_begin, int sec_end,
                                      const void* q_norm_weight, const void* k_norm_weight, const void* freqs,
                                      int freqs_dtype, int64_t f_st, int64_t f_sh, int64_t rot_dim, float eps,
                                      void* q_out, int64_t q_st, int64_t q_sh, void* k_out, int64_t k_st,
                                      int64_t k_sh, void* v_out, int64_t v_st, int64_t v_sh, void* workspace,
                                      int64_t workspace_bytes, h3b200_stream_t stream);

/*
 * W4A8: decode packed uint4 weights to the int8 grid,
 * clamp(rne((u - 8) * s_rel[row, group]), -127, 127), even column = low nibble.
 * Replaces _C.dequant_int4_grouped_to_int8 (dlpack_bindings.cpp:2781-2790;
 * kernel backends/cuda/ops/w4a8_gemm.cu:36-90; eager eager/w4a8_int8.py:344-363).
 * qdata: int8 [n, k/2]; s_rel: fp32 [n, k/group]; out: int8 [n, k].
 */
H3B200_API int h3b200_dequant_int4_grouped_to_int8(const int8_t* qdata, const float* s_rel, int64_t n, int64_t k,
                                        int64_t group_size, int8_t* out, h3b200_stream_t stream);

/*
 * The same decode for every scale type and level table of the reference:
 * q = clamp(rne(level(u) * s_rel[row, group]), -127, 127) with level(u) = u - 8
 * (codebook NULL) or codebook[u] (16 fp32 levels, the H3 release format's
 * Lloyd-Max table). s_rel_dtype: H3B200_DTYPE_F32 (fp32 [n, k/group]) or
 * H3B200_DTYPE_E4M3 (float8_e4m3fn bytes [n, k/group], widened exactly).
 * group_size 4, 8 or a multiple of 16. NaN scales decode to 0.
 * Replaces launch_dequant_int4_grouped_to_int8 and
 * launch_dequant_int4_grouped_to_int8_e4m3 (backends/cuda/ops/w4a8_gemm.cu:92-121,
 * kernel :36-90; eager _dequant_int4_grouped_to_int8 eager/w4a8_int8.py:344-363).
 */
H3B200_API int h3b200_dequant_int4_grouped_to_int8_ex(const int8_t* qdata, const void* s_rel, int s_rel_dtype,
                                                      const float* codebook, int64_t n, int64_t k, int64_t group_size,
                                                      int8_t* out, h3b200_stream_t stream);

/*
 * ConvRot (regular Hadamard, group 256) + per-row INT8 quantization, with an
 * optional activation applied first.
 * Replaces _C.quantize_int8_rowwise_convrot / quantize_int8_rowwise_convrot64
 * (dlpack_bindings.cpp:2835; kernels backends/cuda/ops/int8_linear.cu:256-340,
 * 942-1027; eager quantize_and_rotate_rowwise eager/quantization.py:878-895).
 * The rotated row is rounded to bf16 before quantization, as the reference's
 * bf16 rotation matmul does. k % 256 == 0.
 */
H3B200_API int h3b200_quantize_int8_rowwise_convrot(const void* x, int64_t m, int64_t k, int64_t ldx, int64_t group_size,
                                         int act, int8_t* q, float* scale, h3b200_stream_t stream);

/*
 * W4A8 INT8 linear with asymmetric group correction:
 *   xr, xq, xs = convrot-quantize(act(x)); acc = xq . grid^T;
 *   out = bf16(bf16(acc * (xs * s_channel)) + (bf16(bf16(sum_g xq) * bf16(xs)) . correction))
 * Replaces comfy_kitchen w4a8_int8_linear (tensor/w4a8_int8.py:89-115; CUDA
 * backends/cuda/__init__.py:2139-2298, asymmetric correction :2294-2297).
 * grid: int8 [n, k] decoded weight (h3b200_dequant_int4_grouped_to_int8);
 * s_channel: fp32 [n]; correction: bf16 [k/group, n] or NULL (symmetric);
 * bias: bf16 [n] or NULL. Symmetric weights: the call is
 * int8_linear(x, grid, s_channel, bias, convrot=True) (eager/w4a8_int8.py:494-508).
 * With a correction the bias joins the dequantized value before the correction is
 * added: out = bf16(bf16(bf16(acc * (xs * s_channel)) + bias) + corr), the order of the
 * reference's CUDA path (bias in the dequant epilogue, then out.addmm_(sx, correction),
 * backends/cuda/__init__.py:2265-2297); the eager path (a bf16 F.linear on the
 * dequantized weight, eager/w4a8_int8.py:481-492) agrees within the tolerances.
 * workspace: h3b200_w4a8_linear_workspace_bytes(m, n, k, group) bytes. The
 * correction is accumulated on the tensor cores inside the INT8 GEMM's
 * epilogue (bf16 operands, fp32 accumulation), at most 128 groups.
 */
H3B200_API int64_t h3b200_w4a8_linear_workspace_bytes(int64_t m, int64_t n, int64_t k, int64_t group_size);
H3B200_API int h3b200_w4a8_int8_linear(const void* x, int64_t ldx, const int8_t* grid, const float* s_channel,
                            const void* correction, const void* bias, int64_t group_size, int64_t convrot_group,
                            int act, void* out,
                            int64_t m, int64_t n, int64_t k, void* workspace, int64_t workspace_bytes,
                            h3b200_stream_t stream);

/*
 * The same linear from the packed int4 weight itself (qdata [n, k/2], even column in the
 * low nibble; s_rel fp32 or fp8-e4m3 [n, k/group] per s_rel_dtype; codebook 16 fp32
 * levels or NULL for u - 8), the reference's w4a8_int8_linear(x, qdata, s_rel, s_channel,
 * codebook, correction, bias, group_size, convrot_groupsize) (tensor/w4a8_int8.py:89-115;
 * CUDA backends/cuda/__init__.py:2139-2298 decodes into an int8 workspace first).
 * For m <= 32, or m <= 16 with a correction (and k % 128 == 0, group a
 * multiple of 16 dividing 128 or a multiple of 128, at most 128 correction groups), the
 * GEMM reads the packed weight through TMA and unpacks it to int8 in shared memory, tile by
 * tile, so the weight crosses HBM at 4 bits per element; K is split over CTAs so that few
 * rows still fill the GPU, and the correction is summed on CUDA cores from a shared-memory
 * copy (fp32, one rounding). Otherwise the grid is decoded once into the workspace and the
 * call takes h3b200_w4a8_int8_linear. workspace: h3b200_w4a8_linear_packed_workspace_bytes(m, n, k, group).
 */
H3B200_API int64_t h3b200_w4a8_linear_packed_workspace_bytes(int64_t m, int64_t n, int64_t k, int64_t group_size);
H3B200_API int h3b200_w4a8_int8_linear_packed(const void* x, int64_t ldx, const uint8_t* qdata, const void* s_rel,
                                              int s_rel_dtype, const float* codebook, const float* s_channel,
                                              const void* correction, const void* bias, int64_t group_size,
                                              int64_t convrot_group, int act, void* out, int64_t m, int64_t n,
                                              int64_t k, void* workspace, int64_t workspace_bytes,
                                              h3b200_stream_t stream);

/*
 * Fused gated W4A8 MLP on a token chunk (config 2):
 *   h = w4a8_linear(x, W1); a = gelu_tanh(h); y = w4a8_linear(a, W2);
 *   out = residual + y * gate   (bf16 addcmul)
 * with w4a8_linear as h3b200_w4a8_int8_linear (ConvRot-256 + per-token INT8
 * activations, asymmetric group correction). The weights stay in the
 * reference's packed format (int4 at rest: qdata int8 [n, k/2], s_rel fp32
 * [n, k/group], s_channel fp32 [n], correction bf16 [k/group, n]); each call
 * decodes them into an int8 grid in the workspace (the GEMM then reads it
 * from L2). Composition of w4a8_int8_linear (tensor/w4a8_int8.py:89-115),
 * apply_input_act (backends/_activations.py:40-53) and the addcmul of
 * try_fused_gated_mlp (h3serve/native_engine/model/fused_mlp.py:414-425).
 * x, residual, out: bf16 [m, d] (out may alias residual); gate: bf16 [d];
 * W1 is [ffn, d], W2 is [d, ffn]; d and ffn multiples of 256 and of group_size.
 */
H3B200_API int64_t h3b200_fused_gated_mlp_w4a8_workspace_bytes(int64_t m, int64_t d, int64_t ffn,
                                                              int64_t group_size);
H3B200_API int h3b200_fused_gated_mlp_w4a8(const void* x, int64_t ldx, const int8_t* qdata1, const float* s_rel1,
                                           const float* s_channel1, const void* correction1, const int8_t* qdata2,
                                           const float* s_rel2, const float* s_channel2, const void* correction2,
                                           const void* gate, const void* residual, int64_t ldr, void* out,
                                           int64_t ldo, int64_t m, int64_t d, int64_t ffn, int64_t group_size,
                                           int act, void* workspace, int64_t workspace_bytes,
                                           h3b200_stream_t stream);

/*
 * Fused gated SwiGLU INT8 MLP, the H3 production path (hidden d, fc1 out 2 ffn):
 *   raw = int8_linear(x, W1, s1, b1, convrot = fc1_convrot_group);
 *   y   = int8_linear(raw, W2, s2, b2, convrot = 256, input_act = "swiglu");
 *   out[t] = residual[t] + y[t] * gate[row_map[t]]   (bf16 addcmul per token)
 * Drop-in for try_fused_gated_mlp's INT8 path (h3serve/native_engine/model/
 * fused_mlp.py:269-426: fc1 :366, fused-act fc2 :393-405, per-segment
 * addcmul :410-424, segment row map _segment_row_map :34-55) with
 * int8_linear as in eager/quantization.py:971-1056 (ConvRot weights are
 * rotated offline along their input dimension).
 * x, residual, out: bf16 [m, d] (out may alias residual); W1 int8 [2 ffn, d]
 * ([gate | up] output rows), s1 fp32 [2 ffn] or [1], b1 bf16 [2 ffn] or NULL;
 * W2 int8 [d, ffn], s2 fp32 [d] or [1], b2 bf16 [d] or NULL.
 * gate: bf16 [d] when row_map is NULL, else bf16 [rows, ldg] and row_map
 * int32 [m] gives each token's modulation row. fc1_convrot_group: 0 or 256.
 * ffn (and d with fc1 ConvRot) multiples of 256. Tokens are processed in
 * chunks of chunk_tokens; workspace:
 * h3b200_fused_gated_mlp_swiglu_workspace_bytes(min(chunk_tokens, m), d, ffn).
 */
H3B200_API int64_t h3b200_fused_gated_mlp_swiglu_workspace_bytes(int64_t chunk_tokens, int64_t d, int64_t ffn);
H3B200_API int h3b200_fused_gated_mlp_swiglu(const void* x, int64_t ldx, const int8_t* w1, const float* s1,
                                             int64_t s1_numel, const void* b1, const int8_t* w2, const float* s2,
                                             int64_t s2_numel, const void* b2, const void* gate, int64_t ldg,
                                             const int32_t* row_map, const void* residual, int64_t ldr, void* out,
                                             int64_t ldo, int64_t m, int64_t d, int64_t ffn,
                                             int64_t fc1_convrot_group, int64_t chunk_tokens, void* workspace,
                                             int64_t workspace_bytes, h3b200_stream_t stream);

/*
 * The H3 SwiGLU MLP on W4A8 weights in the H3 release format (group 16,
 * fp8-e4m3 s_rel, 16-level codebook, symmetric; ConvRot-256 on both linears):
 *   raw = w4a8_linear(x, W1, b1); y = w4a8_linear(silu(raw_gate) * raw_up, W2, b2);
 *   out[t] = residual[t] + y[t] * gate[row_map[t]]
 * with w4a8_linear(v, W, b) = int8_linear(v, decode(W), s_channel, b, convrot=True).
 * Drop-in for try_fused_gated_mlp's W4A8 path, _chunked_module_gated_mlp
 * (h3serve/native_engine/model/fused_mlp.py:222-266) over ConvRotW4A8Linear
 * modules (quantization.py:416-600) bound to comfy_kitchen.w4a8_int8_linear
 * (quantization.py:64-95). Both int4 weights are decoded once per call into
 * the workspace (h3b200_dequant_int4_grouped_to_int8_ex), then the token
 * chunks run as h3b200_fused_gated_mlp_swiglu with fc1 ConvRot on.
 * qdata1 int8 [2 ffn, d/2], s_rel1 [2 ffn, d/group], s_channel1 fp32 [2 ffn],
 * codebook1 fp32 [16] or NULL, b1 bf16 [2 ffn] or NULL; qdata2 int8 [d, ffn/2],
 * s_rel2 [d, ffn/group], s_channel2 fp32 [d], codebook2, b2 bf16 [d] or NULL;
 * s_rel_dtype H3B200_DTYPE_F32 or H3B200_DTYPE_E4M3 (both weights). Other
 * arguments as h3b200_fused_gated_mlp_swiglu. workspace:
 * h3b200_fused_gated_mlp_swiglu_w4a8_workspace_bytes(min(chunk_tokens, m), d, ffn).
 */
H3B200_API int64_t h3b200_fused_gated_mlp_swiglu_w4a8_workspace_bytes(int64_t chunk_tokens, int64_t d, int64_t ffn);
H3B200_API int h3b200_fused_gated_mlp_swiglu_w4a8(const void* x, int64_t ldx, const int8_t* qdata1,
                                                  const void* s_rel1, const float* s_channel1, const float* codebook1,
                                                  const void* b1, const int8_t* qdata2, const void* s_rel2,
                                                  const float* s_channel2, const float* codebook2, const void* b2,
                                                  int s_rel_dtype, int64_t group_size, const void* gate, int64_t ldg,
                                                  const int32_t* row_map, const void* residual, int64_t ldr,
                                                  void* out, int64_t ldo, int64_t m, int64_t d, int64_t ffn,
                                                  int64_t chunk_tokens, void* workspace, int64_t workspace_bytes,
                                                  h3b200_stream_t stream);

/*
 * Tensor-parallel gated W8A8 MLP over NVLink peer memory (one process per GPU).
 * The reference runs the MLP on one GPU (try_fused_gated_mlp,
 * h3serve/native_engine/model/fused_mlp.py:269-426); this splits it over a group
 * of `world` GPUs: rank r owns fc1 rows [r ffn/world, (r+1) ffn/world) of W1 and the
 * same columns of W2 (w1q int8 [ffn_shard, d], s1 fp32 [ffn_shard], w2q int8
 * [d, ffn_shard] contiguous, s2 fp32 [d]); x, residual and gate are replicated.
 * Per token chunk of c rows: quantize x, fc1 + GELU + row absmax on the own columns,
 * the row absmax max-reduced over the ranks (pushed into every rank's slot, barrier,
 * max), fc2 quantizing its own input with that global absmax and storing each int32
 * partial row straight into the receive slot of the rank that owns the row (blocks of
 * 128 rows round-robin: row r belongs to rank (r / 128) % world), barrier, then each owner
 * sums the ranks' partials, applies dequant + gated residual and writes its rows to
 * its own out and to every rank's gather buffer (copied into out after the next
 * barrier). No NCCL call on the data path. out is bit-identical to
 * h3b200_fused_gated_mlp on one GPU (int32 sums are exact; the requant uses the
 * global absmax).
 *
 * Set-up: every rank calls h3b200_tp_comm_create with identical max_rows / d /
 * ffn_shard and its rank, exchanges the H3B200_TP_HANDLE_BYTES handle bytes with the
 * others (any host transport), and calls h3b200_tp_comm_open with all handles in rank
 * order (CUDA IPC mappings; world == 1 needs no open). Then h3b200_tp_gated_mlp on
 * every rank, with the same m and chunk_rows, in the same order. The cross-GPU
 * barrier waits at most barrier_timeout_ns (0: 5 s) and records device status 0x201
 * on expiry; the ranks' barrier counts then disagree, so clear the status and create
 * new communicators on every rank before the next call. h3b200_tp_comm_destroy after
 * the last call has completed on every rank (no peer may still write into the region).
 * A communicator is used by one host thread at a time; its calls are ordered on the
 * stream they are given.
 *
 * h3b200_tp_stage / h3b200_tp_barrier expose the pipeline's steps (stage 1: quantize,
 * fc1, absmax push; 2: absmax max, fc2 with routed rows; 3: owner rows; 4: copy the
 * other owners' rows of chunk `chunk` into out). h3b200_tp_comm_link_local makes
 * `world` communicators created in ONE process on ONE device each other's peers
 * (no IPC; barriers become no-ops), so a test can run every rank's stages in
 * order on one GPU.
 */
#define H3B200_TP_HANDLE_BYTES 192
H3B200_API int h3b200_tp_comm_create(int rank, int world, int64_t max_rows, int64_t d, int64_t ffn_shard,
                                     int64_t barrier_timeout_ns, void** comm, uint8_t* handle);
H3B200_API int h3b200_tp_comm_open(void* comm, const uint8_t* handles);
H3B200_API int h3b200_tp_comm_link_local(void* const* comms, int world);
H3B200_API int h3b200_tp_comm_destroy(void* comm);
H3B200_API int h3b200_tp_barrier(void* comm, h3b200_stream_t stream);
H3B200_API int h3b200_tp_stage(void* comm, int stage, int64_t chunk, const void* x, int64_t ldx,
                               const void* residual, int64_t ldr, const void* gate, const int8_t* w1q,
                               const float* s1, const int8_t* w2q, const float* s2, void* out, int64_t ldo,
                               int64_t lo, int64_t hi, h3b200_stream_t stream);
H3B200_API int h3b200_tp_gated_mlp(void* comm, const void* x, int64_t ldx, const void* residual, int64_t ldr,
                                   const void* gate, const int8_t* w1q, const float* s1, const int8_t* w2q,
                                   const float* s2, void* out, int64_t ldo, int64_t m, int64_t chunk_rows,
                                   h3b200_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* H3B200_H_ */
