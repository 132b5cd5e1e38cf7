/*
 * ctu_b200.h -- C ABI of the B200 (sm_100a) ConvRot quantized-linear library
 * (libctu_b200.so).  Plain pointers, sizes and a CUDA stream; no framework types.
 *
 * Every device pointer must be a CUDA device (or managed) address on the current
 * device.  Entry points enqueue work on `stream` (a cudaStream_t; NULL = legacy
 * default stream) and return without synchronizing.  Return value: CTU_OK, or an
 * error code with a message available from ctu_last_error() (thread-local).
 *
 * Each entry point names the reference interface it replaces (comfyui-turing-utils,
 * kernel package 0.31.0; paths relative to the reference repository).
 */
#ifndef CTU_B200_H_
#define CTU_B200_H_

#include <stdint.h>

#if defined(__GNUC__)
#define CTU_API __attribute__((visibility("default")))
#else
#define CTU_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define CTU_OK 0
#define CTU_ERR_INVALID_ARGUMENT 1 /* shape, alignment or dtype contract violated */
#define CTU_ERR_UNSUPPORTED 2      /* valid request this build does not implement */
#define CTU_ERR_CUDA 3             /* a CUDA runtime/driver call failed */

/* Activation fused in front of the rotation. */
#define CTU_ACT_NONE 0
#define CTU_ACT_SWIGLU 1    /* x is [rows, 2k] = [gate | up]; silu(gate) * up */
#define CTU_ACT_GELU_TANH 2 /* tanh-approximate GELU, rounded to bf16 */

/* Storage types of the norm entry points (every floating tensor of one call). */
#define CTU_DTYPE_BF16 0
#define CTU_DTYPE_FP16 1
#define CTU_DTYPE_FP32 2

/* Library version, (major << 16) | (minor << 8) | patch. */
CTU_API int ctu_version(void);

/* Message for the most recent failing call on this thread ("" if none). */
CTU_API const char *ctu_last_error(void);

/*
 * Device error word: kernels record bounded-wait timeouts here instead of hanging.
 * Reads (and, with clear != 0, resets) the flags for `device`.  Synchronizes the
 * device.  Flag bits: 1 tile wait, 2 stage wait, 4 accumulator wait, 8 accumulator
 * release wait, 16 teardown drain, 32 TMEM allocation, 64 injected test timeout.
 */
CTU_API int ctu_get_device_error(int device, uint32_t *flags, int clear);

/*
 * ConvRot rotate + per-token quantize of a bf16 activation.
 *   x      bf16 [rows, k] (act NONE / GELU_TANH) or [rows, 2k] (act SWIGLU), row-major,
 *          16-byte aligned
 *   codes  bits = 8: int8 [rows, k]; bits = 4: packed int4 [rows, k/2], even column in
 *          the low nibble; 16-byte aligned
 *   scales fp32 [rows]
 * k must be a positive multiple of 256 (the rotation group).
 * Replaces turing_utils::bf16_int8_convrot_quantize / bf16_int4_convrot_quantize
 * (kernel/comfyui_turing_utils_kernel/ops.py:290-343; kernel/csrc/bindings.cpp:636-717;
 * kernel/csrc/turing/convrot_quant.cu:417-511,665-713) and, with act = GELU_TANH, the
 * bf16_gelu_* variants (ops.py:346-385; convrot_quant.cu:715-745).
 */
CTU_API int ctu_convrot_quantize(const void *x, int64_t rows, int64_t k, int act, int bits, int8_t *codes, float *scales,
                         void *stream);

/*
 * ConvRot int8 quantize with rotation block 128 (the block size the benchmark's configs
 * name; the reference's ops accept 256 only -- dispatch.py:765, convrot_quant.cu:24 -- so
 * this rotation is this library's definition, parity unpinned): each 128-column block is
 * rotated by (1/sqrt 2) H2 (x) M (x) M (x) M, evaluated as the reference's radix-4 stages at
 * strides 1, 4, 16 followed by a radix-2 stage at stride 64,
 *   y0 = (x0 + x1) * c,  y1 = (x0 - x1) * c,  c = RN_fp32(1/sqrt 2),
 * then quantized with the int8 chain of ctu_convrot_quantize (per-row scale absmax / 127).
 *   x bf16 [rows, k] (k % 256 == 0, k <= 32768), codes int8 [rows, k], scales fp32 [rows].
 */
CTU_API int ctu_convrot_quantize_b128(const void *x, int64_t rows, int64_t k, int8_t *codes, float *scales,
                                      void *stream);

/*
 * The staged quantizers (replace turing_swiglu_int{8,4}_convrot_quantize and
 * turing_gelu_int{8,4}_convrot_quantize, kernel/csrc/bindings.cpp:474-633 ->
 * kernel/csrc/turing/convrot_quant.cu:184-358, 577-663): ctu_convrot_quantize with the
 * staged kernels' per-row scale max(min(absmax, BF16_MAX) * (1/qmax), floor) -- a
 * multiplication by the fp32 constant 1/qmax where the row-buffer kernel divides, so
 * some rows' scales (and rarely codes) differ from ctu_convrot_quantize's.  act must be
 * CTU_ACT_SWIGLU or CTU_ACT_GELU_TANH for dtype CTU_DTYPE_FP16 (like the reference, fp16
 * rows round the rotated values, the scale and the quotient to fp16 and clamp at
 * 65504); otherwise the same arguments and constraints as ctu_convrot_quantize.
 */
CTU_API int ctu_convrot_quantize_staged(const void *x, int64_t rows, int64_t k, int act, int bits, int dtype,
                                        int8_t *codes, float *scales, void *stream);

/*
 * SwiGLU + ConvRot rotate of one channel shard, quantized to int8 with caller-supplied
 * per-row scales (the whole row's scales, computed over every shard beforehand):
 *   x      bf16 or fp16 (dtype CTU_DTYPE_BF16 / CTU_DTYPE_FP16) [rows, 2k] (gate | up
 *          halves of the shard), 16-byte aligned
 *   scales fp32 [rows], read only
 *   codes  int8 [rows, k], 16-byte aligned
 * code = clamp(rint(T(T(y) / T(scale))), -128, 127), T the input type, as the unscaled op.
 * k must be a positive multiple of 256.
 * Replaces turing_utils::swiglu_int8_convrot_quantize_scaled (ops.py:189-219;
 * bindings.cpp:512-545; convrot_quant.cu:138-161,239-278,591-621).
 */
CTU_API int ctu_swiglu_int8_convrot_quantize_scaled(const void *x, int64_t rows, int64_t k, int dtype,
                                                    const float *scales, int8_t *codes, void *stream);

/*
 * W8A8 linear with the fused dequant + bias epilogue:
 *   out[m, n] = bf16(fma(float(sum_k a[m,k] * w[n,k]) * a_scale[m], w_scale[n], bias[n]))
 * (the weight-scale multiply and the bias add as one fma, as the reference's build
 * contracts them; a null bias adds +0)
 *   a int8 [m, k], w int8 [n, k] (K-contiguous rows), a_scale fp32 [m],
 *   w_scale fp32 [n] (w_scale_count = n) or a scalar (w_scale_count = 1),
 *   bias fp32 [n] or NULL, out bf16 [m, n].
 * Requires k % 16 == 0, n % 8 == 0, a/w/out 16-byte aligned.
 * Replaces turing_utils::int8_linear (ops.py:96-126; bindings.cpp:371-421;
 * kernel/csrc/turing/w4a8.cu:1185-1219, CUTLASS SM75 GEMM w4a8.cu:376-618).
 */
CTU_API int ctu_int8_linear(const int8_t *a, const int8_t *w, const float *a_scale, const float *w_scale,
                    int64_t w_scale_count, const float *bias, void *out, int64_t m, int64_t n, int64_t k,
                    void *stream);

/*
 * ConvRot W8A8 linear from bf16 rows in one call: ctu_convrot_quantize(x, m, k, NONE, 8,
 * codes, scales) followed by ctu_int8_linear(codes, w, scales, w_scale, ..., out), with
 * the same codes, scales and outputs bit for bit.  Replaces the plugin's
 * dispatch.int8_linear for plain ConvRot W8A8 rows (comfyui_turing_utils/quantization/
 * dispatch.py:748-800: _quantize_turing_int8_activation, then turing_int8_linear).
 *   x bf16 [m, k] (k % 256 == 0), w int8 [n, k], w_scale fp32 [n] or scalar, bias fp32 [n]
 *   or NULL, out bf16 [m, n]; codes int8 [m, k] and scales fp32 [m] receive the quantized
 *   activation; sync is a workspace of ctu_convrot_int8_linear_sync_words(m) uint32 words
 *   (4-byte aligned; cleared on the stream by the call).
 * For k <= 5120, n <= 8192 and m >= 16384 one kernel does both: quantizer warps inside the
 * CTA-pair GEMM publish each finished 128-row block and the GEMM loads a block once it is
 * complete, so the rotation of later rows overlaps the tensor-core work on earlier ones.
 * Otherwise (where that measured slower) the quantizer and the GEMM run back to back.
 * Requires n % 8 == 0 and 16-byte aligned x, w, codes and out.
 */
CTU_API int ctu_convrot_int8_linear(const void *x, const int8_t *w, const float *w_scale, int64_t w_scale_count,
                                    const float *bias, void *out, int8_t *codes, float *scales, uint32_t *sync,
                                    int64_t m, int64_t n, int64_t k, void *stream);

/* Words of the sync workspace ctu_convrot_int8_linear needs for m rows:
 * 1 + ceil(m / 128). */
CTU_API int64_t ctu_convrot_int8_linear_sync_words(int64_t m);

/*
 * W4A8 linear: as ctu_int8_linear, with signed 4-bit weights packed two per byte,
 *   w_packed int8 [n, k/2], byte j of a row = k 2j (low nibble) and 2j+1 (high nibble),
 *   each nibble two's-complement in [-8, 7].  The packed tile is sign-extended to int8
 *   in shared memory ahead of the int8 tensor-core MMA.
 * Requires k % 32 == 0, n % 8 == 0, a/w_packed/out 16-byte aligned.
 * Replaces turing_utils::w4a8_linear (ops.py:8-35; bindings.cpp:167-260;
 * kernel/csrc/turing/w4a8.cu:1000-1086 with TuringW4ToS8 w4a8.cu:34-72).
 */
CTU_API int ctu_w4a8_linear(const int8_t *a, const int8_t *w_packed, const float *a_scale, const float *w_scale,
                            int64_t w_scale_count, const float *bias, void *out, int64_t m, int64_t n, int64_t k,
                            void *stream);

/*
 * W4A4 linear: both operands signed 4-bit, packed two per byte (even k in the low
 * nibble): a_packed [m, k/2] (the int4 ConvRot codes of ctu_convrot_quantize(bits=4)),
 * w_packed [n, k/2]; per-token activation scale [m], per-channel weight scale [n] or
 * scalar, optional bias; same epilogue as ctu_int8_linear.  Both tiles are
 * sign-extended to int8 in shared memory ahead of the int8 tensor-core MMA.
 * Requires k % 32 == 0, n % 8 == 0, 16-byte aligned operands.
 * Replaces the int4 GEMM the reference takes from comfy-kitchen for
 * convrot_w4a4_linear(linear_dtype="int4") (comfyui_turing_utils/quantization/
 * dispatch.py:916-934, kitchen int4_linear; third-party source, not in the reference).
 */
CTU_API int ctu_w4a4_linear(const int8_t *a_packed, const int8_t *w_packed, const float *a_scale, const float *w_scale,
                            int64_t w_scale_count, const float *bias, void *out, int64_t m, int64_t n, int64_t k,
                            void *stream);

/*
 * Raw W8A8 contraction to int32: acc[m, n] (row stride ldc elements) = sum_k a[m,k] * w[n,k].
 * Same alignment rules as ctu_int8_linear; ldc % 4 == 0.
 * Replaces the int32 GEMM the reference takes from comfy-kitchen's cuBLAS binding
 * (comfyui_turing_utils/quantization/dispatch.py:559-613, cublas_gemm_int8).
 */
CTU_API int ctu_int8_gemm_s32(const int8_t *a, const int8_t *w, int32_t *acc, int64_t ldc, int64_t m, int64_t n, int64_t k,
                      void *stream);

/*
 * Grouped-codebook W4A8 linear:
 *   w[n, c] = clamp(rint(codebook[code] * e4m3(group_scale[n, c / group_size])), -127, 127)
 *   out[m, n] = bf16(fma(float(sum_c a[m, c] * w[n, c]) * a_scale[m], channel_scale[n], bias[n]))
 *   a            int8 [m, k]; w_packed: 4-bit codes [n, k/2], even column in the low nibble
 *   group_scale  float8 e4m3fn bytes [n, k / group_size]; codebook fp32 [16]
 *   channel_scale fp32 [n]; bias fp32 [n] or NULL; out bf16 [m, n]
 *   workspace    int8 [workspace_rows, k]: output channels are decoded workspace_rows at a
 *                time (a multiple of 8) and each chunk runs the W8A8 tensor-core GEMM.
 * Requires k % 16 == 0, n % 8 == 0, group_size >= 4 dividing k with 16 % group_size == 0
 * or group_size % 16 == 0; a, w_packed, out and workspace 16-byte aligned.
 * Replaces turing_utils::codebook_w4a8_linear (ops.py:38-93; bindings.cpp:262-370;
 * kernel/csrc/turing/w4a8.cu:89-242, 903-976, 1088-1182).
 */
CTU_API int ctu_codebook_w4a8_linear(const int8_t *a, const int8_t *w_packed, const float *a_scale,
                                     const uint8_t *group_scale, const float *channel_scale, const float *codebook,
                                     const float *bias, void *out, int8_t *workspace, int64_t workspace_rows,
                                     int64_t m, int64_t n, int64_t k, int64_t group_size, void *stream);

/*
 * The codebook decode alone: int8 [rows, k] from w_packed [rows, k/2], group_scale
 * [rows, k / group_size] and codebook [16], as in ctu_codebook_w4a8_linear.  Replaces the
 * reference's internal staged decode (w4a8.cu:903-976), which has no public entry.
 */
CTU_API int ctu_codebook_decode_s8(const int8_t *w_packed, const uint8_t *group_scale, const float *codebook,
                                   int8_t *out, int64_t rows, int64_t k, int64_t group_size, void *stream);

/*
 * Packed signed int4 [rows, k/2] (even column in the low nibble, w4a8.cu:34-72) widened
 * to int8 [rows, k].  k % 32 == 0; both tensors 16-byte aligned.  The W4 linears of the
 * op layer use it at long sequences (widen, then ctu_int8_linear).  No reference
 * counterpart (the reference widens inside its GEMM's shared-memory fill).
 */
CTU_API int ctu_int4_unpack_s8(const int8_t *packed, int8_t *out, int64_t rows, int64_t k, void *stream);

/*
 * Per-group (128 columns of K) formats.  The reference has no kernel or checkpoint layout
 * for them: its W4A4 path (comfyui_turing_utils/quantization/dispatch.py:876-936) hands
 * int4 activations to comfy-kitchen's int4_linear (not in the reference) with 64-column
 * weight groups, and its asymmetric W4A8 format (asym_w4a8_int8, AsymW4A8Int8Layout,
 * fusions.py:14-16) is the grouped codebook of ctu_codebook_w4a8_linear.  The arithmetic
 * below is this library's definition (parity unpinned).
 *
 * ctu_convrot_quantize_int4_g128: the ConvRot rotation of ctu_convrot_quantize (bf16 x
 * [rows, k], k % 256 == 0), then every 128 columns of each rotated row quantized on
 * their own with the int4 chain: group_scales[r, g] = max(min(absmax, bf16 max) / 7,
 * 1e-10), codes [rows, k/2] packed (even column in the low nibble) =
 * clamp(rint(bf16(y) * (1 / scale)), -7, 7).  group_scales is fp32 [rows, k/128].
 */
CTU_API int ctu_convrot_quantize_int4_g128(const void *x, int64_t rows, int64_t k, int8_t *codes,
                                           float *group_scales, void *stream);

/* ctu_convrot_quantize_int4_g128 with the block-128 rotation of ctu_convrot_quantize_b128
 * (each 128-column block rotated on its own, then scaled and quantized on its own). */
CTU_API int ctu_convrot_quantize_int4_g128_b128(const void *x, int64_t rows, int64_t k, int8_t *codes,
                                                float *group_scales, void *stream);

/*
 * Asymmetric uint4 W4A8: a int8 [m, k] with per-token a_scale [m]; w_packed uint8
 * [n, k/2] (nibbles 0..15, even column in the low nibble) with, per 128 columns, a zero
 * point w_zero uint8 [n, k/128] (0..15) and a scale given group-major as fp32
 * w_scale_gn [k/128, n] (the checkpoint's fp16 scales widened).  With acc_g the exact
 * int32 sum over group g of a[m, c] * (nibble[n, c] - zero[n, g]):
 *   t = 0; for g in order: t = fma(w_scale_gn[g, n], float(acc_g), t)
 *   out[m, n] = bf16(fma(t, a_scale[m], bias[n]))          (null bias: +0)
 * w_workspace: int8 [n, k], 16-byte aligned (the widened weights).  k % 128 == 0,
 * n % 8 == 0.
 */
CTU_API int ctu_asym_w4a8_g128_linear(const int8_t *a, const uint8_t *w_packed, const float *a_scale,
                                      const float *w_scale_gn, const uint8_t *w_zero, const float *bias, void *out,
                                      int8_t *w_workspace, int64_t m, int64_t n, int64_t k, void *stream);

/*
 * W4A4 with per-token-per-group activation scales: a_packed / w_packed signed int4
 * [m, k/2] / [n, k/2] (even column in the low nibble), a_scale_mg fp32 [m, k/128] (as
 * written by ctu_convrot_quantize_int4_g128), w_scale_gn fp32 [k/128, n]:
 *   t = 0; for g in order: t = fma(float(acc_g) * a_scale_mg[m, g], w_scale_gn[g, n], t)
 *   out[m, n] = bf16(t + bias[n])                          (null bias: +0)
 * a_workspace int8 [m, k] and w_workspace int8 [n, k] receive the sign-extended
 * operands.  k % 128 == 0, n % 8 == 0.
 */
CTU_API int ctu_w4a4_g128_linear(const int8_t *a_packed, const int8_t *w_packed, const float *a_scale_mg,
                                 const float *w_scale_gn, const float *bias, void *out, int8_t *a_workspace,
                                 int8_t *w_workspace, int64_t m, int64_t n, int64_t k, void *stream);

/*
 * Affine RMSNorm + segmented AdaLN (replaces turing_segmented_rms_adaln,
 * kernel/csrc/bindings.cpp:767-834 -> kernel/csrc/turing/segmented_rms_adaln.cu:133-232,
 * 288-340).  out[r, c] = ((x[r, c] * rsqrt(mean(x[r]^2) + epsilon)) * weight[c])
 * * (1 + scale[m, c]) + shift[m, c], where m is the modulation row of the segment
 * (start, stop, row) of `segments` that holds r (row 0 when none does or when the row is
 * outside [0, param_rows)).  x and out are [rows, hidden]; scale and shift rows lie
 * scale_stride / shift_stride elements apart.  dtype is CTU_DTYPE_*, the type of every
 * floating tensor.  Bit-identical to the reference for the same inputs, including its
 * choice between 16-byte vector and per-element order (by alignment and strides).
 */
CTU_API int ctu_segmented_rms_adaln(const void *x, const void *weight, const void *scale, int64_t scale_stride,
                                    const void *shift, int64_t shift_stride, const int32_t *segments,
                                    int64_t segment_count, void *out, int64_t rows, int64_t hidden,
                                    int64_t param_rows, float epsilon, int dtype, void *stream);

/*
 * LayerNorm (no affine) + Wan AdaLN (replaces turing_layer_norm_adaln,
 * kernel/csrc/bindings.cpp:836-880 -> kernel/csrc/turing/segmented_rms_adaln.cu:234-297,
 * 365-407).  x and out are [batch, sequence, hidden]; scale and shift are
 * [batch, modulation_steps, hidden]; token t of a batch uses modulation step
 * min(t / g, modulation_steps - 1), g = sequence / modulation_steps (integer division),
 * plus one when that does not divide sequence evenly.  out = round(round(normalized) *
 * round(1 + scale) + shift), each round to the storage type.
 */
CTU_API int ctu_layer_norm_adaln(const void *x, const void *scale, const void *shift, void *out, int64_t batch,
                                 int64_t sequence, int64_t hidden, int64_t modulation_steps, float epsilon,
                                 int dtype, void *stream);

/*
 * int32 accumulator -> bf16: out[r, c] = bf16((float(acc[r, c]) * a_scale[r]) * w_scale[c]),
 * acc row stride acc_stride (>= cols), w_scale [cols] or scalar (w_scale_count = 1),
 * out bf16 [rows, cols] contiguous.
 * Replaces turing_utils::dequantize_int8_bf16 (ops.py:129-160; bindings.cpp:423-472;
 * kernel/csrc/turing/bf16_epilogue.cu:146-217).
 */
CTU_API int ctu_dequantize_int8_bf16(const int32_t *acc, int64_t acc_stride, const float *a_scale, const float *w_scale,
                             int64_t w_scale_count, void *out, int64_t rows, int64_t cols, void *stream);

/*
 * ConvRot W8A8 linear in one call that allocates no device memory (no counterpart in
 * the reference).  For callers that cannot call cudaMalloc -- code inside a region
 * where allocation is forbidden or would break a pre-reserved memory pool, or hosts
 * without an allocator: the quantized activation (int8 codes and fp32 per-token
 * scales) and the kernels' error word live in a file-scope device array of the
 * library (16 MiB of codes + 65536 scales, held by every GPU that loads the library
 * until exit) instead of caller- or library-allocated buffers.
 *   x bf16 [m, k] (k % 256 == 0), w int8 [n, k] (n % 8 == 0), w_scale [n] or scalar,
 *   bias fp32 [n] or NULL, out bf16 [m, n]; same numerics as ctu_convrot_quantize
 *   followed by ctu_int8_linear.
 * Rejects m * k > 16 MiB or m > 65536.  All calls on a device share the array: calls
 * that can overlap on the GPU race and must be ordered.  The first call on each
 * device resolves the array's address (cudaGetSymbolAddress) and clears the error
 * word; make it before any stream capture.
 */
CTU_API int ctu_convrot_w8a8_linear_static_scratch(const void *x, const int8_t *w, const float *w_scale,
                                                   int64_t w_scale_count, const float *bias, void *out, int64_t m,
                                                   int64_t n, int64_t k, void *stream);

/* Test hook: launch the GEMM with its MMA issuer waiting on a barrier nothing arrives
 * on, bounded by timeout_ns; the kernel must stop cleanly and raise flag 64. */
CTU_API int ctu_debug_gemm_injected_timeout(const int8_t *a, const int8_t *w, int32_t *acc, int64_t m, int64_t n, int64_t k,
                                    uint64_t timeout_ns, void *stream);

/* Test hook (no counterpart in the reference): choose the integer GEMM kernel for
 * every later call in this process.  0 = per problem (default: the CTA-pair kernel
 * when M > 128; the single-CTA tiling for the per-group-128 linears), 1 = single-CTA
 * kernel, 2 = CTA-pair kernel (both also for the per-group-128 linears).  Returns the
 * previous selector, or a negative error code. */
CTU_API int ctu_debug_set_gemm_kernel(int which);

/* Test hook (no counterpart in the reference): how ctu_convrot_int8_linear runs.  0 = per
 * problem (default; see ctu_convrot_int8_linear), 1 = always the separate quantizer and
 * GEMM, 2 = the fused kernel wherever it applies (k <= 5120, more than 128 rows).  Returns
 * the previous setting, or a negative error code. */
CTU_API int ctu_debug_set_fused_linear(int which);

/* Test hook (no counterpart in the reference): how many of the last 256 x 256 output tiles
 * the CTA-pair W8A8 GEMM runs as two 256 x 128 halves, for every later call in this
 * process.  -1 = per problem (default: the last round's tiles when that halves the last
 * round), 0 = never, n > 0 = the last n tiles.  Returns the previous setting, or a
 * negative error code. */
CTU_API int ctu_debug_set_gemm_split(int tiles);

/* Test hook (no counterpart in the reference): choose the ConvRot quantizer for every
 * later call in this process.  0 = per width (the library's measured choice; see
 * ctu_debug_quant_plan), 1 = two-pass kernel, 2 = register-resident kernel, 3 = four-lane
 * kernel, 4 = eight-lane kernel, 5 = multi-group eight-lane kernel (groups per team
 * chosen per width), 6 / 7 = multi-group eight-lane kernel with 1 / 2 groups per team,
 * 8 = warp-row kernel (plain and GELU rows of at most 24 groups), all but the first
 * wherever the width allows them.  Returns the previous selector, or a negative error
 * code. */
CTU_API int ctu_debug_set_quant_kernel(int which);

/* Test hook (host only, no GPU needed): the quantizer plan a call of width k would use on a
 * device with `smem_optin` bytes of opt-in shared memory per block, under the current
 * selector: kind 0 = two-pass, 1 = register-resident, 2 = four-lane, 3 = eight-lane,
 * 4 = multi-group eight-lane; the CTA's warps and rows per batch. */
CTU_API int ctu_debug_quant_plan(int64_t k, int act, int bits, int smem_optin, int *kind, int *warps,
                                 int *rows_per_batch);

#ifdef __cplusplus
}
#endif

#endif /* CTU_B200_H_ */
