/*
 * CPU oracle for the ConvRot quantized-linear path.  TEST INFRASTRUCTURE ONLY:
 * nothing in the shipped library links or calls this file.  It is imported by
 * tests/, by __graft_entry__.smoke() as the checker, and by bench.py's
 * cpu_baseline leg / `--impl reference` arm.
 *
 * It restates, in plain C with IEEE single precision and no FMA contraction
 * (built with -ffp-contract=off, no -ffast-math), the arithmetic of the
 * reference kernels of comfyui-turing-utils (kernel package 0.31.0):
 *
 *   kernel/csrc/turing/convrot_quant.cu:104-116   radix-4 stage, fp32 order
 *   kernel/csrc/turing/convrot_quant.cu:444-473   stage order S = 1, 4, 16, 64
 *   kernel/csrc/turing/convrot_quant.cu:360-376   fp32 -> bf16 RNE, NaN -> 0x7fff
 *   kernel/csrc/turing/convrot_quant.cu:378-397   bf16 store of y, fp32 absmax
 *   kernel/csrc/turing/convrot_quant.cu:475-510   per-token scale and codes
 *   kernel/csrc/turing/convrot_quant.cu:163-182   SwiGLU / tanh-GELU loaders
 *   kernel/csrc/turing/w4a8.cu:474-525            epilogue ((acc*a_s)*w_s)+bias
 *   kernel/csrc/turing/bf16_epilogue.cu:105-113   epilogue (acc*a_s)*w_s
 *   kernel/csrc/turing/w4a8.cu:34-72              signed int4, low nibble first
 *   kernel/csrc/turing/segmented_rms_adaln.cu:75-232   RMSNorm + segmented AdaLN
 *   kernel/csrc/turing/segmented_rms_adaln.cu:82-107,234-297  LayerNorm + AdaLN
 *
 * The norms reproduce the reference's reduction tree exactly (per-thread
 * partials over the 256-thread row mapping, the shfl_down warp tree, the
 * in-order combine of 8 warps) with the contractions nvcc makes by default
 * (a += b*c -> fma).  The one step this file cannot reproduce bit for bit is
 * the device rsqrtf (a hardware approximation, max 2 ulp per the CUDA
 * Programming Guide); here it is the correctly rounded 1/sqrt.  Tests of the
 * norms against this file therefore allow one output ulp where the inverse
 * differs, and pin the device kernels bit for bit to fixtures produced by the
 * reference kernels themselves.
 *
 * The int32 contraction itself is exact integer arithmetic and lives in the
 * Python wrapper (torch._int_mm / numpy).
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define KGROUP 256

static inline uint32_t f2u(float v) { uint32_t u; memcpy(&u, &v, 4); return u; }
static inline float u2f(uint32_t u) { float v; memcpy(&v, &u, 4); return v; }

/* convrot_quant.cu:360-372: round to nearest even, any NaN -> 0x7fff. */
uint16_t ctu_oracle_f32_to_bf16(float value) {
    const uint32_t bits = f2u(value);
    if ((bits & 0x7fffffffu) > 0x7f800000u) return 0x7fffu;
    uint16_t upper = (uint16_t)(bits >> 16);
    const uint32_t rem = bits << 16;
    if (rem > 0x80000000u || (rem == 0x80000000u && (upper & 1u))) ++upper;
    return upper;
}

static inline float bf16_to_f32(uint16_t v) { return u2f((uint32_t)v << 16); }
static inline float round_bf16(float v) { return bf16_to_f32(ctu_oracle_f32_to_bf16(v)); }

/* convrot_quant.cu:104-116 for one stride S over a 256-group, out of place.
 * Lane l of the reference's 64-thread group owns base = l%S + (l/S)*4S. */
static void fht_stage(const float *src, float *dst, int S) {
    for (int lane = 0; lane < 64; ++lane) {
        const int base = (lane % S) + (lane / S) * (4 * S);
        const float x0 = src[base], x1 = src[base + S];
        const float x2 = src[base + 2 * S], x3 = src[base + 3 * S];
        dst[base] = 0.5f * (x0 + x1 + x2 - x3);
        dst[base + S] = 0.5f * (x0 + x1 - x2 + x3);
        dst[base + 2 * S] = 0.5f * (x0 - x1 + x2 + x3);
        dst[base + 3 * S] = 0.5f * (-x0 + x1 + x2 + x3);
    }
}

/* The 4-stage radix-4 rotation of one 256-group (strides 1, 4, 16, 64). */
void ctu_oracle_rotate_group(const float *in, float *out) {
    float a[KGROUP], b[KGROUP];
    fht_stage(in, a, 1);
    fht_stage(a, b, 4);
    fht_stage(b, a, 16);
    fht_stage(a, out, 64);
}

/* convrot_quant.cu:163-169: silu(gate) * up in fp32 with the accurate expf. */
static inline float swiglu_value(float gate, float up) {
    return (gate / (1.0f + expf(-gate))) * up;
}

/* convrot_quant.cu:171-182: tanh-GELU in fp32, rounded to the input dtype.
 * The reference is compiled with nvcc's default FMA contraction; the two
 * products feeding an addition are contracted exactly as written here with
 * fmaf so the C restatement follows the device's evaluation. */
static inline float gelu_tanh_activated(float x, int contract) {
    const float kAlpha = 0.7978845608028654f;
    const float kBeta = 0.044715f;
    float inner;
    if (contract) {
        inner = fmaf((kBeta * x) * x, x, x);
    } else {
        inner = x + ((kBeta * x) * x) * x;
    }
    const float t = tanhf(kAlpha * inner);
    return (0.5f * x) * (1.0f + t);
}

static inline float gelu_tanh_value(float x, int contract) { return round_bf16(gelu_tanh_activated(x, contract)); }

/*
 * Rotate one activation row and return the fp32 absmax over the rotated
 * (unrounded) values, writing bf16(y) into ybits.  `mode`: 0 = plain bf16 row of
 * k values, 1 = SwiGLU row of 2k values [gate | up], 2 = tanh-GELU row, 3 = GELU
 * evaluated without contraction.
 */
static float rotate_row(const uint16_t *row, int k, int mode, uint16_t *ybits, float *yf) {
    float absmax = 0.0f;
    float in[KGROUP], out[KGROUP];
    for (int g = 0; g < k / KGROUP; ++g) {
        for (int i = 0; i < KGROUP; ++i) {
            const int col = g * KGROUP + i;
            float v;
            if (mode == 1) {
                v = swiglu_value(bf16_to_f32(row[col]), bf16_to_f32(row[k + col]));
            } else if (mode == 2 || mode == 3) {
                v = gelu_tanh_value(bf16_to_f32(row[col]), mode == 2);
            } else {
                v = bf16_to_f32(row[col]);
            }
            in[i] = v;
        }
        ctu_oracle_rotate_group(in, out);
        for (int i = 0; i < KGROUP; ++i) {
            const float y = out[i];
            ybits[g * KGROUP + i] = ctu_oracle_f32_to_bf16(y);
            if (yf) yf[g * KGROUP + i] = y;
            /* convrot_quant.cu:396: fmaxf(fmaxf(|y0|,|y1|), fmaxf(|y2|,|y3|)),
             * fmaxf ignores NaN, so the reduction order is immaterial. */
            absmax = fmaxf(absmax, fabsf(y));
        }
    }
    return absmax;
}

/* Rotated values only (fp32), for the rotation parity checks. */
void ctu_oracle_rotate(const uint16_t *x, float *y, long rows, int k, int mode) {
    const int width = mode == 1 ? 2 * k : k;
#pragma omp parallel
    {
        uint16_t ybits[65536];
#pragma omp for schedule(static)
        for (long r = 0; r < rows; ++r) {
            if (k <= 65536) rotate_row(x + r * width, k, mode, ybits, y + r * (long)k);
        }
    }
}

/* The per-row scale.  The row-buffer kernel divides the clamped absmax by qmax
 * (convrot_quant.cu:475-478); the staged kernels multiply it by the fp32 constant
 * 1/qmax (convrot_quant.cu:300-303, 335-338), which can round differently. */
static float row_scale(float absmax, int bits, int staged) {
    const float clamped = fminf(absmax, 3.38953139e38f);
    if (bits == 4) return fmaxf(staged ? clamped * (1.0f / 7.0f) : clamped / 7.0f, 1.0e-10f);
    return fmaxf(staged ? clamped * (1.0f / 127.0f) : clamped / 127.0f, 1.0e-30f);
}

/* convrot_quant.cu:475-510, int8 branch. */
static void quantize_row_int8(const uint16_t *ybits, int k, float absmax, int8_t *codes, float *scale_out,
                              int staged) {
    const float scale = row_scale(absmax, 8, staged);
    *scale_out = scale;
    const float rounded_scale = round_bf16(scale);
    for (int c = 0; c < k; ++c) {
        const float value = bf16_to_f32(ybits[c]);
        const float divided = round_bf16(value / rounded_scale);
        float q = nearbyintf(divided);
        q = fminf(127.0f, fmaxf(-128.0f, q));
        codes[c] = (int8_t)q;
    }
}

/* convrot_quant.cu:475-500, int4 branch: multiply by the fp32 reciprocal of the
 * unrounded scale, clamp to [-7, 7], pack the even column in the low nibble. */
static void quantize_row_int4(const uint16_t *ybits, int k, float absmax, int8_t *packed, float *scale_out,
                              int staged) {
    const float scale = row_scale(absmax, 4, staged);
    *scale_out = scale;
    const float inv_scale = 1.0f / scale;
    for (int p = 0; p < k / 2; ++p) {
        float lo = nearbyintf(bf16_to_f32(ybits[2 * p]) * inv_scale);
        float hi = nearbyintf(bf16_to_f32(ybits[2 * p + 1]) * inv_scale);
        lo = fminf(7.0f, fmaxf(-7.0f, lo));
        hi = fminf(7.0f, fmaxf(-7.0f, hi));
        const uint8_t lb = (uint8_t)(int8_t)lo & 0x0f;
        const uint8_t hb = (uint8_t)(int8_t)hi & 0x0f;
        packed[p] = (int8_t)(lb | (hb << 4));
    }
}

/*
 * Whole-row ConvRot quantize (the reference's bf16 row-buffer kernel,
 * convrot_quant.cu:417-511).  x: rows x (mode==1 ? 2k : k) bf16 bit patterns.
 * bits = 8: codes rows x k int8; bits = 4: rows x k/2 packed int4.  Returns 0, or
 * -1 on an unsupported k.
 */
/* turing_swiglu_int8_convrot_quantize_scaled (convrot_quant.cu:138-161, 239-278):
 * rotate each row as ctu_oracle_convrot_quantize does and quantize with the caller's
 * scale instead of the row's absmax:
 *   code = clamp(rint(bf16(bf16(y) / bf16(scale))), -128, 127). */
static void quantize_row_int8_given(const uint16_t *ybits, int k, float scale, int8_t *codes) {
    const float rounded_scale = round_bf16(scale);
    for (int c = 0; c < k; ++c) {
        const float value = bf16_to_f32(ybits[c]);
        const float divided = round_bf16(value / rounded_scale);
        float q = nearbyintf(divided);
        q = fminf(127.0f, fmaxf(-128.0f, q));
        codes[c] = (int8_t)q;
    }
}

int ctu_oracle_convrot_quantize_scaled(const uint16_t *x, const float *scales, int8_t *codes,
                                       long rows, int k, int mode) {
    if (k <= 0 || k % KGROUP != 0 || k > 65536) return -1;
    const int width = mode == 1 ? 2 * k : k;
#pragma omp parallel
    {
        uint16_t ybits[65536];
#pragma omp for schedule(static)
        for (long r = 0; r < rows; ++r) {
            (void)rotate_row(x + r * width, k, mode, ybits, 0);
            quantize_row_int8_given(ybits, k, scales[r], codes + r * k);
        }
    }
    return 0;
}

static int convrot_quantize(const uint16_t *x, int8_t *codes, float *scales, long rows, int k, int bits, int mode,
                            int staged) {
    if (k <= 0 || k % KGROUP != 0 || k > 65536) return -1;
    const int width = mode == 1 ? 2 * k : k;
    const int out_width = bits == 4 ? k / 2 : k;
#pragma omp parallel
    {
        uint16_t ybits[65536];
#pragma omp for schedule(static)
        for (long r = 0; r < rows; ++r) {
            const float absmax = rotate_row(x + r * width, k, mode, ybits, 0);
            if (bits == 4) {
                quantize_row_int4(ybits, k, absmax, codes + r * out_width, scales + r, staged);
            } else {
                quantize_row_int8(ybits, k, absmax, codes + r * out_width, scales + r, staged);
            }
        }
    }
    return 0;
}

int ctu_oracle_convrot_quantize(const uint16_t *x, int8_t *codes, float *scales,
                                long rows, int k, int bits, int mode) {
    return convrot_quantize(x, codes, scales, rows, k, bits, mode, 0);
}

/* The staged quantizers (turing_swiglu_int{8,4}_convrot_quantize, turing_gelu_int{8,4}_
 * convrot_quantize; convrot_quant.cu:184-358, 577-663): the same rotation and codes
 * with the multiply-by-reciprocal row scale. */
int ctu_oracle_convrot_quantize_staged(const uint16_t *x, int8_t *codes, float *scales,
                                       long rows, int k, int bits, int mode) {
    return convrot_quantize(x, codes, scales, rows, k, bits, mode, 1);
}

/*
 * Epilogue over an int32 accumulator (row stride acc_stride), w4a8.cu:474-525:
 * out = bf16(((float(acc) * a_s[m]) * w_s[n]) + bias[n]).  `fused` selects a
 * single-rounding fma for the last multiply-add, which is what the reference's
 * build produces (nvcc's default FMA contraction of the bias node inlined after
 * the scale node; checked element by element against the reference kernels);
 * `has_bias` = 0 reproduces bf16_epilogue.cu:105-113 (no addition at all).
 * w_scale_count = 1 broadcasts a scalar weight scale.
 */
void ctu_oracle_epilogue(const int32_t *acc, long acc_stride, const float *a_scale,
                         const float *w_scale, long w_scale_count, const float *bias,
                         uint16_t *out, long m, long n, int has_bias, int fused) {
#pragma omp parallel for schedule(static)
    for (long i = 0; i < m; ++i) {
        const float as = a_scale[i];
        for (long j = 0; j < n; ++j) {
            const float ws = w_scale[w_scale_count == 1 ? 0 : j];
            const float scaled = (float)acc[i * acc_stride + j] * as;
            float v;
            if (!has_bias) {
                v = scaled * ws;
            } else if (fused) {
                v = fmaf(scaled, ws, bias[j]);
            } else {
                const float t = scaled * ws;
                v = t + bias[j];
            }
            out[i * n + j] = ctu_oracle_f32_to_bf16(v);
        }
    }
}


/* ---------------------------------------------------------------------------------
 * Rotation block 128 (the benchmark's configs[0]-[3] name it; the reference's ops accept
 * 256 only, dispatch.py:765, convrot_quant.cu:24, so this is this build's definition and
 * its parity is UNPINNED).  The 128-point rotation is (1/sqrt 2) H2 (x) M (x) M (x) M with
 * M the reference's radix-4 stage (fht_stage): the three radix-4 stages at strides 1, 4
 * and 16 exactly as the reference evaluates them, then one radix-2 stage at stride 64,
 *   y0 = (x0 + x1) * c,  y1 = (x0 - x1) * c,  c = RN_fp32(1/sqrt 2) = 0x1.6a09e6p-1,
 * each operation rounded to fp32.  The radix-2 stage comes last so that it stays inside
 * one lane of the GPU kernels' layout.  A 256-column group holds two independent
 * 128-blocks.  Codes and scales follow the int8 chain of the 256 rotation.
 * --------------------------------------------------------------------------------- */
#define RSQRT2_F32 0x1.6a09e6p-1f

void ctu_oracle_rotate_group_b128(const float *in, float *out) {
    float a[KGROUP], b[KGROUP];
    fht_stage(in, a, 1);
    fht_stage(a, b, 4);
    fht_stage(b, a, 16);
    for (int blk = 0; blk < KGROUP; blk += 128) {
        for (int i = 0; i < 64; ++i) {
            const float x0 = a[blk + i], x1 = a[blk + 64 + i];
            out[blk + i] = (x0 + x1) * RSQRT2_F32;
            out[blk + 64 + i] = (x0 - x1) * RSQRT2_F32;
        }
    }
}

int ctu_oracle_convrot_quantize_b128(const uint16_t *x, int8_t *codes, float *scales, long rows, int k) {
    if (k <= 0 || k % KGROUP != 0 || k > 65536) return -1;
#pragma omp parallel
    {
        uint16_t ybits[65536];
        float in[KGROUP], out[KGROUP];
#pragma omp for schedule(static)
        for (long r = 0; r < rows; ++r) {
            const uint16_t *row = x + r * (long)k;
            float absmax = 0.0f;
            for (int g = 0; g < k / KGROUP; ++g) {
                for (int i = 0; i < KGROUP; ++i) in[i] = bf16_to_f32(row[g * KGROUP + i]);
                ctu_oracle_rotate_group_b128(in, out);
                for (int i = 0; i < KGROUP; ++i) {
                    ybits[g * KGROUP + i] = ctu_oracle_f32_to_bf16(out[i]);
                    absmax = fmaxf(absmax, fabsf(out[i]));
                }
            }
            quantize_row_int8(ybits, k, absmax, codes + r * (long)k, scales + r, 0);
        }
    }
    return 0;
}


/* ---------------------------------------------------------------------------------
 * Per-group (128 along K) formats of the W4A8 / W4A4 linears.  The reference has no
 * kernel or checkpoint layout for them: its W4A4 path (dispatch.py:876-936) hands int4
 * activations to comfy-kitchen's int4_linear (source not available) with 64-column
 * weight groups, and its asymmetric W4A8 checkpoint format (asym_w4a8_int8,
 * AsymW4A8Int8Layout, fusions.py:14-16) is the grouped codebook.  The definitions below
 * are this build's, and the parity of these two formats is UNPINNED: they follow the bundled kernels' arithmetic where it
 * exists (rotation, int4 scale and code chain of convrot_quant.cu:475-500) and fix an
 * fp32 accumulation order over the 128-column groups for the rest.
 * --------------------------------------------------------------------------------- */
#define QGROUP 128

/* Rotate each row (256-column ConvRot groups), then quantize every 128-column group on
 * its own: scale = max(min(absmax, FLT_MAX) / 7, 1e-10) over the group's rotated fp32
 * values, codes = clamp(rint(bf16(y) * (1/scale)), -7, 7), even column in the low
 * nibble.  packed: rows x k/2; scales: rows x k/128. */
/* block = 256: the reference's rotation; block = 128: ctu_oracle_rotate_group_b128. */
static int convrot_quantize_int4_g128(const uint16_t *x, int8_t *packed, float *scales, long rows, int k, int block) {
    if (k <= 0 || k % KGROUP != 0 || k > 65536) return -1;
    const int groups = k / QGROUP;
#pragma omp parallel
    {
        uint16_t *ybits = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)k);
        float *yf = (float *)malloc(sizeof(float) * (size_t)k);
#pragma omp for schedule(static)
        for (long r = 0; r < rows; ++r) {
            if (block == 128) {
                float in[KGROUP], out[KGROUP];
                for (int g = 0; g < k / KGROUP; ++g) {
                    for (int i = 0; i < KGROUP; ++i) in[i] = bf16_to_f32(x[r * (long)k + g * KGROUP + i]);
                    ctu_oracle_rotate_group_b128(in, out);
                    for (int i = 0; i < KGROUP; ++i) {
                        ybits[g * KGROUP + i] = ctu_oracle_f32_to_bf16(out[i]);
                        yf[g * KGROUP + i] = out[i];
                    }
                }
            } else {
                (void)rotate_row(x + r * (long)k, k, 0, ybits, yf);
            }
            for (int g = 0; g < groups; ++g) {
                float absmax = 0.0f;
                for (int i = 0; i < QGROUP; ++i) absmax = fmaxf(absmax, fabsf(yf[g * QGROUP + i]));
                quantize_row_int4(ybits + g * QGROUP, QGROUP, absmax, packed + r * (long)(k / 2) + g * (QGROUP / 2),
                                  scales + r * (long)groups + g, 0);
            }
        }
        free(ybits);
        free(yf);
    }
    return 0;
}

int ctu_oracle_convrot_quantize_int4_g128(const uint16_t *x, int8_t *packed, float *scales, long rows, int k) {
    return convrot_quantize_int4_g128(x, packed, scales, rows, k, 256);
}

/* The same with the block-128 rotation (this build's definition, parity unpinned). */
int ctu_oracle_convrot_quantize_int4_g128_b128(const uint16_t *x, int8_t *packed, float *scales, long rows, int k) {
    return convrot_quantize_int4_g128(x, packed, scales, rows, k, 128);
}

/* Epilogue over per-group int32 partials acc[g][i][j] (groups x m x n), fp32 weight
 * scales w_scale_gn[g][j] (the fp16 checkpoint scales widened, group-major):
 *   mode 0 (W4A8, per-token activation scale a_scale[i]):
 *       t = 0; for g: t = fma(w_s[g][j], float(acc_g), t);   out = bf16(fma(t, a_s[i], bias[j]))
 *   mode 1 (W4A4, per-token-per-group activation scale a_scale[i][g]):
 *       t = 0; for g: t = fma(float(acc_g) * a_s[i][g], w_s[g][j], t);   out = bf16(t + bias[j])
 * A null bias adds +0.0. */
void ctu_oracle_grouped_epilogue(const int32_t *acc, int groups, const float *a_scale, const float *w_scale_gn,
                                 const float *bias, uint16_t *out, long m, long n, int mode) {
#pragma omp parallel for schedule(static)
    for (long i = 0; i < m; ++i) {
        for (long j = 0; j < n; ++j) {
            float t = 0.0f;
            for (int g = 0; g < groups; ++g) {
                const float v = (float)acc[((long)g * m + i) * n + j];
                const float s = w_scale_gn[(long)g * n + j];
                if (mode == 0) {
                    t = fmaf(s, v, t);
                } else {
                    const float u = v * a_scale[i * groups + g];
                    t = fmaf(u, s, t);
                }
            }
            const float b = bias ? bias[j] : 0.0f;
            const float v = mode == 0 ? fmaf(t, a_scale[i], b) : t + b;
            out[i * n + j] = ctu_oracle_f32_to_bf16(v);
        }
    }
}

/* ---------------------------------------------------------------------------------
 * Grouped-codebook W4A8 weight decode (kernel/csrc/turing/w4a8.cu:75-80, 903-976 and
 * the inline iterator :216-240): weight[n][c] = clamp(rint(codebook[code] * s), -127,
 * 127) with code the 4-bit value of column c (even column in the low nibble of the
 * packed byte), s the float8 e4m3fn group scale of group c / group_size in row n,
 * the product in fp32 and rint ties-to-even.  A NaN product decodes to 0 (the device
 * float-to-int conversion of NaN); +-inf saturates to +-127. */
static float e4m3fn_to_f32(uint8_t v) {
    const int sign = v >> 7;
    const int e = (v >> 3) & 0xF;
    const int m = v & 0x7;
    float mag;
    if (e == 0xF && m == 0x7) return u2f(0x7FC00000u);            /* NaN (no infinities) */
    if (e == 0) mag = ldexpf((float)m, -9);                          /* subnormal: m * 2^-9 */
    else mag = ldexpf(1.0f + (float)m / 8.0f, e - 7);
    return sign ? -mag : mag;
}

static int8_t decode_weight(float codebook_value, float scale) {
    const float value = codebook_value * scale;
    if (value != value) return 0;
    float q = nearbyintf(value);
    q = fminf(127.0f, fmaxf(-127.0f, q));
    return (int8_t)q;
}

void ctu_oracle_codebook_decode(const int8_t *packed, const uint8_t *group_scale, const float *codebook,
                                int8_t *out, long rows, int k, int group_size) {
    const int groups = k / group_size;
#pragma omp parallel for schedule(static)
    for (long r = 0; r < rows; ++r) {
        for (int c = 0; c < k; ++c) {
            const uint8_t byte = (uint8_t)packed[r * (k / 2) + c / 2];
            const int code = (c & 1) ? (byte >> 4) : (byte & 0xF);
            const float scale = e4m3fn_to_f32(group_scale[r * groups + c / group_size]);
            out[r * k + c] = decode_weight(codebook[code], scale);
        }
    }
}

/* Worker threads of every later OpenMP region of this library, whatever OMP_NUM_THREADS
 * the process started with (a launcher may pin it to 1 per rank). */
void ctu_oracle_set_threads(int threads) { omp_set_num_threads(threads > 0 ? threads : 1); }

int ctu_oracle_get_threads(void) { return omp_get_max_threads(); }

/* ---------------------------------------------------------------- norms */

/* Storage types of the norm ops: 0 = bf16, 1 = fp16, 2 = fp32. */
static inline float load_val(const void *p, long i, int dtype) {
    if (dtype == 0) return bf16_to_f32(((const uint16_t *)p)[i]);
    if (dtype == 1) {
        _Float16 h;
        memcpy(&h, (const uint16_t *)p + i, 2);
        return (float)h;
    }
    return ((const float *)p)[i];
}

/* from_float<T> of segmented_rms_adaln.cu:44-60: RNE to the storage type. */
static inline void store_val(void *p, long i, int dtype, float v) {
    if (dtype == 0) {
        ((uint16_t *)p)[i] = ctu_oracle_f32_to_bf16(v);
    } else if (dtype == 1) {
        const _Float16 h = (_Float16)v;
        memcpy((uint16_t *)p + i, &h, 2);
    } else {
        ((float *)p)[i] = v;
    }
}

static inline float round_to(float v, int dtype) {
    if (dtype == 0) return round_bf16(v);
    if (dtype == 1) return (float)(_Float16)v;
    return v;
}

static inline float host_rsqrt(float v) { return (float)(1.0 / sqrt((double)v)); }

/* segmented_rms_adaln.cu:114-131: first segment whose stop exceeds the row. */
static int find_modulation_row(const int32_t *segments, int count, long row) {
    int low = 0, high = count;
    while (low < high) {
        const int mid = low + (high - low) / 2;
        if (row < segments[mid * 3 + 1]) high = mid; else low = mid + 1;
    }
    if (low >= count || row < segments[low * 3]) return -1;
    return segments[low * 3 + 2];
}

/* warp_reduce_sum (segmented_rms_adaln.cu:75-81): shfl_down tree; a lane whose
 * source is past lane 31 reads its own value. */
static float warp_tree_sum(float *lane_val) {
    float next[32];
    for (int off = 16; off > 0; off >>= 1) {
        for (int l = 0; l < 32; ++l) next[l] = lane_val[l] + (l + off < 32 ? lane_val[l + off] : lane_val[l]);
        memcpy(lane_val, next, sizeof(next));
    }
    return lane_val[0];
}

/* segmented_rms_adaln.cu:133-232.  `vectorized` selects the reference's per-thread
 * element order (16-byte vectors t, t+256, ... or columns t, t+256, ...), which the
 * caller derives from the same alignment rule as the device launch (:308-313). */
void ctu_oracle_segmented_rms_adaln(const void *x, const void *weight, const void *scale, const void *shift,
                                    const int32_t *segments, void *out, long rows, int hidden, int param_rows,
                                    long scale_stride, long shift_stride, int segment_count, float epsilon,
                                    int dtype, int vectorized) {
    const int width = dtype == 2 ? 4 : 8;
#pragma omp parallel for schedule(static)
    for (long row = 0; row < rows; ++row) {
        const long base = row * (long)hidden;
        const int mapped = find_modulation_row(segments, segment_count, row);
        const int mod_row = mapped >= 0 && mapped < param_rows ? mapped : 0;
        float warp_sums[8];
        for (int w = 0; w < 8; ++w) {
            float lane_sum[32];
            for (int l = 0; l < 32; ++l) {
                const int t = w * 32 + l;
                float acc = 0.0f;
                if (vectorized) {
                    for (int j = t; j < hidden / width; j += 256)
                        for (int item = 0; item < width; ++item) {
                            const float v = load_val(x, base + (long)j * width + item, dtype);
                            acc = fmaf(v, v, acc);
                        }
                } else {
                    for (int c = t; c < hidden; c += 256) {
                        const float v = load_val(x, base + c, dtype);
                        acc = fmaf(v, v, acc);
                    }
                }
                lane_sum[l] = acc;
            }
            warp_sums[w] = warp_tree_sum(lane_sum);
        }
        float total = 0.0f;
        for (int w = 0; w < 8; ++w) total += warp_sums[w];
        const float inv = host_rsqrt(total / (float)hidden + epsilon);
        const long srow = (long)mod_row * scale_stride, hrow = (long)mod_row * shift_stride;
        for (int c = 0; c < hidden; ++c) {
            const float normalized = load_val(x, base + c, dtype) * inv;
            const float modulated = normalized * load_val(weight, c, dtype);
            const float result = fmaf(modulated, 1.0f + load_val(scale, srow + c, dtype), load_val(shift, hrow + c, dtype));
            store_val(out, base + c, dtype, result);
        }
    }
}

typedef struct { float mean, m2; int count; } welford_t;

/* welford_combine, segmented_rms_adaln.cu:89-105. */
static welford_t welford_combine(welford_t left, welford_t right) {
    if (right.count == 0) return left;
    if (left.count == 0) return right;
    const int count = left.count + right.count;
    const float delta = right.mean - left.mean;
    left.mean += delta * (float)right.count / (float)count;
    left.m2 += right.m2 + delta * delta * (float)left.count * (float)right.count / (float)count;
    left.count = count;
    return left;
}

/* segmented_rms_adaln.cu:234-297: Welford per thread over columns t, t+256, ...,
 * the shfl_down Welford tree, the in-order combine of 8 warps, then the
 * bf16/fp16-rounded normalised value times the rounded (1 + scale) plus shift. */
void ctu_oracle_layer_norm_adaln(const void *x, const void *scale, const void *shift, void *out, long batch,
                                 long sequence, int hidden, int modulation_steps, float epsilon, int dtype) {
    const long rows = batch * sequence;
#pragma omp parallel for schedule(static)
    for (long row = 0; row < rows; ++row) {
        const long b = row / sequence, token = row - b * sequence;
        long mtoken = 0;
        if (modulation_steps > 1) {
            const long repeats = sequence / modulation_steps;
            const long group = repeats * modulation_steps == sequence ? repeats : repeats + 1;
            mtoken = token / (group > 1 ? group : 1);
            if (mtoken > modulation_steps - 1) mtoken = modulation_steps - 1;
        }
        const long base = row * (long)hidden;
        const long mbase = (b * modulation_steps + mtoken) * (long)hidden;
        welford_t warps[8];
        for (int w = 0; w < 8; ++w) {
            welford_t lane[32];
            for (int l = 0; l < 32; ++l) {
                welford_t st = {0.0f, 0.0f, 0};
                for (int c = w * 32 + l; c < hidden; c += 256) {
                    const float v = load_val(x, base + c, dtype);
                    ++st.count;
                    const float delta = v - st.mean;
                    st.mean += delta / (float)st.count;
                    st.m2 = fmaf(delta, v - st.mean, st.m2);
                }
                lane[l] = st;
            }
            welford_t next[32];
            for (int off = 16; off > 0; off >>= 1) {
                for (int l = 0; l < 32; ++l) next[l] = welford_combine(lane[l], l + off < 32 ? lane[l + off] : lane[l]);
                memcpy(lane, next, sizeof(next));
            }
            warps[w] = lane[0];
        }
        welford_t st = {0.0f, 0.0f, 0};
        for (int w = 0; w < 8; ++w) st = welford_combine(st, warps[w]);
        const float mean = st.mean;
        const float variance = st.m2 / (float)st.count;
        const float inv = host_rsqrt(variance + epsilon);
        for (int c = 0; c < hidden; ++c) {
            const float normalized = round_to((load_val(x, base + c, dtype) - mean) * inv, dtype);
            const float multiplier = round_to(1.0f + load_val(scale, mbase + c, dtype), dtype);
            store_val(out, base + c, dtype, fmaf(normalized, multiplier, load_val(shift, mbase + c, dtype)));
        }
    }
}

/* ------------------------------------------------------------ fp16 staged rows */

/* The staged quantizers' fp16 instantiation (convrot_quant.cu:184-358 with
 * InputType = half): values convert exactly to fp32, GELU rounds to fp16, the
 * rotated values are stored as fp16, the scale clamps at 65504 and is formed with
 * the reciprocal constant, and the int8 chain rounds the scale and the quotient to
 * fp16 (convrot_quant.cu:66-73). */
static inline float f16_to_f32(uint16_t v) {
    _Float16 h;
    memcpy(&h, &v, 2);
    return (float)h;
}
static inline uint16_t f32_to_f16(float v) {
    const _Float16 h = (_Float16)v;
    uint16_t u;
    memcpy(&u, &h, 2);
    return u;
}
static inline float round_f16(float v) { return (float)(_Float16)v; }

static float rotate_row_f16(const uint16_t *row, int k, int mode, uint16_t *ybits) {
    float absmax = 0.0f;
    float in[KGROUP], out[KGROUP];
    for (int g = 0; g < k / KGROUP; ++g) {
        for (int i = 0; i < KGROUP; ++i) {
            const int col = g * KGROUP + i;
            in[i] = mode == 1 ? swiglu_value(f16_to_f32(row[col]), f16_to_f32(row[k + col]))
                              : round_f16(gelu_tanh_activated(f16_to_f32(row[col]), 1));
        }
        ctu_oracle_rotate_group(in, out);
        for (int i = 0; i < KGROUP; ++i) {
            ybits[g * KGROUP + i] = f32_to_f16(out[i]);
            absmax = fmaxf(absmax, fabsf(out[i]));
        }
    }
    return absmax;
}

static void quantize_row_int8_f16(const uint16_t *ybits, int k, float scale, int8_t *codes) {
    const float rounded_scale = round_f16(scale);
    for (int c = 0; c < k; ++c) {
        float q = nearbyintf(round_f16(f16_to_f32(ybits[c]) / rounded_scale));
        q = fminf(127.0f, fmaxf(-128.0f, q));
        codes[c] = (int8_t)q;
    }
}

/* mode 1 = SwiGLU ([rows, 2k] gate | up), 2 = tanh-GELU; fp16 bit patterns in x. */
int ctu_oracle_convrot_quantize_staged_f16(const uint16_t *x, int8_t *codes, float *scales, long rows, int k, int bits,
                                           int mode) {
    if (k <= 0 || k % KGROUP != 0 || k > 65536 || (mode != 1 && mode != 2)) return -1;
    const int width = mode == 1 ? 2 * k : k;
    const int out_width = bits == 4 ? k / 2 : k;
#pragma omp parallel
    {
        uint16_t ybits[65536];
#pragma omp for schedule(static)
        for (long r = 0; r < rows; ++r) {
            const float clamped = fminf(rotate_row_f16(x + r * width, k, mode, ybits), 65504.0f);
            if (bits == 4) {
                const float scale = fmaxf(clamped * (1.0f / 7.0f), 1.0e-10f);
                scales[r] = scale;
                const float inv_scale = 1.0f / scale;
                int8_t *packed = codes + r * out_width;
                for (int p = 0; p < k / 2; ++p) {
                    const float lo = fminf(7.0f, fmaxf(-7.0f, nearbyintf(f16_to_f32(ybits[2 * p]) * inv_scale)));
                    const float hi = fminf(7.0f, fmaxf(-7.0f, nearbyintf(f16_to_f32(ybits[2 * p + 1]) * inv_scale)));
                    packed[p] = (int8_t)(((uint8_t)(int8_t)lo & 0x0f) | (((uint8_t)(int8_t)hi & 0x0f) << 4));
                }
            } else {
                const float scale = fmaxf(clamped * (1.0f / 127.0f), 1.0e-30f);
                scales[r] = scale;
                quantize_row_int8_f16(ybits, k, scale, codes + r * out_width);
            }
        }
    }
    return 0;
}

/* turing_swiglu_int8_convrot_quantize_scaled on fp16 rows (convrot_quant.cu:239-278). */
int ctu_oracle_convrot_quantize_scaled_f16(const uint16_t *x, const float *scales, int8_t *codes, long rows, int k) {
    if (k <= 0 || k % KGROUP != 0 || k > 65536) return -1;
#pragma omp parallel
    {
        uint16_t ybits[65536];
#pragma omp for schedule(static)
        for (long r = 0; r < rows; ++r) {
            (void)rotate_row_f16(x + r * 2 * k, k, 1, ybits);
            quantize_row_int8_f16(ybits, k, scales[r], codes + r * k);
        }
    }
    return 0;
}

