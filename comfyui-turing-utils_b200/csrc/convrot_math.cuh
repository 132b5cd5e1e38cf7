// Arithmetic shared by the ConvRot quantizer kernels: the radix-4 butterfly, the fused
// input activations, the swizzled group loads and the per-8-value code conversions.
// Every function follows the reference's fp32 evaluation order
// (kernel/csrc/turing/convrot_quant.cu:104-182, 417-511).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "convrot_quant.cuh"
#include "ptx.cuh"

namespace ctu {
namespace rot {

constexpr float kBf16Max = 3.38953139e38f;  // largest finite bf16

// ---------------------------------------------------------------------------
// Radix-4 butterfly on two independent 4-tuples at once (packed f32x2), with the
// reference's association: y0 = ((x0+x1)+x2)-x3, y1 = ((x0+x1)-x2)+x3,
// y2 = ((x0-x1)+x2)+x3, y3 = ((-x0+x1)+x2)+x3, each times 0.5.
__device__ __forceinline__ void butterfly2(f32x2 &x0, f32x2 &x1, f32x2 &x2, f32x2 &x3, f32x2 half) {
    const f32x2 t = fadd2(x0, x1);
    const f32x2 b = fsub2(x0, x1);  // x0 - x1;  (-x0 + x1) == -(x0 - x1) exactly
    const f32x2 y0 = fmul2(half, fsub2(fadd2(t, x2), x3));
    const f32x2 y1 = fmul2(half, fadd2(fsub2(t, x2), x3));
    const f32x2 y2 = fmul2(half, fadd2(fadd2(b, x2), x3));
    const f32x2 y3 = fmul2(half, fadd2(fsub2(x2, b), x3));  // (-b) + x2 == x2 - b exactly
    x0 = y0;
    x1 = y1;
    x2 = y2;
    x3 = y3;
}

// Physical shared-memory byte offset of 16-byte chunk `c` of 128-byte slice `r`
// as written by a TMA load with CU_TENSOR_MAP_SWIZZLE_128B.
__device__ __forceinline__ uint32_t sw128(uint32_t r, uint32_t c) { return r * 128u + ((c ^ (r & 7u)) << 4); }

// The reference's input activations (convrot_quant.cu:163-182) evaluated on one bf16
// input given as fp32 bits: the SwiGLU gate factor gate / (1 + exp(-gate)) in fp32,
// and tanh-GELU rounded back to bf16.  Only act_lut_fill_kernel evaluates them.
__device__ __forceinline__ float silu_factor(float gate) { return gate / (1.0f + expf(-gate)); }

__device__ __forceinline__ float gelu_fp32(float x) {
    constexpr float kAlpha = 0.7978845608028654f;
    constexpr float kBeta = 0.044715f;
    return 0.5f * x * (1.0f + tanhf(kAlpha * (x + kBeta * x * x * x)));
}

__device__ __forceinline__ float gelu_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(gelu_fp32(x))); }

// Both activations take a bf16 input, so each is a function of 65536 bit patterns:
// act_lut_fill_kernel evaluates them once per device into these tables (the SwiGLU
// gate factor as fp32, GELU as bf16 bits), and the quantizers look the values up
// instead of evaluating expf / tanhf per element.  The tables hold exactly the values
// the expressions give, so the codes are unchanged.
struct ActLut {
    const float *silu;       // [65536] gate / (1 + expf(-gate)), indexed by the gate's bf16 bits
    const uint16_t *gelu;    // [65536] bf16 bits of tanh-GELU, indexed by the input's bf16 bits
    const float *silu16;     // the same two for fp16 inputs (the staged quantizers):
    const uint16_t *gelu16;  //   indexed by fp16 bits, GELU rounded to fp16
};

template <int Act>
__device__ __forceinline__ float activate(uint32_t gate_bits, uint32_t up_bits, const ActLut &lut);

template <>
__device__ __forceinline__ float activate<kActNone>(uint32_t x, uint32_t, const ActLut &) {
    return __uint_as_float(x);
}

// (gate / (1 + expf(-gate))) * up (convrot_quant.cu:163-169)
template <>
__device__ __forceinline__ float activate<kActSwiGLU>(uint32_t gate_bits, uint32_t up_bits, const ActLut &lut) {
    return __fmul_rn(__ldg(lut.silu + (gate_bits >> 16)), __uint_as_float(up_bits));
}

// bf16(tanh-GELU(x)) (convrot_quant.cu:171-182)
template <>
__device__ __forceinline__ float activate<kActGelu>(uint32_t x_bits, uint32_t, const ActLut &lut) {
    return __uint_as_float(static_cast<uint32_t>(__ldg(lut.gelu + (x_bits >> 16))) << 16);
}

// Load one lane's 128 inputs of a group: chunk0 = elements h*64+[0,64) (bit 7 = 0),
// chunk1 = 128+h*64+[0,64).  `row64` is the 128-byte slice index of chunk0 inside the
// batch buffer; chunk1 sits two slices later.  For SwiGLU the `up` half of the row
// starts `up_off` slices after the gate.  v[j] = (chunk0[j], chunk1[j]).
template <int Act>
__device__ __forceinline__ void load_group(const uint8_t *buf, uint32_t row64, uint32_t up_off, f32x2 (&v)[64],
                                           const ActLut &lut) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const uint4 a = *reinterpret_cast<const uint4 *>(buf + sw128(row64, c));
        const uint4 b = *reinterpret_cast<const uint4 *>(buf + sw128(row64 + 2, c));
        const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
        const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
        if constexpr (Act == kActSwiGLU) {
            const uint4 ua = *reinterpret_cast<const uint4 *>(buf + sw128(row64 + up_off, c));
            const uint4 ub = *reinterpret_cast<const uint4 *>(buf + sw128(row64 + up_off + 2, c));
            const uint32_t uaw[4] = {ua.x, ua.y, ua.z, ua.w};
            const uint32_t ubw[4] = {ub.x, ub.y, ub.z, ub.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                v[8 * c + 2 * q] = pk2(activate<Act>(aw[q] << 16, uaw[q] << 16, lut), activate<Act>(bw[q] << 16, ubw[q] << 16, lut));
                v[8 * c + 2 * q + 1] = pk2(activate<Act>(aw[q] & 0xFFFF0000u, uaw[q] & 0xFFFF0000u, lut),
                                           activate<Act>(bw[q] & 0xFFFF0000u, ubw[q] & 0xFFFF0000u, lut));
            }
        } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                v[8 * c + 2 * q] = pk2(activate<Act>(aw[q] << 16, 0, lut), activate<Act>(bw[q] << 16, 0, lut));
                v[8 * c + 2 * q + 1] = pk2(activate<Act>(aw[q] & 0xFFFF0000u, 0, lut), activate<Act>(bw[q] & 0xFFFF0000u, 0, lut));
            }
        }
    }
}

// ---------------------------------------------------------------------------
// fp16 inputs (the staged quantizers' other storage type, convrot_quant.cu:577-663):
// the values convert with __half2float and the rotated values round to fp16.
__device__ __forceinline__ float f16_to_f32(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16)));
}
__device__ __forceinline__ float f16lo(uint32_t w) { return f16_to_f32(w & 0xFFFFu); }
__device__ __forceinline__ float f16hi(uint32_t w) { return f16_to_f32(w >> 16); }

// Two fp32 -> packed fp16x2 (round to nearest even); `lo` lands in bits [0,16).
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

template <int Act>
__device__ __forceinline__ float activate_f16(uint32_t x16, uint32_t up16, const ActLut &lut) {
    if constexpr (Act == kActSwiGLU) {
        return __fmul_rn(__ldg(lut.silu16 + x16), f16_to_f32(up16));
    } else if constexpr (Act == kActGelu) {
        return f16_to_f32(__ldg(lut.gelu16 + x16));
    } else {
        return f16_to_f32(x16);
    }
}

// load_group for fp16 rows (same layout: v[j] = (chunk0[j], chunk1[j])).
template <int Act>
__device__ __forceinline__ void load_group_f16(const uint8_t *buf, uint32_t row64, uint32_t up_off,
                                               f32x2 (&v)[64], const ActLut &lut) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const uint4 a = *reinterpret_cast<const uint4 *>(buf + sw128(row64, c));
        const uint4 b = *reinterpret_cast<const uint4 *>(buf + sw128(row64 + 2, c));
        const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
        const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
        uint32_t uaw[4] = {0, 0, 0, 0}, ubw[4] = {0, 0, 0, 0};
        if constexpr (Act == kActSwiGLU) {
            const uint4 ua = *reinterpret_cast<const uint4 *>(buf + sw128(row64 + up_off, c));
            const uint4 ub = *reinterpret_cast<const uint4 *>(buf + sw128(row64 + up_off + 2, c));
            uaw[0] = ua.x, uaw[1] = ua.y, uaw[2] = ua.z, uaw[3] = ua.w;
            ubw[0] = ub.x, ubw[1] = ub.y, ubw[2] = ub.z, ubw[3] = ub.w;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            v[8 * c + 2 * q] = pk2(activate_f16<Act>(aw[q] & 0xFFFFu, uaw[q] & 0xFFFFu, lut),
                                   activate_f16<Act>(bw[q] & 0xFFFFu, ubw[q] & 0xFFFFu, lut));
            v[8 * c + 2 * q + 1] = pk2(activate_f16<Act>(aw[q] >> 16, uaw[q] >> 16, lut),
                                       activate_f16<Act>(bw[q] >> 16, ubw[q] >> 16, lut));
        }
    }
}

// int8 codes of 8 consecutive fp16(y) values, the staged chain for fp16
// (convrot_quant.cu:66-73,304-310): clamp(rint(fp16(y / fp16(scale))), -128, 127), with
// the IEEE quotient (NaN -> -128 as fminf/fmaxf give it).
__device__ __forceinline__ uint2 quant8_int8_f16(uint4 w, float rounded_scale) {
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    uint32_t out[2] = {0, 0};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float y = (i & 1) ? f16hi(ww[i >> 1]) : f16lo(ww[i >> 1]);
        const float divided = __half2float(__float2half_rn(__fdiv_rn(y, rounded_scale)));
        const float qf = fminf(127.0f, fmaxf(-128.0f, nearbyintf(divided)));
        out[i >> 2] |= (static_cast<uint32_t>(static_cast<int32_t>(qf)) & 0xFFu) << (8 * (i & 3));
    }
    return make_uint2(out[0], out[1]);
}

// Packed int4 codes of 8 consecutive fp16(y) values: clamp(rint(y * inv), -7, 7).
__device__ __forceinline__ uint32_t quant8_int4_f16(uint4 w, float inv) {
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    uint32_t out = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float lo = fminf(7.0f, fmaxf(-7.0f, nearbyintf(__fmul_rn(f16lo(ww[i]), inv))));
        const float hi = fminf(7.0f, fmaxf(-7.0f, nearbyintf(__fmul_rn(f16hi(ww[i]), inv))));
        const uint32_t lb = static_cast<uint32_t>(static_cast<int32_t>(lo)) & 0xFu;
        const uint32_t hb = static_cast<uint32_t>(static_cast<int32_t>(hi)) & 0xFu;
        out |= (lb | (hb << 4)) << (8 * i);
    }
    return out;
}

// Quantize 8 consecutive bf16(y) values of one row to int8 with the fast chain.
__device__ __forceinline__ uint2 quant8_int8_fast(uint4 w, f32x2 rcp2) {
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    int c[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float lo, hi;
        unpk2(fmul2(pk2(bf16lo(ww[i]), bf16hi(ww[i])), rcp2), lo, hi);
        const uint32_t qb = pack_bf16x2(lo, hi);
        c[2 * i] = __float2int_rn(bf16lo(qb));
        c[2 * i + 1] = __float2int_rn(bf16hi(qb));
    }
    // cvt.pack.sat.s8.s32.b32 d, a, b, c: d = {sat8(b), sat8(a), c[0:16)} from the low byte up.
    uint32_t t0, t1, lo, hi;
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(t0) : "r"(c[3]), "r"(c[2]), "r"(0u));
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(lo) : "r"(c[1]), "r"(c[0]), "r"(t0));
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(t1) : "r"(c[7]), "r"(c[6]), "r"(0u));
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(hi) : "r"(c[5]), "r"(c[4]), "r"(t1));
    return make_uint2(lo, hi);
}

// Per-row scale from the row's NaN-ignoring absmax.  The row-buffer kernels divide the
// clamped absmax by qmax (convrot_quant.cu:475-478); the staged kernels multiply it by
// the fp32 constant 1/qmax (convrot_quant.cu:300-303, 335-338), which rounds differently
// for some rows.
// The clamp is the input type's largest finite value (bf16, or 65504 for fp16 input).
// The row-buffer quotient clamped / qmax is formed by the correction step of Markstein's
// division with r = RN(1 / qmax): q0 = clamped * r, q = fma(fma(-q0, qmax, clamped), r, q0)
// equals the IEEE quotient for every dividend in [2^-96, FLT_MAX] and integer divisors up
// to 16384 (tests/native/division_check.c); a smaller dividend gives a quotient far below
// the floor on both paths, so the scale is the floor either way.
template <int Bits>
__device__ __forceinline__ float row_scale(float amax, bool staged, float finite_max = kBf16Max) {
    constexpr float qmax = Bits == 4 ? 7.0f : 127.0f;
    constexpr float rcp = 1.0f / qmax;
    constexpr float floor = Bits == 4 ? 1.0e-10f : 1.0e-30f;
    const float clamped = fminf(amax, finite_max);
    if (staged) return fmaxf(__fmul_rn(clamped, rcp), floor);
    const float q0 = __fmul_rn(clamped, rcp);
    return fmaxf(__fmaf_rn(__fmaf_rn(-q0, qmax, clamped), rcp, q0), floor);
}

// True when the reciprocal-quotient fast chain reproduces bf16(y / rounded_scale) for
// every finite y: the rounded scale is a normal, finite bf16 value.
__device__ __forceinline__ bool fast_chain_scale_ok(float rounded_scale) {
    const float a = fabsf(rounded_scale);
    return a >= 1.17549435e-38f && a <= kBf16Max;
}

// Exact reference chain including NaN (fmaxf(-128, NaN) == -128) for rows that
// contain NaN or infinities.
static __device__ __noinline__ uint2 quant8_int8_exact(uint4 w, float rounded_scale) {
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    uint32_t out[2] = {0, 0};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float y = (i & 1) ? bf16hi(ww[i >> 1]) : bf16lo(ww[i >> 1]);
        const float divided = __bfloat162float(__float2bfloat16_rn(__fdiv_rn(y, rounded_scale)));
        float qf = nearbyintf(divided);
        qf = fminf(127.0f, fmaxf(-128.0f, qf));
        const uint32_t byte = static_cast<uint32_t>(static_cast<int32_t>(qf)) & 0xFFu;
        out[i >> 2] |= byte << (8 * (i & 3));
    }
    return make_uint2(out[0], out[1]);
}

// Quantize 8 consecutive bf16(y) values to packed int4 (exact for every input).
__device__ __forceinline__ uint32_t quant8_int4(uint4 w, f32x2 inv2) {
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    uint32_t out = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float plo, phi;
        unpk2(fmul2(pk2(bf16lo(ww[i]), bf16hi(ww[i])), inv2), plo, phi);
        const float lo = fminf(7.0f, fmaxf(-7.0f, plo));
        const float hi = fminf(7.0f, fmaxf(-7.0f, phi));
        const uint32_t lb = static_cast<uint32_t>(__float2int_rn(lo)) & 0xFu;
        const uint32_t hb = static_cast<uint32_t>(__float2int_rn(hi)) & 0xFu;
        out |= (lb | (hb << 4)) << (8 * i);
    }
    return out;
}

}  // namespace rot
}  // namespace ctu
