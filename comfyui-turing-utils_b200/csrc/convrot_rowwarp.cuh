// Warp-level building blocks of the eight-lane ConvRot quantizers, shared by the
// stand-alone quantizer kernels (convrot_quant_k8.cu) and the fused ConvRot linear
// (gemm_pair.cu): the group rotation with its shared-memory transpose, the fast int8
// code chain, and the warp-row pipeline in which one warp owns a whole token row.
//
// Group layout (eight lanes, "team", per 256-column group; element e has index bits
// 0-7 and radix-4 stage s combines the four elements that differ in bits 2s-2, 2s-1):
// lane q holds elements 16q + j + 128h (j < 16, h < 2) as 16 packed pairs for stages
// 1-2, writes them to a 1 KB transpose area, and reads back the pairs of consecutive
// columns (2q + 16u, 2q + 16u + 1), u < 16, for stages 3-4.  The transpose area of
// team g of a warp is `garea`; `wbase` / `rbase` are the lane's write / read bases:
//   wbase = garea + 16 (4q ^ q / 2 ^ 4 (g % 2)),  rbase = garea + 8 (q % 2) + 16 (q / 2 ^ 4 (g % 2)),
// with garea 1024-byte aligned (the placement is conflict-free for the 16-byte writes of
// each quarter-warp and the 8-byte reads of each half-warp).
//
// Folded halvings.  For bf16-valued inputs (plain rows, tanh-GELU table values) the
// rotation without the four per-stage halvings gives z = 16 y exactly unless z
// overflows (every intermediate is a multiple of 2^-137, so no halving rounds and
// rounding commutes with the power-of-two scaling); a group whose folded outputs are not
// all finite is recomputed in the reference's order.  The int8 codes take the factor
// 1/16 in the reciprocal.  The full argument is written out beside the multi-group
// kernel in convrot_quant_k8.cu.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "convrot_math.cuh"
#include "ptx.cuh"

namespace ctu {
namespace rot {

__device__ __forceinline__ void st_shared_v4(uint32_t addr, float a, float b, float c, float d) {
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

__device__ __forceinline__ float2 ld_shared_v2(uint32_t addr) {
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr) : "memory");
    return v;
}

// Radix-4 butterfly without the halving (the reference's association otherwise).
__device__ __forceinline__ void butterfly2_unscaled(f32x2 &x0, f32x2 &x1, f32x2 &x2, f32x2 &x3) {
    const f32x2 t = fadd2(x0, x1);
    const f32x2 b = fsub2(x0, x1);
    const f32x2 y0 = fsub2(fadd2(t, x2), x3);
    const f32x2 y1 = fadd2(fsub2(t, x2), x3);
    const f32x2 y2 = fadd2(fadd2(b, x2), x3);
    const f32x2 y3 = fadd2(fsub2(x2, b), x3);
    x0 = y0;
    x1 = y1;
    x2 = y2;
    x3 = y3;
}

// max(a, |b|, |c|) propagating NaN (any NaN operand gives NaN).
__device__ __forceinline__ float max_abs3_nan(float a, float b, float c) {
    float r;
    asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(fabsf(b)), "f"(fabsf(c)));
    return r;
}

__device__ __forceinline__ float max_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

__device__ __forceinline__ uint4 ld_shared_v4u(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
                 : "memory");
    return v;
}

// Rotation of the team's group.  kHalve: the reference's order with the per-stage
// halvings (W = bf16(y), NaN-ignoring absmax, NaN probe); otherwise unscaled (W = bf16(z),
// z = 16 y, NaN-propagating absmax of z).  Word W[u] of lane q holds columns 16u + 2q and
// 16u + 2q + 1 of the group.  kHalves: `absmax` covers columns 0..127 (u < 8) and
// `absmax_hi` columns 128..255; otherwise `absmax` covers the whole group.  kTeamReduce:
// the statistics are reduced over the team's 8 lanes; otherwise each lane returns its own
// (the warp-row pipeline reduces once per row).  kBlock128 (with kHalve): rotation
// block 128 -- the last stage is radix-2 at stride 64 scaled by RN(1/sqrt 2), each
// 128-column half of the group on its own (this build's definition; see
// convrot_oracle.c).  All 32 lanes of the warp take part.
template <bool kHalve, bool kHalves = false, bool kTeamReduce = true, bool kBlock128 = false>
__device__ __forceinline__ void g8_rotate(f32x2 (&P)[16], uint32_t wbase, uint32_t rbase, uint32_t (&W)[16],
                                          float &absmax, float &nan_probe, float &absmax_hi) {
    const f32x2 half = pk2(0.5f, 0.5f);
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        if constexpr (kHalve) butterfly2(P[4 * a], P[4 * a + 1], P[4 * a + 2], P[4 * a + 3], half);
        else butterfly2_unscaled(P[4 * a], P[4 * a + 1], P[4 * a + 2], P[4 * a + 3]);
    }
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        if constexpr (kHalve) butterfly2(P[p], P[p + 4], P[p + 8], P[p + 12], half);
        else butterfly2_unscaled(P[p], P[p + 4], P[p + 8], P[p + 12]);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            float v[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float lo, hi;
                unpk2(P[4 * c + i], lo, hi);
                v[i] = h ? hi : lo;
            }
            const uint32_t addr = h ? ((wbase ^ (16u * c) ^ 64u) + 512u) : (wbase ^ (16u * c));
            st_shared_v4(addr, v[0], v[1], v[2], v[3]);
        }
    }
    __syncwarp();
    f32x2 R[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) {
        const float2 v = ld_shared_v2(rbase ^ (16u * ((4u * u) ^ (u >> 1))));
        R[u] = pk2(v.x, v.y);
    }
    __syncwarp();  // the area is rewritten by the next group only after these reads
#pragma unroll
    for (int v = 0; v < 4; ++v) {
        if constexpr (kHalve) butterfly2(R[4 * v], R[4 * v + 1], R[4 * v + 2], R[4 * v + 3], half);
        else butterfly2_unscaled(R[4 * v], R[4 * v + 1], R[4 * v + 2], R[4 * v + 3]);
    }
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        if constexpr (kBlock128) {
            static_assert(kHalve, "the block-128 rotation keeps the halvings");
            // u bit 2 is column bit 6; u bit 3 (column bit 7) selects the 128-block.
            const f32x2 c2 = pk2(0x1.6a09e6p-1f, 0x1.6a09e6p-1f);
#pragma unroll
            for (int blk = 0; blk < 16; blk += 8) {
                const f32x2 t = fadd2(R[w + blk], R[w + blk + 4]);
                const f32x2 d = fsub2(R[w + blk], R[w + blk + 4]);
                R[w + blk] = fmul2(t, c2);
                R[w + blk + 4] = fmul2(d, c2);
            }
        } else if constexpr (kHalve) {
            butterfly2(R[w], R[w + 4], R[w + 8], R[w + 12], half);
        } else {
            butterfly2_unscaled(R[w], R[w + 4], R[w + 8], R[w + 12]);
        }
    }
    float m = 0.0f, mh = 0.0f;
    f32x2 probe = pk2(0.0f, 0.0f);
#pragma unroll
    for (int u = 0; u < 16; ++u) {
        float lo, hi;
        unpk2(R[u], lo, hi);
        float &acc = kHalves && u >= 8 ? mh : m;
        if constexpr (kHalve) {
            probe = fadd2(probe, R[u]);
            acc = max_abs3(acc, lo, hi);
        } else {
            acc = max_abs3_nan(acc, lo, hi);
        }
        W[u] = pack_bf16x2(lo, hi);
    }
    float pr = 0.0f;
    if constexpr (kHalve) {
        float p0, p1;
        unpk2(probe, p0, p1);
        pr = __fadd_rn(p0, p1);
    }
#pragma unroll
    for (int d = 1; d < (kTeamReduce ? 8 : 1); d <<= 1) {
        if constexpr (kHalve) {
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, d));  // NaN-ignoring, as the reference's fmaxf
            if constexpr (kHalves) mh = fmaxf(mh, __shfl_xor_sync(0xffffffffu, mh, d));
            pr = __fadd_rn(pr, __shfl_xor_sync(0xffffffffu, pr, d));
        } else {
            m = max_nan(m, __shfl_xor_sync(0xffffffffu, m, d));
            if constexpr (kHalves) mh = max_nan(mh, __shfl_xor_sync(0xffffffffu, mh, d));
        }
    }
    absmax = m;
    absmax_hi = mh;
    nan_probe = pr;
}

// Two int8 codes of one bf16 word (columns c, c + 1) with the reciprocal chain, in the
// low 16 bits (byte 0 = column c).
__device__ __forceinline__ uint32_t quant2_int8_fast(uint32_t w, f32x2 rcp2) {
    float lo, hi;
    unpk2(fmul2(pk2(bf16lo(w), bf16hi(w)), rcp2), lo, hi);
    const uint32_t qb = pack_bf16x2(lo, hi);
    const int c0 = __float2int_rn(bf16lo(qb));
    const int c1 = __float2int_rn(bf16hi(qb));
    uint32_t d;
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(c1), "r"(c0), "r"(0u));
    return d;
}

// Packed int4 codes of 8 values whose folded words must first be scaled by 1/16 (rows
// whose reciprocal is too small to take the factor without leaving the normal range).
static __device__ __noinline__ uint32_t quant8_int4_prescaled(uint4 w, float inv) {
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    const f32x2 pre = pk2(0.0625f, 0.0625f);
    const f32x2 inv2 = pk2(inv, inv);
    uint32_t out = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float plo, phi;
        unpk2(fmul2(fmul2(pk2(bf16lo(ww[i]), bf16hi(ww[i])), pre), inv2), plo, phi);
        const uint32_t lb = static_cast<uint32_t>(__float2int_rn(fminf(7.0f, fmaxf(-7.0f, plo)))) & 0xFu;
        const uint32_t hb = static_cast<uint32_t>(__float2int_rn(fminf(7.0f, fmaxf(-7.0f, phi)))) & 0xFu;
        out |= (lb | (hb << 4)) << (8 * i);
    }
    return out;
}

// Phase A load of one group from a plain row-major bf16 row in shared memory: lane q
// reads elements 16q .. 16q + 15 and 128 + 16q .. 128 + 16q + 15 of the group at `gaddr`.
template <int Act>
__device__ __forceinline__ void w8_load(uint32_t gaddr, uint32_t q, f32x2 (&P)[16], const ActLut &lut) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        const uint4 a = ld_shared_v4u(gaddr + 32u * q + 16u * c);
        const uint4 b = ld_shared_v4u(gaddr + 256u + 32u * q + 16u * c);
        const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
        const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            P[8 * c + 2 * i] = pk2(activate<Act>(aw[i] << 16, 0, lut), activate<Act>(bw[i] << 16, 0, lut));
            P[8 * c + 2 * i + 1] = pk2(activate<Act>(aw[i] & 0xFFFF0000u, 0, lut),
                                       activate<Act>(bw[i] & 0xFFFF0000u, 0, lut));
        }
    }
}


// ---------------------------------------------------------------------------
// Warp-row pipeline.  The warp's row buffer `buf` holds one whole bf16 row (plain
// row-major, K = 256 * groups columns, 512 bytes per group).  Team g (lanes 8g .. 8g + 7)
// rotates groups g, g + 4, ..., g + 4 (kGt - 1) (slots past the last group rotate the
// last group again and are ignored) and keeps their bf16 words in registers.

// Rotates the row: W[i] / folded[i] for slot i, this lane's absmax over its values of
// the row (of the halved rotation: folded slots are rescaled by 1/16) and whether one of
// its values of a non-folded group is NaN.  The statistics stay per lane -- max and "any"
// do not depend on the order of reduction, and the fold test is a warp-wide vote -- so
// the warp reduces them once per row instead of once per group.  (A row with +inf and
// -inf but no NaN, which a summed probe would flag, has an infinite absmax and takes the
// same exact chain.)  All 32 lanes take part; the buffer is no longer read when this
// returns and every lane has passed a __syncwarp.
// kBlock128: the block-128 rotation, always in the halved order (no fold).
template <int Act, int kGt, bool kBlock128 = false>
__device__ __forceinline__ void w8_rotate_row(uint32_t buf, int groups, uint32_t g, uint32_t q, uint32_t wbase,
                                              uint32_t rbase, const ActLut &lut, uint32_t (&W)[kGt][16],
                                              bool (&folded)[kGt], float &lane_amax, bool &any_nan) {
    float amax = 0.0f;  // non-negative, never NaN
    bool nan_seen = false;
#pragma unroll
    for (int i = 0; i < kGt; ++i) {
        const int grp = static_cast<int>(g) + 4 * i;
        const bool active = grp < groups;
        const uint32_t gaddr = buf + 512u * static_cast<uint32_t>(active ? grp : groups - 1);
        float ga = 0.0f, probe = 0.0f, unused = 0.0f;
        f32x2 P[16];
        if constexpr (kBlock128) {
            w8_load<Act>(gaddr, q, P, lut);
            g8_rotate<true, false, false, true>(P, wbase, rbase, W[i], ga, probe, unused);
            folded[i] = false;
            nan_seen |= active && isnan(probe);
            if (active) amax = fmaxf(amax, ga);
            continue;
        }
        w8_load<Act>(gaddr, q, P, lut);
        g8_rotate<false, false, false>(P, wbase, rbase, W[i], ga, probe, unused);
        folded[i] = !__any_sync(0xffffffffu, active && !(ga <= 3.40282347e38f));
        if (folded[i]) {
            ga *= 0.0625f;
        } else {  // warp-uniform: the reference's order, halvings included
            w8_load<Act>(gaddr, q, P, lut);
            g8_rotate<true, false, false>(P, wbase, rbase, W[i], ga, probe, unused);
            nan_seen |= active && isnan(probe);
        }
        if (active) amax = fmaxf(amax, ga);
    }
    __syncwarp();  // every lane's reads of the buffer are done
    lane_amax = amax;
    any_nan = nan_seen;
}

// Row absmax from the lanes' maxima (every lane receives it).
__device__ __forceinline__ float w8_row_absmax(float lane_amax) {
    float m = lane_amax;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, d));
    return m;
}

// Codes of the row (int8: [K] bytes; int4: [K / 2] packed) from the rotated words,
// given the row's scale and statistics; the reference's int8 chain (exact when the row
// had a NaN or an infinite absmax, otherwise the reciprocal form) or its int4 chain.
template <int Bits, int kGt>
__device__ __forceinline__ void w8_store_codes(const uint32_t (&W)[kGt][16], const bool (&folded)[kGt], float amax,
                                               float scale, bool row_nan, int groups, uint32_t g, uint32_t q,
                                               int8_t *out_row) {
    if constexpr (Bits == 4) {
        const float inv = __fdiv_rn(1.0f, scale);
#pragma unroll
        for (int i = 0; i < kGt; ++i) {
            const int grp = static_cast<int>(g) + 4 * i;
            if (grp >= groups) continue;
            int8_t *out = out_row + grp * 128 + q;
            if (folded[i] && !(inv >= 0x1p-100f)) {
#pragma unroll
                for (int u = 0; u < 16; u += 4) {
                    const uint32_t c =
                        quant8_int4_prescaled(make_uint4(W[i][u], W[i][u + 1], W[i][u + 2], W[i][u + 3]), inv);
#pragma unroll
                    for (int b = 0; b < 4; ++b) out[8 * (u + b)] = static_cast<int8_t>((c >> (8 * b)) & 0xFFu);
                }
            } else {
                const float iv = folded[i] ? inv * 0.0625f : inv;
                const f32x2 i2 = pk2(iv, iv);
#pragma unroll
                for (int u = 0; u < 16; u += 4) {
                    const uint32_t c = quant8_int4(make_uint4(W[i][u], W[i][u + 1], W[i][u + 2], W[i][u + 3]), i2);
#pragma unroll
                    for (int b = 0; b < 4; ++b) out[8 * (u + b)] = static_cast<int8_t>((c >> (8 * b)) & 0xFFu);
                }
            }
        }
    } else {
        const float rs = __bfloat162float(__float2bfloat16_rn(scale));
        const bool exact_chain = row_nan || isinf(amax);
        const float rcp = __frcp_rn(rs);
#pragma unroll
        for (int i = 0; i < kGt; ++i) {
            const int grp = static_cast<int>(g) + 4 * i;
            if (grp >= groups) continue;
            uint16_t *o16 = reinterpret_cast<uint16_t *>(out_row + grp * 256 + 2 * q);
            if (exact_chain) {
                const float divisor = folded[i] ? rs * 16.0f : rs;
#pragma unroll
                for (int u = 0; u < 16; u += 4) {
                    const uint2 c =
                        quant8_int8_exact(make_uint4(W[i][u], W[i][u + 1], W[i][u + 2], W[i][u + 3]), divisor);
                    o16[8 * u] = static_cast<uint16_t>(c.x & 0xFFFFu);
                    o16[8 * u + 8] = static_cast<uint16_t>(c.x >> 16);
                    o16[8 * u + 16] = static_cast<uint16_t>(c.y & 0xFFFFu);
                    o16[8 * u + 24] = static_cast<uint16_t>(c.y >> 16);
                }
            } else {
                const float rc = rcp * (folded[i] ? 0.0625f : 1.0f);
                const f32x2 r2 = pk2(rc, rc);
#pragma unroll
                for (int u = 0; u < 16; ++u) o16[8 * u] = static_cast<uint16_t>(quant2_int8_fast(W[i][u], r2));
            }
        }
    }
}

}  // namespace rot
}  // namespace ctu
