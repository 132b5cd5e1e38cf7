// ConvRot rotate + per-token quantize with eight lanes per 256-column group: the same
// arithmetic as the register-resident and four-lane kernels (convrot_quant_reg.cu,
// convrot_quant_t4.cu; reference kernel/csrc/turing/convrot_quant.cu:417-511) with 32
// values per lane, so a thread needs a quarter of the two-lane kernel's registers and
// several times as many warps share an SM to hide the rotation's dependency chains.
//
// Element e of a group has index bits 0-7; radix-4 stage s combines the four elements
// that differ in bits (2s-2, 2s-1).
//   * Phase A: lane q (0..7) of the group holds elements 16q + j + 128h, j < 16,
//     h < 2, as 16 packed pairs P[j] = (h = 0, h = 1).  Stages 1 and 2 (bits 0-3 = j)
//     run in registers; bit 7 pairs the packed halves, which neither stage touches.
//   * Transpose: each lane writes its 32 values to the warp's shared-memory area as
//     16-byte chunks of 4 consecutive elements; after __syncwarp, lane q' reads the
//     8-byte pairs (2q' + 16u, 2q' + 16u + 1), u < 16.
//   * Phase B: stages 3 and 4 (bits 4-7 = u) run in registers on those pairs; the
//     outputs are bf16 pairs of consecutive columns, whose codes go out as 2-byte
//     (int8) or 1-byte (int4) stores that the group's 8 lanes fill contiguously.
// Shared-memory placement of a group (1 KB, 64 chunks of 16 bytes): chunk t = e / 4 sits
// at slot t ^ ((t / 8) % 8) ^ 4 (g % 2) for the warp-local group index g.  The 16-byte
// writes of each quarter-warp (one group's 8 lanes) and the 8-byte reads of each
// half-warp (two groups) then touch distinct banks.
//
// Batches, row statistics and the quantization chains are those of the other whole-row
// kernels: whole rows per CTA batch streamed in by TMA, per-row absmax in shared memory,
// a NaN probe that selects the exact reference chain, caller-supplied scales for the
// SwiGLU shard op.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "convrot_math.cuh"
#include "convrot_quant.cuh"
#include "convrot_rowwarp.cuh"
#include "ptx.cuh"

namespace ctu {
namespace rot {

namespace {

__device__ __forceinline__ uint32_t k8_slot(uint32_t g, uint32_t t) { return t ^ ((t >> 3) & 7u) ^ (4u * (g & 1u)); }

// Phase A load: lane q's 32 inputs of the group whose first 128-byte slice in the batch
// buffer is `slice0`: P[j] = (element 16q + j, element 16q + j + 128).
template <int Act>
__device__ __forceinline__ void k8_load(const uint8_t *buf, uint32_t slice0, uint32_t q, uint32_t up_off,
                                        f32x2 (&P)[16], const ActLut &lut) {
    const uint32_t s = slice0 + (q >> 2);  // elements 16q.. lie in slice q / 4, chunks 2 (q % 4) and 2 (q % 4) + 1
    const uint32_t c0 = 2u * (q & 3u);
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        const uint4 a = *reinterpret_cast<const uint4 *>(buf + sw128(s, c0 + c));
        const uint4 b = *reinterpret_cast<const uint4 *>(buf + sw128(s + 2, c0 + c));
        const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
        const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
        if constexpr (Act == kActSwiGLU) {
            const uint4 ua = *reinterpret_cast<const uint4 *>(buf + sw128(s + up_off, c0 + c));
            const uint4 ub = *reinterpret_cast<const uint4 *>(buf + sw128(s + up_off + 2, c0 + c));
            const uint32_t uaw[4] = {ua.x, ua.y, ua.z, ua.w};
            const uint32_t ubw[4] = {ub.x, ub.y, ub.z, ub.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                P[8 * c + 2 * i] = pk2(activate<Act>(aw[i] << 16, uaw[i] << 16, lut), activate<Act>(bw[i] << 16, ubw[i] << 16, lut));
                P[8 * c + 2 * i + 1] = pk2(activate<Act>(aw[i] & 0xFFFF0000u, uaw[i] & 0xFFFF0000u, lut),
                                           activate<Act>(bw[i] & 0xFFFF0000u, ubw[i] & 0xFFFF0000u, lut));
            }
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                P[8 * c + 2 * i] = pk2(activate<Act>(aw[i] << 16, 0, lut), activate<Act>(bw[i] << 16, 0, lut));
                P[8 * c + 2 * i + 1] = pk2(activate<Act>(aw[i] & 0xFFFF0000u, 0, lut), activate<Act>(bw[i] & 0xFFFF0000u, 0, lut));
            }
        }
    }
}

// Rotation of the group held by the warp's 8-lane team (all 32 lanes call it together:
// __syncwarp and the team reductions).  Returns the lane's bf16 words
// W[u] = (y[2q + 16u], y[2q + 16u + 1]) and the team's absmax / NaN probe.
__device__ __forceinline__ void k8_rotate(f32x2 (&P)[16], uint32_t garea, uint32_t g, uint32_t q,
                                          uint32_t (&W)[16], float &absmax, float &nan_probe) {
    const f32x2 half = pk2(0.5f, 0.5f);
    // Stage 1 (bits 0-1 of j) and stage 2 (bits 2-3 of j).
#pragma unroll
    for (int a = 0; a < 4; ++a) butterfly2(P[4 * a], P[4 * a + 1], P[4 * a + 2], P[4 * a + 3], half);
#pragma unroll
    for (int p = 0; p < 4; ++p) butterfly2(P[p], P[p + 4], P[p + 8], P[p + 12], half);
    // Transpose: chunk t = 4q + c + 32h holds elements 16q + 4c + 128h + (0..3).
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
            const uint32_t t = 4u * q + static_cast<uint32_t>(c) + 32u * static_cast<uint32_t>(h);
            st_shared_v4(garea + 16u * k8_slot(g, t), v[0], v[1], v[2], v[3]);
        }
    }
    __syncwarp();
    f32x2 R[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) {
        const uint32_t t = 4u * static_cast<uint32_t>(u) + (q >> 1);
        const float2 v = ld_shared_v2(garea + 16u * k8_slot(g, t) + 8u * (q & 1u));
        R[u] = pk2(v.x, v.y);
    }
    __syncwarp();  // the area is rewritten by the next batch only after these reads
    // Stage 3 (bits 4-5 = bits 0-1 of u) and stage 4 (bits 6-7 = bits 2-3 of u).
#pragma unroll
    for (int v = 0; v < 4; ++v) butterfly2(R[4 * v], R[4 * v + 1], R[4 * v + 2], R[4 * v + 3], half);
#pragma unroll
    for (int w = 0; w < 4; ++w) butterfly2(R[w], R[w + 4], R[w + 8], R[w + 12], half);
    float m = 0.0f;
    f32x2 probe = pk2(0.0f, 0.0f);
#pragma unroll
    for (int u = 0; u < 16; ++u) {
        float lo, hi;
        unpk2(R[u], lo, hi);
        probe = fadd2(probe, R[u]);
        m = max_abs3(m, lo, hi);
        W[u] = pack_bf16x2(lo, hi);
    }
    float p0, p1;
    unpk2(probe, p0, p1);
    float pr = __fadd_rn(p0, p1);
    // Team (8 lanes) reductions; NaN-ignoring max as the reference's fmaxf.
#pragma unroll
    for (int d = 1; d < 8; d <<= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, d));
        pr = __fadd_rn(pr, __shfl_xor_sync(0xffffffffu, pr, d));
    }
    absmax = m;
    nan_probe = pr;
}

}  // namespace

// 96 registers a thread (no spills; 21 warps per SM): the budget is set directly, as no
// launch bound expresses it for CTAs of up to kK8MaxThreads threads.
template <int Act, int Bits>
__global__ void __maxnreg__(kK8Registers)
    convrot_quant_k8_kernel(const __grid_constant__ CUtensorMap tmap_x, const QuantArgs args) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int K = args.k;
    const int B = args.rows_per_batch;
    const int Kin = Act == kActSwiGLU ? 2 * K : K;
    const int Kout = Bits == 4 ? K / 2 : K;
    const int groups = K / 256;
    const int nwarps = blockDim.x >> 5;
    const uint32_t in_bytes = static_cast<uint32_t>(args.box_rows) * args.copies * 128u;  // multiple of 1024
    const uint32_t slices_per_row = Kin / 64;
    uint8_t *inbuf = smem;
    uint8_t *xbase = smem + in_bytes;                                                     // nwarps x 4 KB
    uint32_t *row_absmax = reinterpret_cast<uint32_t *>(xbase + nwarps * kK8WarpBytes);  // [2][B]
    uint32_t *row_nan = row_absmax + 2 * B;                                               // [2][B]
    uint64_t *full = reinterpret_cast<uint64_t *>(row_nan + 2 * B);                      // 8-byte aligned

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const uint32_t g = static_cast<uint32_t>(lane >> 3);  // group slot in the warp
    const uint32_t q = static_cast<uint32_t>(lane & 7);   // lane in the group's team
    const uint32_t garea = smem_u32(xbase + warp * kK8WarpBytes) + g * kK8GroupBytes;
    const int num_batches = (args.m + B - 1) / B;
    const uint32_t slices_per_batch = static_cast<uint32_t>(B) * slices_per_row;
    const bool given = args.given_scales != nullptr;  // uniform: a kernel argument
    const ActLut lut{args.silu_lut, args.gelu_lut};

    auto issue_load = [&](int batch) {
        mbar_arrive_expect_tx(full, in_bytes);
        for (int c = 0; c < args.copies; ++c) {
            const uint32_t s0 = static_cast<uint32_t>(c * args.box_rows);
            tma_load_2d(inbuf + s0 * 128u, &tmap_x, 0, static_cast<int>(batch * slices_per_batch + s0), full);
        }
    };

    if (tid == 0) {
        mbar_init(full, 1);
        fence_mbar_init();
    }
    for (int i = tid; i < 4 * B; i += blockDim.x) row_absmax[i] = 0u;  // also clears row_nan
    __syncthreads();
    uint32_t issued = 0;
    if (tid == 0) {
        prefetch_tmap(&tmap_x);
        if (blockIdx.x < num_batches) {
            issue_load(blockIdx.x);
            issued = 1;
        }
    }

    const int team = warp * 4 + static_cast<int>(g);  // group task of this lane's team
    // Every batch holds B whole rows, so a team's row and group within the batch are fixed.
    const int team_r = team / groups;
    const int team_grp = team - team_r * groups;
    bool alive = true;

    for (int it = 0;; ++it) {
        const int batch = blockIdx.x + it * gridDim.x;
        if (batch >= num_batches) break;
        const int par = it & 1;
        const int row0 = batch * B;
        const int rows = min(B, args.m - row0);
        const int tasks = rows * groups;
        const bool warp_busy = warp * 4 < tasks;  // warp-uniform
        const bool active = team < tasks;
        const int r = active ? team_r : 0;
        const int grp = active ? team_grp : 0;

        if (alive) alive = mbar_wait(full, static_cast<uint32_t>(it & 1), nullptr, args.err, kErrTimeoutFull);
        f32x2 P[16];
        if (warp_busy && alive)
            k8_load<Act>(inbuf, r * slices_per_row + grp * 4, q, static_cast<uint32_t>(K / 64), P, lut);
        __syncthreads();  // the batch is in registers: the buffer may be refilled
        if (tid == 0 && alive) {
            const int next = batch + gridDim.x;
            if (next < num_batches) {
                issue_load(next);
                ++issued;
            }
        }
        for (int i = tid; i < B; i += blockDim.x) {
            row_absmax[(par ^ 1) * B + i] = 0u;
            row_nan[(par ^ 1) * B + i] = 0u;
        }

        uint32_t W[16];
        bool group_nan = false;
        if (warp_busy && alive) {
            float amax, probe;
            k8_rotate(P, garea, g, q, W, amax, probe);
            if (active && q == 0 && !given) {
                atomicMax(&row_absmax[par * B + r], __float_as_uint(amax));
                if (isnan(probe)) atomicOr(&row_nan[par * B + r], 1u);
            }
            group_nan = isnan(probe);
        }
        if (!given) __syncthreads();  // every group of every row has reported its absmax

        if (active && alive) {
            const float amax = given ? 0.0f : __uint_as_float(row_absmax[par * B + r]);
            const float scale =
                given ? args.given_scales[row0 + r] : row_scale<Bits>(amax, args.scale_mul != 0);
            if (grp == 0 && q == 0 && !given) args.scales[row0 + r] = scale;
            int8_t *out = args.codes + static_cast<int64_t>(row0 + r) * Kout;
            if constexpr (Bits == 4) {
                // Columns 2q + 16u and 2q + 16u + 1 share byte q + 8u of the group's 128.
                const float inv = __fdiv_rn(1.0f, scale);
                const f32x2 i2 = pk2(inv, inv);
                out += grp * 128 + q;
#pragma unroll
                for (int u = 0; u < 16; u += 4) {
                    const uint32_t c = quant8_int4(make_uint4(W[u], W[u + 1], W[u + 2], W[u + 3]), i2);
#pragma unroll
                    for (int i = 0; i < 4; ++i) out[8 * (u + i)] = static_cast<int8_t>((c >> (8 * i)) & 0xFFu);
                }
            } else {
                const float rs = __bfloat162float(__float2bfloat16_rn(scale));
                const bool exact = given ? (group_nan || !fast_chain_scale_ok(rs))
                                         : (row_nan[par * B + r] != 0u || isinf(amax));
                const float qparam = exact ? rs : __frcp_rn(rs);
                const f32x2 r2 = pk2(qparam, qparam);
                out += grp * 256 + 2 * q;
#pragma unroll
                for (int u = 0; u < 16; u += 4) {
                    const uint4 w4 = make_uint4(W[u], W[u + 1], W[u + 2], W[u + 3]);
                    const uint2 c = exact ? quant8_int8_exact(w4, qparam) : quant8_int8_fast(w4, r2);
                    uint16_t *o16 = reinterpret_cast<uint16_t *>(out + 16 * u);
                    o16[0] = static_cast<uint16_t>(c.x & 0xFFFFu);
                    o16[8] = static_cast<uint16_t>(c.x >> 16);
                    o16[16] = static_cast<uint16_t>(c.y & 0xFFFFu);
                    o16[24] = static_cast<uint16_t>(c.y >> 16);
                }
            }
        }
    }
    if (tid == 0 && !alive && issued > 0) {
        // A wait gave up: let the last copy land before the CTA exits.
        mbar_wait(full, (issued - 1) & 1u, nullptr, args.err, kErrTimeoutDrain);
    }
}

// ---------------------------------------------------------------------------
// Multi-group eight-lane kernel (convrot_quant_g8_kernel): the eight-lane layout above,
// with each 8-lane team rotating G groups per batch, the batch input double-buffered
// so it stays in shared memory until the batch's single CTA barrier, every per-lane
// address and the team's row/group assignment computed once per launch, and -- for
// bf16-valued inputs (plain rows and tanh-GELU, whose table values are bf16) -- the
// four per-stage halvings folded into the quantization.
//
// Why the fold is exact.  Every bf16 value is a multiple of 2^-133 (the bf16
// subnormal spacing), so every intermediate of the reference's rotation is a multiple
// of 2^-137: sums of multiples of a power of two stay multiples of it (a sum is
// rounded only when it needs more than 24 significant bits, and then onto a coarser
// grid that is itself a multiple), and each halving step removes one factor of two.
// 2^-137 is far above the fp32 subnormal spacing 2^-149, so no halving ever rounds and
// no sum in the subnormal range is inexact.  Rounding to nearest commutes with scaling
// by powers of two when nothing overflows, so the rotation without the halvings gives
// z = 16 y exactly, sum by sum, unless z overflows.  An overflow leaves an infinity or
// NaN in some output (neither ever turns finite again), so a group whose folded
// outputs are all finite has y = z / 16 exactly; a group with a non-finite output is
// recomputed in the reference's order from the still-resident input.  The codes then
// take the folded factor 1/16 in the reciprocal: bf16(z) * (r / 16) equals
// bf16(y) * r as exact products (r / 16 stays a normal fp32 value), and outputs small
// enough to fall below the normal range quantize to 0 on both paths.  SwiGLU inputs
// are fp32 products with spacings down to 2^-149, so they keep the halvings.
//
// Transpose addresses.  With garea 1024-byte aligned, the eight-lane placement
// k8_slot reduces to XORs of one per-lane base with constants:
//   write (c, h): garea + 16 k8_slot(g, 4q + c + 32h) = wbase ^ 16c            (h = 0)
//                                                    = (wbase ^ 16c ^ 64) + 512 (h = 1)
//   read u:       garea + 8 (q % 2) + 16 k8_slot(g, 4u + q / 2) = rbase ^ 16 (4u ^ u / 2)
// with wbase = garea + 16 (4q ^ q / 2 ^ 4 (g % 2)) and
// rbase = garea + 8 (q % 2) + 16 (q / 2 ^ 4 (g % 2)).
namespace {

__device__ __forceinline__ uint32_t ld_shared_u32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
    return v;
}

__device__ __forceinline__ void st_shared_u32(uint32_t addr, uint32_t v) {
    asm volatile("st.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ void atom_max_shared(uint32_t addr, uint32_t v) {
    asm volatile("red.shared.max.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ void atom_or_shared(uint32_t addr, uint32_t v) {
    asm volatile("red.shared.or.b32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

// bf16 words of one lane's 32 inputs, unpacked to the phase A pairs (element 16q + j,
// element 16q + j + 128); `ld[c]` / `ld[2 + c]` are the shared addresses of chunk c of
// the lane's slice and of the slice 2 later (the h = 1 half).
template <int Act>
__device__ __forceinline__ void g8_load(uint32_t base, const uint32_t (&ld)[4], f32x2 (&P)[16], const ActLut &lut) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        const uint4 a = ld_shared_v4u(base + ld[c]);
        const uint4 b = ld_shared_v4u(base + ld[2 + c]);
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

// SwiGLU inputs: the gate chunks at `ld`, the up chunks `up_bytes` later (not 1024-byte
// periodic, so their swizzled addresses are formed here from the slice index).
__device__ __forceinline__ void g8_load_swiglu(uint32_t base, uint32_t slice, uint32_t q, uint32_t up_slices,
                                               f32x2 (&P)[16], const ActLut &lut) {
    const uint32_t s = slice + (q >> 2);
    const uint32_t c0 = 2u * (q & 3u);
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        const uint4 a = ld_shared_v4u(base + sw128(s, c0 + c));
        const uint4 b = ld_shared_v4u(base + sw128(s + 2, c0 + c));
        const uint4 ua = ld_shared_v4u(base + sw128(s + up_slices, c0 + c));
        const uint4 ub = ld_shared_v4u(base + sw128(s + up_slices + 2, c0 + c));
        const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
        const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
        const uint32_t uaw[4] = {ua.x, ua.y, ua.z, ua.w};
        const uint32_t ubw[4] = {ub.x, ub.y, ub.z, ub.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            P[8 * c + 2 * i] = pk2(activate<kActSwiGLU>(aw[i] << 16, uaw[i] << 16, lut),
                                   activate<kActSwiGLU>(bw[i] << 16, ubw[i] << 16, lut));
            P[8 * c + 2 * i + 1] = pk2(activate<kActSwiGLU>(aw[i] & 0xFFFF0000u, uaw[i] & 0xFFFF0000u, lut),
                                       activate<kActSwiGLU>(bw[i] & 0xFFFF0000u, ubw[i] & 0xFFFF0000u, lut));
        }
    }
}

}  // namespace

// int4 codes of the 8 words W[u0 .. u0 + 8) with scale `scale` of the unscaled (folded)
// or halved rotation, the reference's int4 chain (see the row kernel below).
__device__ __forceinline__ void g8_int4_half(const uint32_t *W, float scale, bool folded, int8_t *out) {
    const float inv = __fdiv_rn(1.0f, scale);
    if (folded && !(inv >= 0x1p-100f)) {
#pragma unroll
        for (int u = 0; u < 8; u += 4) {
            const uint32_t c = quant8_int4_prescaled(make_uint4(W[u], W[u + 1], W[u + 2], W[u + 3]), inv);
#pragma unroll
            for (int i = 0; i < 4; ++i) out[8 * (u + i)] = static_cast<int8_t>((c >> (8 * i)) & 0xFFu);
        }
    } else {
        const float iv = folded ? inv * 0.0625f : inv;
        const f32x2 i2 = pk2(iv, iv);
#pragma unroll
        for (int u = 0; u < 8; u += 4) {
            const uint32_t c = quant8_int4(make_uint4(W[u], W[u + 1], W[u + 2], W[u + 3]), i2);
#pragma unroll
            for (int i = 0; i < 4; ++i) out[8 * (u + i)] = static_cast<int8_t>((c >> (8 * i)) & 0xFFu);
        }
    }
}

template <int Act, int Bits, int G, bool kGroupScales, bool kBlock128>
__global__ void __launch_bounds__(kG8MaxThreads)
    convrot_quant_g8_kernel(const __grid_constant__ CUtensorMap tmap_x, const QuantArgs args) {
    static_assert(!kGroupScales || (Act == kActNone && Bits == 4), "group scales: plain rows, int4 codes");
    static_assert(!kBlock128 || (Act == kActNone && (Bits == 8) != kGroupScales),
                  "block 128: plain rows, int8 codes or per-group int4 codes");
    constexpr bool kFold = Act != kActSwiGLU && !kBlock128;
    extern __shared__ uint8_t smem_raw[];
    // Shared-space addresses (32-bit), 1024-byte aligned as the 128-byte swizzle needs.
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t sbase = (raw + 1023u) & ~1023u;
    uint8_t *smem = smem_raw + (sbase - raw);
    const int K = args.k;
    const int B = args.rows_per_batch;
    const int Kout = Bits == 4 ? K / 2 : K;
    const int groups = K / 256;
    const int nwarps = blockDim.x >> 5;
    const int teams = 4 * nwarps;
    const uint32_t in_bytes = static_cast<uint32_t>(args.box_rows) * args.copies * 128u;  // multiple of 1024
    const uint32_t slices_per_row = (Act == kActSwiGLU ? 2 * K : K) / 64;
    const uint32_t xarea = sbase + 2 * in_bytes;                         // nwarps x 4 KB
    const uint32_t stats = xarea + static_cast<uint32_t>(nwarps) * kK8WarpBytes;  // absmax [3][B], flags [3][B]
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + 2 * in_bytes + nwarps * kK8WarpBytes + 24 * B);  // [2]

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const uint32_t g = static_cast<uint32_t>(lane >> 3);
    const uint32_t q = static_cast<uint32_t>(lane & 7);
    const int team = warp * 4 + static_cast<int>(g);
    const int num_batches = (args.m + B - 1) / B;
    const uint32_t slices_per_batch = static_cast<uint32_t>(B) * slices_per_row;
    const bool given = args.given_scales != nullptr;
    const ActLut lut{args.silu_lut, args.gelu_lut};

    // Per-lane constants.  Every batch holds B whole rows, so slot s of this team always
    // takes row r[s], group grp[s] of the batch (or nothing, where task >= B * groups).
    const uint32_t garea = xarea + static_cast<uint32_t>(warp) * kK8WarpBytes + g * kK8GroupBytes;
    const uint32_t wbase = garea + 16u * ((4u * q) ^ (q >> 1) ^ (4u * (g & 1u)));
    const uint32_t rbase = garea + 8u * (q & 1u) + 16u * ((q >> 1) ^ (4u * (g & 1u)));
    int r_of[G], grp_of[G];
    uint32_t slice_of[G];
    uint32_t ld[G][4];
#pragma unroll
    for (int s = 0; s < G; ++s) {
        const int task = team + s * teams;
        r_of[s] = task / groups;
        grp_of[s] = task - r_of[s] * groups;
        slice_of[s] = static_cast<uint32_t>(r_of[s]) * slices_per_row + static_cast<uint32_t>(grp_of[s]) * 4u;
        const uint32_t sl = slice_of[s] + (q >> 2);
        const uint32_t c0 = 2u * (q & 3u);
        ld[s][0] = sw128(sl, c0);
        ld[s][1] = sw128(sl, c0 + 1);
        ld[s][2] = sw128(sl + 2, c0);
        ld[s][3] = sw128(sl + 2, c0 + 1);
    }

    auto issue_load = [&](int batch, int buf) {
        mbar_arrive_expect_tx(&full[buf], in_bytes);
        for (int c = 0; c < args.copies; ++c) {
            const uint32_t s0 = static_cast<uint32_t>(c * args.box_rows);
            tma_load_2d(smem + buf * in_bytes + s0 * 128u, &tmap_x, 0, static_cast<int>(batch * slices_per_batch + s0),
                        &full[buf]);
        }
    };

    if (tid == 0) {
        mbar_init(&full[0], 1);
        mbar_init(&full[1], 1);
        fence_mbar_init();
    }
    for (int i = tid; i < 6 * B; i += blockDim.x) st_shared_u32(stats + 4u * i, 0u);
    __syncthreads();
    uint32_t issued[2] = {0, 0};
    if (tid == 0) {
        prefetch_tmap(&tmap_x);
        for (int b = 0; b < 2; ++b) {
            const int batch = blockIdx.x + b * gridDim.x;
            if (batch < num_batches) {
                issue_load(batch, b);
                issued[b] = 1;
            }
        }
    }

    bool alive = true;
    int par = 0;  // statistics slot of this batch: it % 3
    for (int it = 0;; ++it, par = par == 2 ? 0 : par + 1) {
        const int batch = blockIdx.x + it * gridDim.x;
        if (batch >= num_batches) break;
        const int buf = it & 1;
        const int row0 = batch * B;
        const int tasks = min(B, args.m - row0) * groups;
        const uint32_t in = sbase + static_cast<uint32_t>(buf) * in_bytes;
        const uint32_t amax_slot = stats + 4u * static_cast<uint32_t>(par * B);
        const uint32_t flag_slot = amax_slot + 12u * static_cast<uint32_t>(B);

        if (alive) alive = mbar_wait(&full[buf], static_cast<uint32_t>((it >> 1) & 1), nullptr, args.err,
                                     kErrTimeoutFull);
        alive = __all_sync(0xffffffffu, alive);  // the rotation's shuffles need every lane of the warp
        uint32_t W[G][16];
        bool folded[G];
        bool group_nan[G];
#pragma unroll
        for (int s = 0; s < G; ++s) {
            folded[s] = false;
            group_nan[s] = false;
            if (!alive || warp * 4 + s * teams >= tasks) continue;  // warp-uniform
            const bool active = team + s * teams < tasks;
            float amax = 0.0f, probe = 0.0f, amax_hi = 0.0f;
            bool exact = true;
            if constexpr (kFold) {
                f32x2 P[16];
                g8_load<Act>(in, ld[s], P, lut);
                g8_rotate<false, kGroupScales>(P, wbase, rbase, W[s], amax, probe, amax_hi);
                exact = __any_sync(0xffffffffu, !(amax <= 3.40282347e38f) || !(amax_hi <= 3.40282347e38f));
                if (!exact) {
                    folded[s] = true;
                    amax *= 0.0625f;
                    amax_hi *= 0.0625f;
                }
            }
            if (exact) {  // warp-uniform: the reference's order, halvings included
                f32x2 P[16];
                if constexpr (Act == kActSwiGLU) g8_load_swiglu(in, slice_of[s], q, static_cast<uint32_t>(K / 64), P, lut);
                else g8_load<Act>(in, ld[s], P, lut);
                g8_rotate<true, kGroupScales, true, kBlock128>(P, wbase, rbase, W[s], amax, probe, amax_hi);
                group_nan[s] = isnan(probe);
            }
            if constexpr (kGroupScales) {
                // Each 128-column half of the group is quantized on its own, right here.
                if (active) {
                    const int64_t row = row0 + r_of[s];
                    int8_t *out = args.codes + row * (K / 2) + grp_of[s] * 128 + q;
                    float *gs = args.group_scales + row * (K / 128) + 2 * grp_of[s];
                    const float scale_lo = row_scale<4>(amax, false);
                    const float scale_hi = row_scale<4>(amax_hi, false);
                    if (q == 0) {
                        gs[0] = scale_lo;
                        gs[1] = scale_hi;
                    }
                    g8_int4_half(&W[s][0], scale_lo, folded[s], out);
                    g8_int4_half(&W[s][8], scale_hi, folded[s], out + 64);
                }
                continue;
            }
            if (active && q == 0 && !given) {
                atom_max_shared(amax_slot + 4u * r_of[s], __float_as_uint(amax));
                if (group_nan[s]) atom_or_shared(flag_slot + 4u * r_of[s], 1u);
            }
        }
        __syncthreads();  // every group has reported its absmax; buffer `buf` is consumed
        if (tid == 0 && alive) {
            const int next = batch + 2 * gridDim.x;
            if (next < num_batches) {
                issue_load(next, buf);
                ++issued[buf];
            }
        }
        {
            // Slot (it + 2) % 3 was read two batches ago and is written again next batch.
            const uint32_t clear = stats + 4u * static_cast<uint32_t>((par == 0 ? 2 : par - 1) * B);
            for (int i = tid; i < B; i += blockDim.x) {
                st_shared_u32(clear + 4u * i, 0u);
                st_shared_u32(clear + 12u * B + 4u * i, 0u);
            }
        }

        if constexpr (kGroupScales) continue;
#pragma unroll
        for (int s = 0; s < G; ++s) {
            if (!alive || team + s * teams >= tasks) continue;
            const int r = r_of[s];
            const int grp = grp_of[s];
            const float amax = given ? 0.0f : __uint_as_float(ld_shared_u32(amax_slot + 4u * r));
            const float scale = given ? args.given_scales[row0 + r] : row_scale<Bits>(amax, args.scale_mul != 0);
            if (grp == 0 && q == 0 && !given) args.scales[row0 + r] = scale;
            int8_t *out = args.codes + static_cast<int64_t>(row0 + r) * Kout;
            if constexpr (Bits == 4) {
                const float inv = __fdiv_rn(1.0f, scale);
                out += grp * 128 + q;
                if (folded[s] && !(inv >= 0x1p-100f)) {
#pragma unroll
                    for (int u = 0; u < 16; u += 4) {
                        const uint32_t c = quant8_int4_prescaled(
                            make_uint4(W[s][u], W[s][u + 1], W[s][u + 2], W[s][u + 3]), inv);
#pragma unroll
                        for (int i = 0; i < 4; ++i) out[8 * (u + i)] = static_cast<int8_t>((c >> (8 * i)) & 0xFFu);
                    }
                } else {
                    const float iv = folded[s] ? inv * 0.0625f : inv;
                    const f32x2 i2 = pk2(iv, iv);
#pragma unroll
                    for (int u = 0; u < 16; u += 4) {
                        const uint32_t c = quant8_int4(make_uint4(W[s][u], W[s][u + 1], W[s][u + 2], W[s][u + 3]), i2);
#pragma unroll
                        for (int i = 0; i < 4; ++i) out[8 * (u + i)] = static_cast<int8_t>((c >> (8 * i)) & 0xFFu);
                    }
                }
            } else {
                const float rs = __bfloat162float(__float2bfloat16_rn(scale));
                const bool exact_chain = given ? (group_nan[s] || !fast_chain_scale_ok(rs))
                                               : (ld_shared_u32(flag_slot + 4u * r) != 0u || isinf(amax));
                uint16_t *o16 = reinterpret_cast<uint16_t *>(out + grp * 256 + 2 * q);
                if (exact_chain) {
                    const float divisor = folded[s] ? rs * 16.0f : rs;
#pragma unroll
                    for (int u = 0; u < 16; u += 4) {
                        const uint2 c = quant8_int8_exact(make_uint4(W[s][u], W[s][u + 1], W[s][u + 2], W[s][u + 3]),
                                                          divisor);
                        o16[8 * u] = static_cast<uint16_t>(c.x & 0xFFFFu);
                        o16[8 * u + 8] = static_cast<uint16_t>(c.x >> 16);
                        o16[8 * u + 16] = static_cast<uint16_t>(c.y & 0xFFFFu);
                        o16[8 * u + 24] = static_cast<uint16_t>(c.y >> 16);
                    }
                } else {
                    const float rc = __frcp_rn(rs) * (folded[s] ? 0.0625f : 1.0f);
                    const f32x2 r2 = pk2(rc, rc);
#pragma unroll
                    for (int u = 0; u < 16; ++u) o16[8 * u] = static_cast<uint16_t>(quant2_int8_fast(W[s][u], r2));
                }
            }
        }
    }
    if (tid == 0 && !alive) {
        // A wait gave up: let the copies still in flight land before the CTA exits.
        for (int b = 0; b < 2; ++b) {
            if (issued[b] > 0) mbar_wait(&full[b], (issued[b] - 1) & 1u, nullptr, args.err, kErrTimeoutDrain);
        }
    }
}

// ---------------------------------------------------------------------------
// Warp-row kernel (convrot_quant_w8_kernel).  Each warp owns whole rows, so the row
// absmax is a warp reduction and no CTA barrier is ever taken: lane 0 copies the row
// (contiguous bf16) into the warp's buffer with one bulk copy, the four 8-lane teams
// rotate groups team, team + 4, ... (kGt each) exactly as the multi-group kernel does --
// the halvings folded, the reference order recomputed from the still-resident input for
// a slot where any group of the warp left the finite range -- keeping the bf16 words in
// registers, and as soon as the last group is read lane 0 issues the next row's copy,
// which lands while the row is quantized.
//
// Inputs are read as plain row-major bf16 (no swizzle): lane q of a team reads elements
// 16q .. 16q + 15 and 128 + 16q .. 128 + 16q + 15 of its group, the layout the
// transpose of g8_rotate expects.  The rotation and code chains are the warp-row
// pipeline of convrot_rowwarp.cuh.

template <int Act, int Bits, int kGt, bool kBlock128>
__global__ void __launch_bounds__(32 * kW8Warps)
    convrot_quant_w8_kernel(const __grid_constant__ CUtensorMap tmap_x, const QuantArgs args) {
    static_assert(Act != kActSwiGLU, "the warp-row kernel takes bf16-valued rows");
    static_assert(!kBlock128 || (Act == kActNone && Bits == 8), "block 128: plain int8 rows");
    static_assert(kGt >= 1 && kGt <= kW8MaxGroupsPerTeam, "groups per team");
    (void)tmap_x;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t sbase = (raw + 1023u) & ~1023u;
    uint8_t *smem = smem_raw + (sbase - raw);
    const int K = args.k;
    const int groups = K / 256;
    const int Kout = Bits == 4 ? K / 2 : K;
    const uint32_t row_bytes = static_cast<uint32_t>(K) * 2u;
    const uint32_t buf_bytes = (row_bytes + 1023u) & ~1023u;
    const uint32_t warp_stride = buf_bytes + static_cast<uint32_t>(kK8WarpBytes);
    const int nwarps = blockDim.x >> 5;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t g = static_cast<uint32_t>(lane >> 3);  // team
    const uint32_t q = static_cast<uint32_t>(lane & 7);
    const uint32_t buf = sbase + static_cast<uint32_t>(warp) * warp_stride;
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + static_cast<uint32_t>(nwarps) * warp_stride) + warp;
    const uint32_t garea = buf + buf_bytes + g * kK8GroupBytes;
    const uint32_t wbase = garea + 16u * ((4u * q) ^ (q >> 1) ^ (4u * (g & 1u)));
    const uint32_t rbase = garea + 8u * (q & 1u) + 16u * ((q >> 1) ^ (4u * (g & 1u)));
    const ActLut lut{args.silu_lut, args.gelu_lut};
    const uint16_t *x = static_cast<const uint16_t *>(args.x);
    const int row_step = gridDim.x * nwarps;
    const int first = blockIdx.x * nwarps + warp;

    if (lane == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
        if (first < args.m) {
            mbar_arrive_expect_tx(bar, row_bytes);
            bulk_load(smem + (buf - sbase), x + static_cast<int64_t>(first) * K, row_bytes, bar);
        }
    }
    __syncwarp();

    uint32_t it = 0;
    bool pending = first < args.m;  // lane 0: a copy is in flight
    for (int row = first; row < args.m; row += row_step, ++it) {
        const bool ok = mbar_wait(bar, it & 1u, nullptr, args.err, kErrTimeoutFull);
        if (!__all_sync(0xffffffffu, ok)) break;
        pending = false;

        uint32_t W[kGt][16];
        bool folded[kGt];
        bool any_nan = false;
        float amax = 0.0f;
        w8_rotate_row<Act, kGt, kBlock128>(buf, groups, g, q, wbase, rbase, lut, W, folded, amax, any_nan);
        const int next = row + row_step;
        if (lane == 0 && next < args.m) {
            mbar_arrive_expect_tx(bar, row_bytes);
            bulk_load(smem + (buf - sbase), x + static_cast<int64_t>(next) * K, row_bytes, bar);
            pending = true;
        }
        amax = w8_row_absmax(amax);
        const bool row_nan = __any_sync(0xffffffffu, any_nan);
        const float scale = row_scale<Bits>(amax, args.scale_mul != 0);
        if (lane == 0) args.scales[row] = scale;
        w8_store_codes<Bits, kGt>(W, folded, amax, scale, row_nan, groups, g, q,
                                  args.codes + static_cast<int64_t>(row) * Kout);
    }
    if (lane == 0 && pending) {
        // A wait gave up with a copy still in flight: let it land before the CTA exits.
        mbar_wait(bar, it & 1u, nullptr, args.err, kErrTimeoutDrain);
    }
}

template __global__ void convrot_quant_k8_kernel<kActNone, 8>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_k8_kernel<kActNone, 4>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_k8_kernel<kActSwiGLU, 8>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_k8_kernel<kActSwiGLU, 4>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_k8_kernel<kActGelu, 8>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_k8_kernel<kActGelu, 4>(const __grid_constant__ CUtensorMap, const QuantArgs);

template __global__ void convrot_quant_g8_kernel<kActNone, 8, 1>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_g8_kernel<kActNone, 8, 2>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_g8_kernel<kActNone, 4, 1>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_g8_kernel<kActNone, 4, 2>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_g8_kernel<kActSwiGLU, 8, 1>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_g8_kernel<kActSwiGLU, 8, 2>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_g8_kernel<kActSwiGLU, 4, 1>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_g8_kernel<kActSwiGLU, 4, 2>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_g8_kernel<kActGelu, 8, 1>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_g8_kernel<kActGelu, 8, 2>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_g8_kernel<kActGelu, 4, 1>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_g8_kernel<kActGelu, 4, 2>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActNone, 8, 1>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActNone, 8, 2>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActNone, 8, 3>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActNone, 8, 4>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActNone, 8, 5>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActNone, 8, 6>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActNone, 4, 1>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActNone, 4, 2>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActNone, 4, 3>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActNone, 4, 4>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActNone, 4, 5>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActNone, 4, 6>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActGelu, 8, 1>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActGelu, 8, 2>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActGelu, 8, 3>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActGelu, 8, 4>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActGelu, 8, 5>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActGelu, 8, 6>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActGelu, 4, 1>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActGelu, 4, 2>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActGelu, 4, 3>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActGelu, 4, 4>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActGelu, 4, 5>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActGelu, 4, 6>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_g8_kernel<kActNone, 4, 1, true>(const __grid_constant__ CUtensorMap,
                                                                       const QuantArgs);
// Rotation block 128 (plain rows: int8, and per-group int4).
template __global__ void convrot_quant_g8_kernel<kActNone, 4, 1, true, true>(const __grid_constant__ CUtensorMap,
                                                                             const QuantArgs);
template __global__ void convrot_quant_g8_kernel<kActNone, 4, 2, true, true>(const __grid_constant__ CUtensorMap,
                                                                             const QuantArgs);
template __global__ void convrot_quant_g8_kernel<kActNone, 8, 1, false, true>(const __grid_constant__ CUtensorMap,
                                                                              const QuantArgs);
template __global__ void convrot_quant_g8_kernel<kActNone, 8, 2, false, true>(const __grid_constant__ CUtensorMap,
                                                                              const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActNone, 8, 1, true>(const __grid_constant__ CUtensorMap,
                                                                       const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActNone, 8, 2, true>(const __grid_constant__ CUtensorMap,
                                                                       const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActNone, 8, 3, true>(const __grid_constant__ CUtensorMap,
                                                                       const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActNone, 8, 4, true>(const __grid_constant__ CUtensorMap,
                                                                       const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActNone, 8, 5, true>(const __grid_constant__ CUtensorMap,
                                                                       const QuantArgs);
template __global__ void convrot_quant_w8_kernel<kActNone, 8, 6, true>(const __grid_constant__ CUtensorMap,
                                                                       const QuantArgs);
template __global__ void convrot_quant_g8_kernel<kActNone, 4, 2, true>(const __grid_constant__ CUtensorMap,
                                                                       const QuantArgs);

}  // namespace rot
}  // namespace ctu
