// ConvRot rotate + per-token quantize with four lanes per 256-column group and a
// shared-memory transpose between the rotation stages: the same arithmetic as the
// register-resident kernel (convrot_quant_reg.cu; reference kernel/csrc/turing/
// convrot_quant.cu:417-511) at half its registers per lane, so twice the warps fit on
// an SM.  It executes a few more instructions per element than the two-lane kernel (the
// transpose and 4-byte code stores); it wins where the two-lane kernel leaves lane-pair
// slots idle or the activation adds work: narrow rows and the fused SwiGLU / GELU inputs.
//
// Element e of a group has index bits 0-7; each radix-4 stage s combines the four
// elements that differ in bits (2s-2, 2s-1).
//   * Phase A: lane q of the group holds elements 64q + j, j < 64 (one 128-byte TMA
//     slice), as 32 packed pairs (j, j + 32).  Stages 1 and 2 (bits 0-3) run in
//     registers; bit 5 pairs the packed halves, which neither stage touches.
//   * Transpose: each lane writes its 64 values to the warp's shared-memory area as
//     8-byte pairs (e, e + 1); after __syncwarp, lane q' reads the 16-byte chunks of the
//     elements whose bits 2-3 equal q' (16u + 4q' + r, u < 16, r < 4).
//   * Phase B: stages 3 and 4 (bits 4-7 = bits 0-3 of u) run in registers on pairs
//     (r, r + 1); the outputs come out as bf16 pairs of consecutive columns, ready for
//     the code conversion and 4-byte global stores.
// Shared-memory placement of a group (1 KB, 64 chunks of 16 bytes): chunk t = e / 4 sits
// at slot t ^ h(g, t / 16) and word r = e % 4 at position r ^ (t / 16 & 2), with
// h(g, q) = 4 (g & 1) + 2 (g / 2 & 1) + (q & 1) for the warp-local group index g.  The
// 8-byte writes of each half-warp (4 groups x 4 lanes) and the 16-byte reads of each
// quarter-warp (2 groups x 4 lanes) then touch distinct banks, and the word permutation
// only swaps whole pairs, so phase B's packed pairs need no register moves.
//
// Batches, row statistics and the quantization chains are those of the register-resident
// kernel: whole rows per CTA batch, per-row absmax in shared memory, a NaN probe that
// selects the exact reference chain, caller-supplied scales for the SwiGLU shard op.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "convrot_math.cuh"
#include "convrot_quant.cuh"
#include "ptx.cuh"

namespace ctu {
namespace rot {

namespace {

constexpr int kT4GroupWords = 256;                    // fp32 words of one group in the transpose area
constexpr int kT4WarpBytes = 8 * kT4GroupWords * 4;   // 8 groups per warp

__device__ __forceinline__ uint32_t t4_swizzle(uint32_t g, uint32_t q) {
    return 4u * (g & 1u) + 2u * ((g >> 1) & 1u) + (q & 1u);
}

__device__ __forceinline__ void st_shared_f32x2(uint32_t addr, float a, float b) {
    asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(a), "f"(b) : "memory");
}

__device__ __forceinline__ float4 ld_shared_f32x4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}

// Phase A load: lane q's 64 inputs of the group (slice row64 of the batch buffer);
// P[j] = (element j, element j + 32) of the slice.
template <int Act>
__device__ __forceinline__ void t4_load(const uint8_t *buf, uint32_t row64, uint32_t up_off, f32x2 (&P)[32],
                                        const ActLut &lut) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint4 a = *reinterpret_cast<const uint4 *>(buf + sw128(row64, c));
        const uint4 b = *reinterpret_cast<const uint4 *>(buf + sw128(row64, c + 4));
        const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
        const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
        if constexpr (Act == kActSwiGLU) {
            const uint4 ua = *reinterpret_cast<const uint4 *>(buf + sw128(row64 + up_off, c));
            const uint4 ub = *reinterpret_cast<const uint4 *>(buf + sw128(row64 + up_off, c + 4));
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

// Rotation of the group held by the warp's 4-lane team (all 32 lanes call it together:
// __syncwarp and the lane-team reductions).  Returns the lane's bf16 words W[u][h] =
// (y[16u + 4q' + 2h], y[16u + 4q' + 2h + 1]) and the team's absmax / NaN probe.
__device__ __forceinline__ void t4_rotate(f32x2 (&P)[32], uint32_t xarea, uint32_t g, uint32_t q,
                                          uint32_t (&W)[16][2], float &absmax, float &nan_probe) {
    const f32x2 half = pk2(0.5f, 0.5f);
    // Stage 1 (bits 0-1) and stage 2 (bits 2-3) on pairs (j, j + 32).
#pragma unroll
    for (int a = 0; a < 8; ++a) butterfly2(P[4 * a], P[4 * a + 1], P[4 * a + 2], P[4 * a + 3], half);
#pragma unroll
    for (int b = 0; b < 2; ++b) {
#pragma unroll
        for (int p = 0; p < 4; ++p)
            butterfly2(P[16 * b + p], P[16 * b + p + 4], P[16 * b + p + 8], P[16 * b + p + 12], half);
    }
    // Transpose through shared memory: pairs (e, e + 1), e = 64q + j, j even.
    const uint32_t garea = xarea + g * (kT4GroupWords * 4);
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) {
        float a0, a1, b0, b1;
        unpk2(P[2 * jj], a0, a1);      // elements j, j + 32
        unpk2(P[2 * jj + 1], b0, b1);  // elements j + 1, j + 33
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            const uint32_t j = 2u * jj + 32u * hf;
            const uint32_t t = 16u * q + (j >> 2);
            const uint32_t slot = t ^ t4_swizzle(g, q);
            const uint32_t word = (j & 3u) ^ (q & 2u);
            st_shared_f32x2(garea + 16u * slot + 4u * word, hf ? a1 : a0, hf ? b1 : b0);
        }
    }
    __syncwarp();
    f32x2 R[16][2];
#pragma unroll
    for (int u = 0; u < 16; ++u) {
        const uint32_t qw = static_cast<uint32_t>(u) >> 2;  // the phase-A lane that wrote this chunk
        const uint32_t t = 4u * u + q;
        const float4 v = ld_shared_f32x4(garea + 16u * (t ^ t4_swizzle(g, qw)));
        if (qw & 2u) {
            R[u][0] = pk2(v.z, v.w);
            R[u][1] = pk2(v.x, v.y);
        } else {
            R[u][0] = pk2(v.x, v.y);
            R[u][1] = pk2(v.z, v.w);
        }
    }
    __syncwarp();  // the area is rewritten by the next batch only after these reads
    // Stage 3 (bits 4-5 = bits 0-1 of u) and stage 4 (bits 6-7 = bits 2-3 of u).
#pragma unroll
    for (int v = 0; v < 4; ++v) {
#pragma unroll
        for (int h = 0; h < 2; ++h) butterfly2(R[4 * v][h], R[4 * v + 1][h], R[4 * v + 2][h], R[4 * v + 3][h], half);
    }
#pragma unroll
    for (int w = 0; w < 4; ++w) {
#pragma unroll
        for (int h = 0; h < 2; ++h) butterfly2(R[w][h], R[w + 4][h], R[w + 8][h], R[w + 12][h], half);
    }
    float m = 0.0f;
    f32x2 probe = pk2(0.0f, 0.0f);
#pragma unroll
    for (int u = 0; u < 16; ++u) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float lo, hi;
            unpk2(R[u][h], lo, hi);
            probe = fadd2(probe, R[u][h]);
            m = max_abs3(m, lo, hi);
            W[u][h] = pack_bf16x2(lo, hi);
        }
    }
    float p0, p1;
    unpk2(probe, p0, p1);
    float pr = __fadd_rn(p0, p1);
    // Team (4 lanes) reductions; NaN-ignoring max as the reference's fmaxf.
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    pr = __fadd_rn(pr, __shfl_xor_sync(0xffffffffu, pr, 1));
    pr = __fadd_rn(pr, __shfl_xor_sync(0xffffffffu, pr, 2));
    absmax = m;
    nan_probe = pr;
}

}  // namespace

template <int Act, int Bits>
__global__ void __launch_bounds__(kT4MaxThreads, 1)
    convrot_quant_t4_kernel(const __grid_constant__ CUtensorMap tmap_x, const QuantArgs args) {
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
    uint8_t *xbase = smem + in_bytes;                                         // nwarps x 8 KB
    uint32_t *row_absmax = reinterpret_cast<uint32_t *>(xbase + nwarps * kT4WarpBytes);  // [2][B]
    uint32_t *row_nan = row_absmax + 2 * B;                                   // [2][B]
    uint64_t *full = reinterpret_cast<uint64_t *>(row_nan + 2 * B);          // 8-byte aligned

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const uint32_t g = static_cast<uint32_t>(lane >> 2);  // group slot in the warp
    const uint32_t q = static_cast<uint32_t>(lane & 3);   // lane in the group's team
    const uint32_t xarea = smem_u32(xbase + warp * kT4WarpBytes);
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

    const int team = warp * 8 + static_cast<int>(g);  // group task of this lane's team
    bool alive = true;

    for (int it = 0;; ++it) {
        const int batch = blockIdx.x + it * gridDim.x;
        if (batch >= num_batches) break;
        const int par = it & 1;
        const int row0 = batch * B;
        const int rows = min(B, args.m - row0);
        const int tasks = rows * groups;
        const bool warp_busy = warp * 8 < tasks;  // warp-uniform
        const bool active = team < tasks;
        const int task = active ? team : 0;
        const int r = task / groups;
        const int grp = task - r * groups;

        if (alive) alive = mbar_wait(full, static_cast<uint32_t>(it & 1), nullptr, args.err, kErrTimeoutFull);
        f32x2 P[32];
        if (warp_busy && alive)
            t4_load<Act>(inbuf, r * slices_per_row + grp * 4 + q, static_cast<uint32_t>(K / 64), P, lut);
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

        uint32_t W[16][2];
        bool group_nan = false;
        if (warp_busy && alive) {
            float amax, probe;
            t4_rotate(P, xarea, g, q, W, amax, probe);
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
                const float inv = __fdiv_rn(1.0f, scale);
                const f32x2 i2 = pk2(inv, inv);
                out += grp * 128 + 2 * q;
#pragma unroll
                for (int u = 0; u < 16; u += 2) {
                    const uint32_t c = quant8_int4(make_uint4(W[u][0], W[u][1], W[u + 1][0], W[u + 1][1]), i2);
                    *reinterpret_cast<uint16_t *>(out + 8 * u) = static_cast<uint16_t>(c & 0xFFFFu);
                    *reinterpret_cast<uint16_t *>(out + 8 * (u + 1)) = static_cast<uint16_t>(c >> 16);
                }
            } else {
                const float rs = __bfloat162float(__float2bfloat16_rn(scale));
                const bool exact = given ? (group_nan || !fast_chain_scale_ok(rs))
                                         : (row_nan[par * B + r] != 0u || isinf(amax));
                const float qparam = exact ? rs : __frcp_rn(rs);
                const f32x2 r2 = pk2(qparam, qparam);
                out += grp * 256 + 4 * q;
#pragma unroll
                for (int u = 0; u < 16; u += 2) {
                    const uint4 w4 = make_uint4(W[u][0], W[u][1], W[u + 1][0], W[u + 1][1]);
                    const uint2 c = exact ? quant8_int8_exact(w4, qparam) : quant8_int8_fast(w4, r2);
                    *reinterpret_cast<uint32_t *>(out + 16 * u) = c.x;
                    *reinterpret_cast<uint32_t *>(out + 16 * (u + 1)) = c.y;
                }
            }
        }
    }
    if (tid == 0 && !alive && issued > 0) {
        // A wait gave up: let the last copy land before the CTA exits.
        mbar_wait(full, (issued - 1) & 1u, nullptr, args.err, kErrTimeoutDrain);
    }
}

template __global__ void convrot_quant_t4_kernel<kActNone, 8>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_t4_kernel<kActNone, 4>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_t4_kernel<kActSwiGLU, 8>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_t4_kernel<kActSwiGLU, 4>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_t4_kernel<kActGelu, 8>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_t4_kernel<kActGelu, 4>(const __grid_constant__ CUtensorMap, const QuantArgs);

}  // namespace rot
}  // namespace ctu
