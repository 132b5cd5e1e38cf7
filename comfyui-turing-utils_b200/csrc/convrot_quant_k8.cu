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
#include "ptx.cuh"

namespace ctu {
namespace rot {

namespace {

__device__ __forceinline__ uint32_t k8_slot(uint32_t g, uint32_t t) { return t ^ ((t >> 3) & 7u) ^ (4u * (g & 1u)); }

__device__ __forceinline__ void st_shared_v4(uint32_t addr, float a, float b, float c, float d) {
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

__device__ __forceinline__ float2 ld_shared_v2(uint32_t addr) {
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr) : "memory");
    return v;
}

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

template __global__ void convrot_quant_k8_kernel<kActNone, 8>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_k8_kernel<kActNone, 4>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_k8_kernel<kActSwiGLU, 8>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_k8_kernel<kActSwiGLU, 4>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_k8_kernel<kActGelu, 8>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_k8_kernel<kActGelu, 4>(const __grid_constant__ CUtensorMap, const QuantArgs);

}  // namespace rot
}  // namespace ctu
