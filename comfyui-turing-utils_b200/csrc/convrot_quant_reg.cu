// Register-resident ConvRot rotate + per-token quantize for rows of at most
// kRegMaxGroups 256-column groups (K <= 32768; every width the reference's model
// adapters use).  Same arithmetic as the two-pass kernel in convrot_quant.cu, and the
// same reference (kernel/csrc/turing/convrot_quant.cu:417-511); the difference is
// where bf16(y) lives between the rotation and the quantization:
//
//   * A CTA processes a batch of whole rows at a time: every 256-column group of the
//     batch is owned by one lane pair (lane h holds the 128 elements whose bit 6 is h,
//     as 64 packed f32x2 pairs), so all groups of a row are resident in the CTA at once.
//   * The batch streams into shared memory by TMA (2D tensor map over 128-byte slices,
//     128-byte swizzle).  Each lane pair moves its group into registers; one CTA
//     barrier later the buffer is free and the next batch's copy is issued, so it lands
//     while this batch computes.
//   * The rotation (stages 1-3 in registers, stage 4 across the lane pair) leaves
//     bf16(y) packed two per register (64 registers per lane); the group's absmax
//     goes to a per-row slot in shared memory (atomicMax on the float bits).
//   * After a second CTA barrier every lane reads its row's absmax, forms the scale and
//     quantizes its 128 values straight from registers, storing the codes with
//     16-byte global stores.  bf16(y) never returns to shared memory and the codes
//     need no staging buffer.
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

// Stages 1-4 of the group held by this lane pair (inputs in v), producing bf16(y) as
// packed words: wa[i] = (y[h*64 + 2i], y[h*64 + 2i + 1]) and wb[i] the same 128
// columns later, the lane's absmax over the unrounded fp32 y (NaN ignored) and a NaN
// probe (the sum of the lane's y).  All 32 lanes of the warp must call this together.
__device__ __forceinline__ void rotate_to_words(f32x2 (&v)[64], int h, uint32_t (&wa)[32], uint32_t (&wb)[32],
                                                float &absmax, float &nan_probe) {
    const f32x2 half = pk2(0.5f, 0.5f);
#pragma unroll
    for (int q = 0; q < 16; ++q) butterfly2(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3], half);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int p = 0; p < 4; ++p)
            butterfly2(v[16 * c + p], v[16 * c + p + 4], v[16 * c + p + 8], v[16 * c + p + 12], half);
    }
#pragma unroll
    for (int p = 0; p < 16; ++p) butterfly2(v[p], v[p + 16], v[p + 32], v[p + 48], half);

    // Stage 4 (stride 64) across the lane pair; see rotate_group in convrot_quant.cu
    // for the derivation of the lane-uniform form of the four outputs.
    const unsigned full = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    const int lane0 = lane & ~1;
    const f32x2 sgn = h ? pk2(-1.0f, -1.0f) : pk2(1.0f, 1.0f);
    const f32x2 hsgn = h ? pk2(-0.5f, -0.5f) : pk2(0.5f, 0.5f);
    float m = 0.0f;
    f32x2 probe = pk2(0.0f, 0.0f);
#pragma unroll
    for (int j = 0; j < 64; j += 2) {
        float o0, o0y, o1, o1y;
        unpk2(v[j], o0, o0y);
        unpk2(v[j + 1], o1, o1y);
        const float t0 = __shfl_xor_sync(full, o0, 1);
        const float t1 = __shfl_xor_sync(full, o1, 1);
        const float a0 = __shfl_sync(full, o0y, lane0);
        const float a1 = __shfl_sync(full, o1y, lane0);
        const float b0 = __shfl_sync(full, o0y, lane0 + 1);
        const float b1 = __shfl_sync(full, o1y, lane0 + 1);
        const f32x2 own = pk2(o0, o1);
        const f32x2 other = pk2(t0, t1);
        const f32x2 x2 = pk2(a0, a1);
        const f32x2 x3 = pk2(b0, b1);
        const f32x2 p = fadd2(own, other);
        const f32x2 d = fsub2(own, other);
        const f32x2 ya = fmul2(hsgn, fsub2(ffma2(sgn, p, x2), x3));
        const f32x2 yb = fmul2(half, fadd2(fadd2(d, x2), x3));
        probe = fadd2(probe, fadd2(ya, yb));
        float ya0, ya1, yb0, yb1;
        unpk2(ya, ya0, ya1);
        unpk2(yb, yb0, yb1);
        m = max_abs3(m, ya0, ya1);
        m = max_abs3(m, yb0, yb1);
        wa[j >> 1] = pack_bf16x2(ya0, ya1);
        wb[j >> 1] = pack_bf16x2(yb0, yb1);
    }
    float p0, p1;
    unpk2(probe, p0, p1);
    absmax = m;
    nan_probe = __fadd_rn(p0, p1);
}

// int8 codes of 64 consecutive columns (32 words of bf16(y)) to dst (16-byte aligned).
__device__ __forceinline__ void store_run_int8(int8_t *dst, const uint32_t (&w)[32], bool exact, float qparam) {
    const f32x2 r2 = pk2(qparam, qparam);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint4 w0 = make_uint4(w[8 * c], w[8 * c + 1], w[8 * c + 2], w[8 * c + 3]);
        const uint4 w1 = make_uint4(w[8 * c + 4], w[8 * c + 5], w[8 * c + 6], w[8 * c + 7]);
        uint2 q0, q1;
        if (exact) {
            q0 = quant8_int8_exact(w0, qparam);
            q1 = quant8_int8_exact(w1, qparam);
        } else {
            q0 = quant8_int8_fast(w0, r2);
            q1 = quant8_int8_fast(w1, r2);
        }
        *reinterpret_cast<uint4 *>(dst + 16 * c) = make_uint4(q0.x, q0.y, q1.x, q1.y);
    }
}

// Packed int4 codes of 64 consecutive columns to dst (32 bytes, 16-byte aligned).
__device__ __forceinline__ void store_run_int4(int8_t *dst, const uint32_t (&w)[32], float inv) {
    const f32x2 i2 = pk2(inv, inv);
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        uint32_t q[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int b = 16 * c + 4 * e;
            q[e] = quant8_int4(make_uint4(w[b], w[b + 1], w[b + 2], w[b + 3]), i2);
        }
        *reinterpret_cast<uint4 *>(dst + 16 * c) = make_uint4(q[0], q[1], q[2], q[3]);
    }
}

}  // namespace

template <int Act, int Bits>
__global__ void __launch_bounds__(kRegMaxThreads, 1)
    convrot_quant_reg_kernel(const __grid_constant__ CUtensorMap tmap_x, const QuantArgs args) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int K = args.k;
    const int B = args.rows_per_batch;
    const int Kin = Act == kActSwiGLU ? 2 * K : K;
    const int Kout = Bits == 4 ? K / 2 : K;
    const int groups = K / 256;
    const uint32_t in_bytes = static_cast<uint32_t>(args.box_rows) * args.copies * 128u;  // multiple of 1024
    const uint32_t slices_per_row = Kin / 64;
    uint8_t *inbuf = smem;
    uint32_t *row_absmax = reinterpret_cast<uint32_t *>(smem + in_bytes);  // [2][B]
    uint32_t *row_nan = row_absmax + 2 * B;                                // [2][B]
    uint64_t *full = reinterpret_cast<uint64_t *>(row_nan + 2 * B);  // offset in_bytes + 16 B: 8-byte aligned

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int num_batches = (args.m + B - 1) / B;
    const uint32_t slices_per_batch = static_cast<uint32_t>(B) * slices_per_row;

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
    uint32_t issued = 0;  // loads issued by thread 0
    if (tid == 0) {
        prefetch_tmap(&tmap_x);
        if (blockIdx.x < num_batches) {
            issue_load(blockIdx.x);
            issued = 1;
        }
    }

    const int pair = tid >> 1;
    const int h = tid & 1;
    const bool given = args.given_scales != nullptr;  // uniform: a kernel argument
    const ActLut lut{args.silu_lut, args.gelu_lut};
    bool alive = true;

    for (int it = 0;; ++it) {
        const int batch = blockIdx.x + it * gridDim.x;
        if (batch >= num_batches) break;
        const int par = it & 1;
        const int row0 = batch * B;
        const int rows = min(B, args.m - row0);
        const int tasks = rows * groups;
        const bool warp_busy = warp * 16 < tasks;  // warp-uniform
        const bool active = pair < tasks;
        const int task = active ? pair : 0;
        const int r = task / groups;
        const int grp = task - r * groups;

        if (alive) alive = mbar_wait(full, static_cast<uint32_t>(it & 1), nullptr, args.err, kErrTimeoutFull);
        f32x2 v[64];
        if (warp_busy && alive)
            load_group<Act>(inbuf, r * slices_per_row + grp * 4 + h, static_cast<uint32_t>(K / 64), v, lut);
        __syncthreads();  // the batch is in registers: the buffer may be refilled
        if (tid == 0 && alive) {
            const int next = batch + gridDim.x;
            if (next < num_batches) {
                issue_load(next);
                ++issued;
            }
        }
        // The slot the next batch uses was last read before this batch's first barrier.
        for (int i = tid; i < B; i += blockDim.x) {
            row_absmax[(par ^ 1) * B + i] = 0u;
            row_nan[(par ^ 1) * B + i] = 0u;
        }

        uint32_t wa[32], wb[32];
        bool group_nan = false;
        if (warp_busy && alive) {
            float amax, probe;
            rotate_to_words(v, h, wa, wb, amax, probe);
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            probe = __fadd_rn(probe, __shfl_xor_sync(0xffffffffu, probe, 1));
            if (active && h == 0 && !given) {
                atomicMax(&row_absmax[par * B + r], __float_as_uint(amax));
                if (isnan(probe)) atomicOr(&row_nan[par * B + r], 1u);
            }
            group_nan = isnan(probe);
        }
        if (!given) __syncthreads();  // every group of every row has reported its absmax

        if (active && alive) {
            const float amax = given ? 0.0f : __uint_as_float(row_absmax[par * B + r]);
            const float scale = given ? args.given_scales[row0 + r] : row_scale<Bits>(amax, args.scale_mul != 0);
            if (grp == 0 && h == 0 && !given) args.scales[row0 + r] = scale;
            int8_t *out = args.codes + static_cast<int64_t>(row0 + r) * Kout;
            if constexpr (Bits == 4) {
                const float inv = __fdiv_rn(1.0f, scale);
                out += grp * 128 + h * 32;
                store_run_int4(out, wa, inv);
                store_run_int4(out + 64, wb, inv);
            } else {
                const float rs = __bfloat162float(__float2bfloat16_rn(scale));
                // Given scales: this group's own NaN probe decides (the exact chain is
                // correct for any row), plus any scale outside the fast chain's range.
                const bool exact = given ? (group_nan || !fast_chain_scale_ok(rs))
                                         : (row_nan[par * B + r] != 0u || isinf(amax));
                const float qparam = exact ? rs : __frcp_rn(rs);
                out += grp * 256 + h * 64;
                store_run_int8(out, wa, exact, qparam);
                store_run_int8(out + 128, wb, exact, qparam);
            }
        }
    }
    if (tid == 0 && !alive && issued > 0) {
        // A wait gave up: let the last copy land before the CTA exits.  Every copy but
        // the last was waited for, so the barrier is in the last copy's phase.
        mbar_wait(full, (issued - 1) & 1u, nullptr, args.err, kErrTimeoutDrain);
    }
}

template __global__ void convrot_quant_reg_kernel<kActNone, 8>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_reg_kernel<kActNone, 4>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_reg_kernel<kActSwiGLU, 8>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_reg_kernel<kActSwiGLU, 4>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_reg_kernel<kActGelu, 8>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_reg_kernel<kActGelu, 4>(const __grid_constant__ CUtensorMap, const QuantArgs);

}  // namespace rot
}  // namespace ctu
