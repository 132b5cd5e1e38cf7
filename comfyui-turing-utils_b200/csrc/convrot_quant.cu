// Fused ConvRot rotate + per-token quantize (int8 or packed int4), HBM-bound.
//
// Computes, for every row of a bf16 activation [M, K] (or a SwiGLU [M, 2K] /
// tanh-GELU [M, K] input), exactly the reference's row-buffer quantizer
// (kernel/csrc/turing/convrot_quant.cu:417-511):
//   * the 4-stage radix-4 rotation of each 256-column group, stage strides 1, 4,
//     16, 64, each output 0.5f*(x0 (+|-) x1 (+|-) x2 (+|-) x3) evaluated left to
//     right in fp32 (convrot_quant.cu:104-116);
//   * absmax over the unrounded fp32 rotated values, scale =
//     max(min(absmax, BF16_MAX) / qmax, floor);
//   * int8: code = clamp(rint(bf16(bf16(y) / bf16(scale))), -128, 127);
//     int4: code = clamp(rint(bf16(y) * (1 / scale)), -7, 7), low nibble first.
//
// B200 design:
//   * A persistent grid walks batches of B rows.  Each batch is brought into
//     shared memory by TMA (2D tensor map over 64-column slices, 128-byte swizzle),
//     double-buffered so the next batch streams in while this one computes.
//   * Each 256-group is owned by a lane pair.  Lane h of the pair holds the 128
//     elements whose bit 6 equals h, as 64 float2 pairs (element e, e + 128), so
//     stages 1-3 run in registers as packed f32x2 (FADD2/FMUL2) operations and only
//     stage 4 exchanges values between the two lanes (three shuffles per pair of
//     outputs).  The fp32 evaluation order of every output is the reference's.
//   * bf16(y) is written back over the consumed input in shared memory; a second
//     pass turns it into codes with the row scale, and the codes of the whole batch
//     leave through one bulk (TMA) store.
//   * The int8 quotient bf16(y)/bf16(scale) is formed as bf16(y) * rcp(bf16(scale))
//     and rounded to bf16.  Both operands carry 8 significant bits, so the exact
//     quotient is never a bf16 rounding midpoint and lies at least 2^-17 (relative)
//     away from every midpoint, while the product is within 2^-23 of it: the bf16
//     rounding of the product equals the bf16 rounding of the IEEE quotient
//     (exhaustively re-checked in tests/test_quotient_identity.py).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "convrot_math.cuh"
#include "convrot_quant.cuh"
#include "ptx.cuh"

namespace ctu {
namespace rot {

// Rotate the group held by this lane pair, return this lane's absmax (NaN ignored)
// and a NaN probe, and write bf16(y) back in place.  All 32 lanes of the warp must
// call this together (it shuffles with a full mask); a lane pair without work passes
// active = false, computes on a valid group and writes nothing.
template <int Act, bool kHalf>
__device__ __forceinline__ void rotate_group(uint8_t *buf, uint32_t row64, uint32_t up_off, int h, bool active,
                                             float &absmax, float &nan_probe, const ActLut &lut) {
    f32x2 v[64];
    if constexpr (kHalf) {
        load_group_f16<Act>(buf, row64, up_off, v, lut);
    } else {
        load_group<Act>(buf, row64, up_off, v, lut);
    }
    const f32x2 half = pk2(0.5f, 0.5f);

    // Stage 1 (stride 1): bits 0-1 of the element index.
#pragma unroll
    for (int q = 0; q < 16; ++q) butterfly2(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3], half);
    // Stage 2 (stride 4): bits 2-3.
#pragma unroll
    for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int p = 0; p < 4; ++p)
            butterfly2(v[16 * c + p], v[16 * c + p + 4], v[16 * c + p + 8], v[16 * c + p + 12], half);
    }
    // Stage 3 (stride 16): bits 4-5.
#pragma unroll
    for (int p = 0; p < 16; ++p) butterfly2(v[p], v[p + 16], v[p + 32], v[p + 48], half);

    // Stage 4 (stride 64): bit 6 is the lane parity h, bit 7 the half of v[j]
    // (low: bit 7 = 0, high: bit 7 = 1).  The four inputs at position j are
    // x0 = lane0.lo, x1 = lane1.lo, x2 = lane0.hi, x3 = lane1.hi.  Lane h produces
    // y_h (bit 7 = 0) and y_{2+h} (bit 7 = 1):
    //   lane 0: y0 = ((x0+x1)+x2)-x3          y2 = ((x0-x1)+x2)+x3
    //   lane 1: y1 = -((-(x0+x1)+x2)-x3)      y3 = ((x1-x0)+x2)+x3
    // which is the reference's y1 = ((x0+x1)-x2)+x3 with every rounding mirrored
    // (IEEE rounding is symmetric in sign).  Two positions j, j+1 share each packed
    // operation, and their outputs form the bf16x2 words stored back.
    const unsigned full = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    const int lane0 = lane & ~1;
    const f32x2 sgn = h ? pk2(-1.0f, -1.0f) : pk2(1.0f, 1.0f);
    const f32x2 hsgn = h ? pk2(-0.5f, -0.5f) : pk2(0.5f, 0.5f);
    float m = 0.0f;
    f32x2 probe = pk2(0.0f, 0.0f);
    uint32_t wa[4], wb[4];
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
        const f32x2 p = fadd2(own, other);  // x0 + x1 in both lanes
        const f32x2 d = fsub2(own, other);  // x0 - x1 (lane 0) or x1 - x0 (lane 1)
        const f32x2 ya = fmul2(hsgn, fsub2(ffma2(sgn, p, x2), x3));
        const f32x2 yb = fmul2(half, fadd2(fadd2(d, x2), x3));
        probe = fadd2(probe, fadd2(ya, yb));
        float ya0, ya1, yb0, yb1;
        unpk2(ya, ya0, ya1);
        unpk2(yb, yb0, yb1);
        m = max_abs3(m, ya0, ya1);
        m = max_abs3(m, yb0, yb1);
        wa[(j >> 1) & 3] = kHalf ? pack_f16x2(ya0, ya1) : pack_bf16x2(ya0, ya1);
        wb[(j >> 1) & 3] = kHalf ? pack_f16x2(yb0, yb1) : pack_bf16x2(yb0, yb1);
        if ((j & 7) == 6 && active) {
            // bf16(y) of 8 positions back in place over this lane's own (already
            // consumed) input elements.
            const int c = j >> 3;
            *reinterpret_cast<uint4 *>(buf + sw128(row64, c)) = make_uint4(wa[0], wa[1], wa[2], wa[3]);
            *reinterpret_cast<uint4 *>(buf + sw128(row64 + 2, c)) = make_uint4(wb[0], wb[1], wb[2], wb[3]);
        }
    }
    float p0, p1;
    unpk2(probe, p0, p1);
    absmax = active ? m : 0.0f;
    nan_probe = active ? __fadd_rn(p0, p1) : 0.0f;
}

template <int Act, int Bits, bool kHalf>
__global__ void __launch_bounds__(kMaxThreads, 1)
    convrot_quant_kernel(const __grid_constant__ CUtensorMap tmap_x, const QuantArgs args) {
    constexpr float kFiniteMax = kHalf ? 65504.0f : kBf16Max;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int K = args.k;
    const int B = args.rows_per_batch;
    const int Kin = Act == kActSwiGLU ? 2 * K : K;
    const int Kout = Bits == 4 ? K / 2 : K;
    const int groups = K / 256;
    const uint32_t in_bytes = static_cast<uint32_t>(args.box_rows) * args.copies * 128u;  // multiple of 1024
    const uint32_t slices_per_row = Kin / 64;
    uint8_t *inbuf[2] = {smem, smem + in_bytes};
    uint8_t *codebuf = smem + 2 * in_bytes;
    uint32_t *row_absmax = reinterpret_cast<uint32_t *>(codebuf + ((B * Kout + 15) & ~15));  // [2][B]
    uint32_t *row_nan = row_absmax + 2 * B;                                                // [2][B]
    uint64_t *full = reinterpret_cast<uint64_t *>((reinterpret_cast<uintptr_t>(row_nan + 2 * B) + 7) & ~uintptr_t(7));

    const int tid = threadIdx.x;
    const int nthreads = blockDim.x;
    const int num_batches = (args.m + B - 1) / B;
    const uint32_t slices_per_batch = static_cast<uint32_t>(B) * slices_per_row;

    // A batch is slices [batch * slices_per_batch, +slices_per_batch) of the input
    // viewed as 128-byte slices; the last copy may run past the batch (into the next
    // rows or the zero-filled out-of-bounds region) and those bytes are ignored.
    auto issue_load = [&](int batch, int buf) {
        mbar_arrive_expect_tx(&full[buf], in_bytes);
        for (int c = 0; c < args.copies; ++c) {
            const uint32_t s0 = static_cast<uint32_t>(c * args.box_rows);
            tma_load_2d(inbuf[buf] + s0 * 128u, &tmap_x, 0, static_cast<int>(batch * slices_per_batch + s0), &full[buf]);
        }
    };

    if (tid == 0) {
        mbar_init(&full[0], 1);
        mbar_init(&full[1], 1);
        fence_mbar_init();
    }
    for (int i = tid; i < 4 * B; i += nthreads) row_absmax[i] = 0u;  // also clears row_nan
    __syncthreads();
    if (tid == 0) {
        prefetch_tmap(&tmap_x);
        if (blockIdx.x < num_batches) issue_load(blockIdx.x, 0);
        if (blockIdx.x + gridDim.x < num_batches) issue_load(blockIdx.x + gridDim.x, 1);
    }

    const int pair = tid >> 1;
    const int h = tid & 1;
    const int npairs = nthreads >> 1;
    bool alive = true;

    for (int it = 0;; ++it) {
        const int batch = blockIdx.x + it * gridDim.x;
        if (batch >= num_batches) break;
        const int buf = it & 1;
        const int par = it & 1;  // row-statistics parity
        const uint32_t phase = (it >> 1) & 1;
        const int row0 = batch * B;
        const int rows = min(B, args.m - row0);
        if (alive) alive = mbar_wait(&full[buf], phase, nullptr, args.err, kErrTimeoutFull);
        if (tid == 0) bulk_wait_read_all();  // the previous batch's code store has read codebuf

        // -------------------------------------------------------------- rotation
        uint32_t *absmax_rows = row_absmax + par * B;
        uint32_t *nan_rows = row_nan + par * B;
        // Warp-uniform trip count: every lane runs every iteration (full-mask shuffles).
        const int total = rows * groups;
        const int trips = (total + npairs - 1) / npairs;
        for (int trip = 0; trip < trips; ++trip) {
            const int task_raw = trip * npairs + pair;
            const bool active = task_raw < total;
            const int task = active ? task_raw : 0;
            const int r = task / groups;
            const int grp = task - r * groups;
            const uint32_t row64 = r * slices_per_row + grp * 4 + h;
            float amax, probe;
            rotate_group<Act, kHalf>(inbuf[buf], row64, static_cast<uint32_t>(K / 64), h, active, amax, probe,
                                     ActLut{args.silu_lut, args.gelu_lut, args.silu16_lut, args.gelu16_lut});
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            probe = __fadd_rn(probe, __shfl_xor_sync(0xffffffffu, probe, 1));
            if (active && h == 0) {
                atomicMax(&absmax_rows[r], __float_as_uint(amax));
                if (isnan(probe)) atomicOr(&nan_rows[r], 1u);
            }
        }
        __syncthreads();
        // Clear the statistics slot the next batch will use.
        for (int i = tid; i < B; i += nthreads) {
            row_absmax[(par ^ 1) * B + i] = 0u;
            row_nan[(par ^ 1) * B + i] = 0u;
        }

        // -------------------------------------------------------------- per-row scales
        const bool given = args.given_scales != nullptr;
        for (int r = tid; r < rows && !given; r += nthreads) {
            const float amax = __uint_as_float(absmax_rows[r]);
            args.scales[row0 + r] = row_scale<Bits>(amax, args.scale_mul != 0, kFiniteMax);
        }

        // -------------------------------------------------------------- quantize
        const int chunks_per_row = K / 8;
        int r = tid / chunks_per_row;
        int col8 = tid - r * chunks_per_row;
        int cur_row = -1;
        float qparam = 0.0f;
        bool exact = false;
        while (r < rows) {
            if (r != cur_row) {
                cur_row = r;
                const float amax = __uint_as_float(absmax_rows[r]);
                const float scale =
                    given ? args.given_scales[row0 + r] : row_scale<Bits>(amax, args.scale_mul != 0, kFiniteMax);
                if (Bits == 4) {
                    qparam = __fdiv_rn(1.0f, scale);
                } else if (kHalf) {
                    qparam = __half2float(__float2half_rn(scale));
                } else {
                    const float rs = __bfloat162float(__float2bfloat16_rn(scale));
                    exact = nan_rows[r] != 0u || (given ? !fast_chain_scale_ok(rs) : isinf(amax));
                    qparam = exact ? rs : __frcp_rn(rs);
                }
            }
            const uint4 w = *reinterpret_cast<const uint4 *>(inbuf[buf] + sw128(r * slices_per_row + (col8 >> 3), col8 & 7));
            if (Bits == 4) {
                *reinterpret_cast<uint32_t *>(codebuf + r * Kout + col8 * 4) =
                    kHalf ? quant8_int4_f16(w, qparam) : quant8_int4(w, pk2(qparam, qparam));
            } else {
                const uint2 q = kHalf   ? quant8_int8_f16(w, qparam)
                                : exact ? quant8_int8_exact(w, qparam)
                                        : quant8_int8_fast(w, pk2(qparam, qparam));
                *reinterpret_cast<uint2 *>(codebuf + r * Kout + col8 * 8) = q;
            }
            col8 += nthreads;
            while (col8 >= chunks_per_row) {
                col8 -= chunks_per_row;
                ++r;
            }
        }
        fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
            bulk_store(args.codes + static_cast<int64_t>(row0) * Kout, codebuf, static_cast<uint32_t>(rows * Kout));
            bulk_commit();
            const int next = batch + 2 * gridDim.x;
            if (next < num_batches) issue_load(next, buf);
        }
    }
    if (tid == 0) bulk_wait_all();
}

// One thread per bf16 bit pattern: the SwiGLU gate factor and the rounded tanh-GELU
// of every bf16 value, exactly as the activations define them (silu_factor, gelu_bf16).
__global__ void act_lut_fill_kernel(float *silu, uint16_t *gelu, float *silu16, uint16_t *gelu16) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= 65536u) return;
    const float x = __uint_as_float(i << 16);
    silu[i] = silu_factor(x);
    gelu[i] = static_cast<uint16_t>(__float_as_uint(gelu_bf16(x)) >> 16);
    const float xh = f16_to_f32(i);
    silu16[i] = silu_factor(xh);
    gelu16[i] = __half_as_ushort(__float2half_rn(gelu_fp32(xh)));
}

template __global__ void convrot_quant_kernel<kActNone, 8>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_kernel<kActNone, 4>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_kernel<kActSwiGLU, 8>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_kernel<kActSwiGLU, 4>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_kernel<kActGelu, 8>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_kernel<kActGelu, 4>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_kernel<kActSwiGLU, 8, true>(const __grid_constant__ CUtensorMap,
                                                                    const QuantArgs);
template __global__ void convrot_quant_kernel<kActSwiGLU, 4, true>(const __grid_constant__ CUtensorMap,
                                                                    const QuantArgs);
template __global__ void convrot_quant_kernel<kActGelu, 8, true>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_kernel<kActGelu, 4, true>(const __grid_constant__ CUtensorMap, const QuantArgs);

}  // namespace rot
}  // namespace ctu
