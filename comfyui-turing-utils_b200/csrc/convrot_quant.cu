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
#include <cuda_runtime.h>

#include <cstdint>

#include "convrot_quant.cuh"
#include "ptx.cuh"

namespace ctu {
namespace rot {

constexpr float kBf16Max = 3.38953139e38f;

// ---------------------------------------------------------------------------
// Radix-4 butterfly on two independent 4-tuples at once (packed f32x2), with the
// reference's association: y0 = ((x0+x1)+x2)-x3, y1 = ((x0+x1)-x2)+x3,
// y2 = ((x0-x1)+x2)+x3, y3 = ((-x0+x1)+x2)+x3, each times 0.5.
__device__ __forceinline__ void butterfly2(float2 &x0, float2 &x1, float2 &x2, float2 &x3) {
    const float2 half = make_float2(0.5f, 0.5f);
    const float2 t = add2(x0, x1);
    const float2 b = sub2(x0, x1);   // x0 - x1;  (-x0 + x1) == -(x0 - x1) exactly
    const float2 y0 = mul2(half, sub2(add2(t, x2), x3));
    const float2 y1 = mul2(half, add2(sub2(t, x2), x3));
    const float2 y2 = mul2(half, add2(add2(b, x2), x3));
    const float2 y3 = mul2(half, add2(sub2(x2, b), x3));  // (-b) + x2 == x2 - b exactly
    x0 = y0;
    x1 = y1;
    x2 = y2;
    x3 = y3;
}

// Physical shared-memory byte offset of 16-byte chunk `c` of 128-byte slice `r`
// as written by a TMA load with CU_TENSOR_MAP_SWIZZLE_128B.
__device__ __forceinline__ uint32_t sw128(uint32_t r, uint32_t c) { return r * 128u + ((c ^ (r & 7u)) << 4); }

template <int Act>
__device__ __forceinline__ float activate(uint32_t gate_bits, uint32_t up_bits);

template <>
__device__ __forceinline__ float activate<kActNone>(uint32_t x, uint32_t) {
    return __uint_as_float(x);
}

// convrot_quant.cu:163-169
template <>
__device__ __forceinline__ float activate<kActSwiGLU>(uint32_t gate_bits, uint32_t up_bits) {
    const float gate = __uint_as_float(gate_bits);
    const float up = __uint_as_float(up_bits);
    return (gate / (1.0f + expf(-gate))) * up;
}

// convrot_quant.cu:171-182 (tanh-GELU, result rounded back to bf16)
template <>
__device__ __forceinline__ float activate<kActGelu>(uint32_t x_bits, uint32_t) {
    const float x = __uint_as_float(x_bits);
    constexpr float kAlpha = 0.7978845608028654f;
    constexpr float kBeta = 0.044715f;
    const float activated = 0.5f * x * (1.0f + tanhf(kAlpha * (x + kBeta * x * x * x)));
    return __bfloat162float(__float2bfloat16_rn(activated));
}

// Load one lane's 128 inputs of a group: chunk0 = elements h*64+[0,64) (bit 7 = 0),
// chunk1 = 128+h*64+[0,64).  `row64` is the 128-byte slice index of chunk0 inside the
// batch buffer; chunk1 sits two slices later.  For SwiGLU the `up` half of the row
// starts `up_off` slices after the gate.
template <int Act>
__device__ __forceinline__ void load_group(const uint8_t *buf, uint32_t row64, uint32_t up_off, float2 (&v)[64]) {
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
                v[8 * c + 2 * q] = make_float2(activate<Act>(aw[q] << 16, uaw[q] << 16),
                                               activate<Act>(bw[q] << 16, ubw[q] << 16));
                v[8 * c + 2 * q + 1] = make_float2(activate<Act>(aw[q] & 0xFFFF0000u, uaw[q] & 0xFFFF0000u),
                                                   activate<Act>(bw[q] & 0xFFFF0000u, ubw[q] & 0xFFFF0000u));
            }
        } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                v[8 * c + 2 * q] = make_float2(activate<Act>(aw[q] << 16, 0), activate<Act>(bw[q] << 16, 0));
                v[8 * c + 2 * q + 1] =
                    make_float2(activate<Act>(aw[q] & 0xFFFF0000u, 0), activate<Act>(bw[q] & 0xFFFF0000u, 0));
            }
        }
    }
}

// Rotate the group held by this lane pair, return this lane's absmax (NaN ignored)
// and a NaN probe, and write bf16(y) back in place.  All 32 lanes of the warp must
// call this together (it shuffles with a full mask); a lane pair without work passes
// active = false, computes on a valid group and writes nothing.
template <int Act>
__device__ __forceinline__ void rotate_group(uint8_t *buf, uint32_t row64, uint32_t up_off, int h, bool active,
                                             float &absmax, float &nan_probe) {
    float2 v[64];
    load_group<Act>(buf, row64, up_off, v);

    // Stage 1 (stride 1): bits 0-1 of the element index.
#pragma unroll
    for (int q = 0; q < 16; ++q) butterfly2(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    // Stage 2 (stride 4): bits 2-3.
#pragma unroll
    for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int p = 0; p < 4; ++p) butterfly2(v[16 * c + p], v[16 * c + p + 4], v[16 * c + p + 8], v[16 * c + p + 12]);
    }
    // Stage 3 (stride 16): bits 4-5.
#pragma unroll
    for (int p = 0; p < 16; ++p) butterfly2(v[p], v[p + 16], v[p + 32], v[p + 48]);

    // Stage 4 (stride 64): bit 6 is the lane parity h, bit 7 is the pair index
    // inside v[j] (.x: bit 7 = 0, .y: bit 7 = 1).  The four inputs of position j
    // are x0 = lane0.x, x1 = lane1.x, x2 = lane0.y, x3 = lane1.y.  Lane h produces
    // y_h into .x and y_{2+h} into .y:
    //   lane 0: y0 = ((x0+x1)+x2)-x3          y2 = ((x0-x1)+x2)+x3
    //   lane 1: y1 = -((-(x0+x1)+x2)-x3)      y3 = ((x1-x0)+x2)+x3
    // which is the reference's y1 = ((x0+x1)-x2)+x3 with every rounding mirrored.
    const unsigned full = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    const int lane0 = lane & ~1;
    const float sgn = h ? -1.0f : 1.0f;
    const float hsgn = h ? -0.5f : 0.5f;
    float m = 0.0f;
    float probe = 0.0f;
#pragma unroll
    for (int j = 0; j < 64; ++j) {
        const float own = v[j].x;
        const float other = __shfl_xor_sync(full, own, 1);
        const float x2 = __shfl_sync(full, v[j].y, lane0);
        const float x3 = __shfl_sync(full, v[j].y, lane0 + 1);
        const float p = __fadd_rn(own, other);   // x0 + x1 in both lanes
        const float d = __fsub_rn(own, other);   // x0 - x1 (lane 0) or x1 - x0 (lane 1)
        const float ya = __fmul_rn(hsgn, __fsub_rn(__fmaf_rn(sgn, p, x2), x3));
        const float yb = __fmul_rn(0.5f, __fadd_rn(__fadd_rn(d, x2), x3));
        v[j] = make_float2(ya, yb);
        m = fmaxf(m, fmaxf(fabsf(ya), fabsf(yb)));
        probe = __fadd_rn(probe, __fadd_rn(ya, yb));
    }
    absmax = active ? m : 0.0f;
    nan_probe = active ? probe : 0.0f;
    if (!active) return;

    // bf16(y) back in place (this lane's own element positions).
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        uint4 a, b;
        a.x = pack_bf16x2(v[8 * c + 0].x, v[8 * c + 1].x);
        a.y = pack_bf16x2(v[8 * c + 2].x, v[8 * c + 3].x);
        a.z = pack_bf16x2(v[8 * c + 4].x, v[8 * c + 5].x);
        a.w = pack_bf16x2(v[8 * c + 6].x, v[8 * c + 7].x);
        b.x = pack_bf16x2(v[8 * c + 0].y, v[8 * c + 1].y);
        b.y = pack_bf16x2(v[8 * c + 2].y, v[8 * c + 3].y);
        b.z = pack_bf16x2(v[8 * c + 4].y, v[8 * c + 5].y);
        b.w = pack_bf16x2(v[8 * c + 6].y, v[8 * c + 7].y);
        *reinterpret_cast<uint4 *>(buf + sw128(row64, c)) = a;
        *reinterpret_cast<uint4 *>(buf + sw128(row64 + 2, c)) = b;
    }
}

// Quantize 8 consecutive bf16(y) values of one row to int8 with the fast chain.
__device__ __forceinline__ uint2 quant8_int8_fast(uint4 w, float rcp) {
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    uint32_t q[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 pr = mul2(make_float2(bf16lo(ww[i]), bf16hi(ww[i])), make_float2(rcp, rcp));
        q[i] = pack_bf16x2(pr.x, pr.y);  // bf16(y / bf16(scale))
    }
    int c[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        c[2 * i] = __float2int_rn(bf16lo(q[i]));
        c[2 * i + 1] = __float2int_rn(bf16hi(q[i]));
    }
    // cvt.pack.sat.s8.s32.b32 d, a, b, c: d = {sat8(b), sat8(a), c[0:16)} from the low byte up.
    uint32_t t0, t1, lo, hi;
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(t0) : "r"(c[3]), "r"(c[2]), "r"(0u));
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(lo) : "r"(c[1]), "r"(c[0]), "r"(t0));
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(t1) : "r"(c[7]), "r"(c[6]), "r"(0u));
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(hi) : "r"(c[5]), "r"(c[4]), "r"(t1));
    return make_uint2(lo, hi);
}

// Exact reference chain including NaN (fmaxf(-128, NaN) == -128) for rows that
// contain NaN or infinities.
__device__ __forceinline__ uint2 quant8_int8_exact(uint4 w, float rounded_scale) {
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
__device__ __forceinline__ uint32_t quant8_int4(uint4 w, float inv_scale) {
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    uint32_t out = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 pr = mul2(make_float2(bf16lo(ww[i]), bf16hi(ww[i])), make_float2(inv_scale, inv_scale));
        const float lo = fminf(7.0f, fmaxf(-7.0f, pr.x));
        const float hi = fminf(7.0f, fmaxf(-7.0f, pr.y));
        const uint32_t lb = static_cast<uint32_t>(__float2int_rn(lo)) & 0xFu;
        const uint32_t hb = static_cast<uint32_t>(__float2int_rn(hi)) & 0xFu;
        out |= (lb | (hb << 4)) << (8 * i);
    }
    return out;
}

template <int Act, int Bits>
__global__ void __launch_bounds__(kMaxThreads, 1)
    convrot_quant_kernel(const __grid_constant__ CUtensorMap tmap_x, const QuantArgs args) {
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
            rotate_group<Act>(inbuf[buf], row64, static_cast<uint32_t>(K / 64), h, active, amax, probe);
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
        for (int r = tid; r < rows; r += nthreads) {
            const float amax = __uint_as_float(absmax_rows[r]);
            const float qmax = Bits == 4 ? 7.0f : 127.0f;
            const float floor = Bits == 4 ? 1.0e-10f : 1.0e-30f;
            args.scales[row0 + r] = fmaxf(__fdiv_rn(fminf(amax, kBf16Max), qmax), floor);
        }

        // -------------------------------------------------------------- quantize
        const int chunks_per_row = K / 8;
        const int total_chunks = rows * chunks_per_row;
        int cur_row = -1;
        float qparam = 0.0f;
        bool exact = false;
        for (int ch = tid; ch < total_chunks; ch += nthreads) {
            const int r = ch / chunks_per_row;
            const int col8 = ch - r * chunks_per_row;
            if (r != cur_row) {
                cur_row = r;
                const float amax = __uint_as_float(absmax_rows[r]);
                const float qmax = Bits == 4 ? 7.0f : 127.0f;
                const float floor = Bits == 4 ? 1.0e-10f : 1.0e-30f;
                const float scale = fmaxf(__fdiv_rn(fminf(amax, kBf16Max), qmax), floor);
                if (Bits == 4) {
                    qparam = __fdiv_rn(1.0f, scale);
                } else {
                    const float rs = __bfloat162float(__float2bfloat16_rn(scale));
                    exact = nan_rows[r] != 0u || isinf(amax);
                    qparam = exact ? rs : __frcp_rn(rs);
                }
            }
            // bf16(y) chunk: slice = r*slices_per_row + col8/8, 16-byte chunk col8 % 8.
            const uint4 w = *reinterpret_cast<const uint4 *>(
                inbuf[buf] + sw128(r * slices_per_row + (col8 >> 3), col8 & 7));
            if (Bits == 4) {
                *reinterpret_cast<uint32_t *>(codebuf + r * Kout + col8 * 4) = quant8_int4(w, qparam);
            } else {
                const uint2 q = exact ? quant8_int8_exact(w, qparam) : quant8_int8_fast(w, qparam);
                *reinterpret_cast<uint2 *>(codebuf + r * Kout + col8 * 8) = q;
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

template __global__ void convrot_quant_kernel<kActNone, 8>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_kernel<kActNone, 4>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_kernel<kActSwiGLU, 8>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_kernel<kActSwiGLU, 4>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_kernel<kActGelu, 8>(const __grid_constant__ CUtensorMap, const QuantArgs);
template __global__ void convrot_quant_kernel<kActGelu, 4>(const __grid_constant__ CUtensorMap, const QuantArgs);

}  // namespace rot
}  // namespace ctu
