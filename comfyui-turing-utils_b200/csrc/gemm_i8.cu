// Integer GEMMs on the 5th-generation tensor cores (tcgen05, kind::i8) with the
// ConvRot dequant + bias epilogue fused:
//
//   out[m, n] = bf16( fma(float(acc[m, n]) * a_scale[m], w_scale[n], bias[n]) )
//   acc[m, n] = sum_k a[m, k] * w[n, k]          (exact int32)
//
// W8A8 (kModeW8A8) replaces the reference's CUTLASS SM75 mma.sync GEMM
// (kernel/csrc/turing/w4a8.cu:376-618, entry w4a8.cu:1185-1219); W4A8 (kModeW4A8)
// replaces its signed packed-int4 variant (w4a8.cu:34-72, 1000-1086): weights hold
// two signed 4-bit values per byte, the even k in the low nibble.  W4A4 (kModeW4A4)
// packs the activations the same way (the int4 ConvRot codes).  All keep the
// reference's epilogue order (w4a8.cu:474-525: activation scale, weight scale, bias,
// round to bf16).
//
// Design (one CTA per SM, persistent over 128 x 256 output tiles):
//   warp 0      TMA producer: A [128 x 128 B] (128-byte swizzle) and the weight tile
//               (W8: [256 x 128 B] swizzled; W4: packed [256 x 64 B]) into a
//               kStages-deep shared-memory ring (mbarrier per stage)
//   warp 1      MMA issuer: owns the TMEM allocation (512 columns = two 128x256 int32
//               accumulators), issues tcgen05.mma M=128 N=256 K=32, frees ring stages
//               with tcgen05.commit
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time, fused scale/bias/bf16,
//               16-byte global stores; releases the accumulator buffer so the next
//               tile's MMAs overlap this tile's epilogue
//   warps 6..9  (int4 modes) converters: sign-extend each packed tile into a
//               double-buffered int8 tile in the same 128-byte-swizzled layout the
//               MMA reads, then fence the generic writes for the async proxy
// Tiles are visited n-fastest so the CTAs resident at one time share the same A
// rows and the whole weight matrix stays L2-resident.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "gemm_i8.cuh"
#include "gemm_tile.cuh"
#include "ptx.cuh"

namespace ctu {
namespace gemm {

struct Smem {
    uint64_t full[kStages];
    uint64_t empty[kStages];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint64_t bu_full[2];   // W4: converted weight tile ready
    uint64_t bu_empty[2];  // W4: converted weight tile consumed by the MMA
    uint64_t drain;
    uint32_t tmem_base;
    int abort_flag;
    int conv_ok;
    float col_scale[kBN];
    float col_bias[kBN];
};

template <int kMode>
struct Layout {
    static constexpr bool kAPacked = kMode == kModeW4A4;
    static constexpr bool kBPacked = kMode != kModeW8A8;
    static constexpr bool kConvert = kAPacked || kBPacked;
    static constexpr int kAStageBytes = kAPacked ? kAPackedBytes : kABytes;  // activation bytes per ring stage
    static constexpr int kBStageBytes = kBPacked ? kBPackedBytes : kBBytes;  // weight bytes per ring stage
    static constexpr int kRingBytes = kStages * (kAStageBytes + kBStageBytes);
    // Converted (int8, 128-byte swizzled) tiles, double-buffered: A first, then B.
    static constexpr int kConvABytes = kAPacked ? 2 * kABytes : 0;
    static constexpr int kConvBBytes = kBPacked ? 2 * kBBytes : 0;
    static constexpr int kSmemStructOffset = kRingBytes + kConvABytes + kConvBBytes;
};

template <int kMode>
__global__ void __launch_bounds__(kMode == kModeW8A8 ? kThreads : kThreadsW4, 1)
    int8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                     const GemmArgs args) {
    using L = Layout<kMode>;
    constexpr bool kConvert = L::kConvert;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;                                     // ring activation tiles (packed for W4A4)
    uint8_t *sB = smem + kStages * L::kAStageBytes;         // ring weight tiles (packed for W4A8/W4A4)
    uint8_t *sAu = smem + L::kRingBytes;                    // converted activation tiles
    uint8_t *sBu = sAu + L::kConvABytes;                    // converted weight tiles
    Smem &S = *reinterpret_cast<Smem *>(smem + L::kSmemStructOffset);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_n = (args.n + kBN - 1) / kBN;
    const int num_m = (args.m + kBM - 1) / kBM;
    const int num_tiles = num_m * num_n;
    const int nk = (args.k + kBK - 1) / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&S.full[s], 1);
            // With converters a stage is free once both the MMA and the converters are done.
            mbar_init(&S.empty[s], kConvert ? 2 : 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&S.acc_full[b], 1);
            mbar_init(&S.acc_empty[b], kEpilogueWarps);
            mbar_init(&S.bu_full[b], 1);
            mbar_init(&S.bu_empty[b], 1);
        }
        mbar_init(&S.drain, 1);
        S.abort_flag = 0;
        S.conv_ok = 1;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(&S.tmem_base, kTmemCols);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_b);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = S.tmem_base;
    volatile int *abort_flag = &S.abort_flag;

    if (warp == 0) {
        // ------------------------------------------------------------------ producer
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            uint32_t fills = 0;  // total stage fills issued by this thread
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                const int m0 = (t / num_n) * kBM;
                const int n0 = (t % num_n) * kBN;
                for (int kb = 0; kb < nk; ++kb) {
                    if (!mbar_wait(&S.empty[s], ph ^ 1u, abort_flag, args.err, kErrTimeoutEmpty)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&S.full[s], L::kAStageBytes + L::kBStageBytes);
                    tma_load_2d(sA + s * L::kAStageBytes, &tmap_a, kb * (L::kAPacked ? kBK / 2 : kBK), m0, &S.full[s]);
                    tma_load_2d(sB + s * L::kBStageBytes, &tmap_b, kb * (L::kBPacked ? kBK / 2 : kBK), n0, &S.full[s]);
                    ++fills;
                    if (++s == kStages) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
            }
            if (!ok || *abort_flag) {
                // Another role gave up: let every tile still in flight land before the
                // CTA can exit (the normal path consumes them all).
                for (uint32_t i = 0; i < kStages && i < fills; ++i) {
                    const uint32_t fill = fills - 1 - i;
                    mbar_wait(&S.full[fill % kStages], (fill / kStages) & 1u, nullptr, args.err, kErrTimeoutDrain);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8(kBM, kBN);
            int s = 0;
            uint32_t ph = 0;
            uint32_t conv = 0;  // converted tiles consumed so far
            int local = 0;
            bool ok = true;
            if (args.inject_timeout) {
                // Test hook: wait on a barrier nothing arrives on; the bounded wait
                // must time out, record kErrInjected and stop the kernel cleanly.
                mbar_wait(&S.drain, 0u, abort_flag, args.err, kErrInjected, args.inject_timeout_ns);
                ok = false;
            }
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++local) {
                const int ab = local & 1;
                const uint32_t aph = (local >> 1) & 1;
                if (!mbar_wait(&S.acc_empty[ab], aph ^ 1u, abort_flag, args.err, kErrTimeoutAccumFree)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(ab * kBN);
                for (int kb = 0; kb < nk; ++kb) {
                    if (!mbar_wait(&S.full[s], ph, abort_flag, args.err, kErrTimeoutFull)) {
                        ok = false;
                        break;
                    }
                    const int bb = conv & 1;
                    if (kConvert && !mbar_wait(&S.bu_full[bb], (conv >> 1) & 1u, abort_flag, args.err, kErrTimeoutFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = L::kAPacked ? smem_u32(sAu + bb * kABytes) : smem_u32(sA + s * kABytes);
                    const uint32_t b_addr = L::kBPacked ? smem_u32(sBu + bb * kBBytes) : smem_u32(sB + s * kBBytes);
#pragma unroll
                    for (int k = 0; k < kBK / kUmmaK; ++k) {
                        mma_i8(d_tmem, smem_desc_sw128(a_addr + k * kUmmaK), smem_desc_sw128(b_addr + k * kUmmaK),
                               idesc, (kb | k) != 0 ? 1u : 0u);
                    }
                    mma_commit(&S.empty[s]);
                    if (kConvert) {
                        mma_commit(&S.bu_empty[bb]);
                        ++conv;
                    }
                    if (++s == kStages) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
                if (!ok) break;
                mma_commit(&S.acc_full[ab]);
            }
            // Whatever was issued must finish before TMEM and smem go away.
            mma_commit(&S.drain);
            mbar_wait(&S.drain, 0u, nullptr, args.err, kErrTimeoutDrain);
        }
    } else if (warp < 2 + kEpilogueWarps) {
        // ------------------------------------------------------------------ epilogue
        // Every epilogue warp runs the same number of named barriers per tile even
        // after an abort, so a failed wait can never strand a warp at bar.sync.
        const int quad = warp & 3;  // TMEM lanes [32*quad, 32*quad+32) are visible to this warp
        const int ethread = threadIdx.x - 2 * 32;
        bool alive = true;
        int local = 0;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
            const int ab = local & 1;
            const uint32_t aph = (local >> 1) & 1;
            const int m0 = (t / num_n) * kBM;
            const int n0 = (t % num_n) * kBN;
            // Stage this tile's column scales and bias (previous tile's readers are done).
            named_barrier(1, kEpilogueThreads);
            if (args.out_mode == kOutBf16) {
                for (int c = ethread; c < kBN; c += kEpilogueThreads) {
                    const int n = n0 + c;
                    const bool in = n < args.n;
                    S.col_scale[c] = in ? args.w_scale[args.w_scale_count == 1 ? 0 : n] : 0.0f;
                    S.col_bias[c] = (in && args.bias != nullptr) ? args.bias[n] : 0.0f;
                }
            }
            named_barrier(1, kEpilogueThreads);
            if (alive) {
                int ok = 1;
                if (lane == 0) ok = mbar_wait(&S.acc_full[ab], aph, abort_flag, args.err, kErrTimeoutAccum) ? 1 : 0;
                alive = __shfl_sync(0xffffffffu, ok, 0) != 0;
            }
            if (!alive) continue;
            tc_fence_after();
            const int row = quad * 32 + lane;
            const int m = m0 + row;
            const bool row_ok = m < args.m;
            const float a_s = (row_ok && args.out_mode == kOutBf16) ? args.a_scale[m] : 0.0f;
#pragma unroll 1
            for (int c = 0; c < kBN / 32; ++c) {
                uint32_t acc[32];
                tmem_ld_32x32b_x32(tmem_base + static_cast<uint32_t>(ab * kBN + c * 32) +
                                       (static_cast<uint32_t>(quad * 32) << 16),
                                   acc);
                tmem_ld_wait();
                const int n = n0 + c * 32;
                const int valid = args.n - n;
                if (row_ok && valid > 0) {
                    if (args.out_mode == kOutBf16) {
                        __nv_bfloat16 *dst = static_cast<__nv_bfloat16 *>(args.out) + static_cast<int64_t>(m) * args.ldc + n;
                        store_chunk_bf16(dst, acc, a_s, &S.col_scale[c * 32], &S.col_bias[c * 32], valid);
                    } else {
                        int32_t *dst = static_cast<int32_t *>(args.out) + static_cast<int64_t>(m) * args.ldc + n;
                        store_chunk_s32(dst, acc, valid);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.acc_empty[ab]);
        }
    } else if (kConvert) {
        // ------------------------------------------------------------------ int4 converters
        // 128 threads turn the packed tiles of ring stage s (k pairs per byte) into the
        // int8 tiles of buffer bb.  One leader waits on the barriers; the decision is
        // shared through the converters' named barrier so all 128 threads always take
        // the same path.
        const int cthread = threadIdx.x - (2 + kEpilogueWarps) * 32;
        int s = 0;
        uint32_t ph = 0;
        uint32_t conv = 0;
        bool alive = true;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
            for (int kb = 0; kb < nk; ++kb) {
                const int bb = conv & 1;
                if (cthread == 0) {
                    bool ok = alive && mbar_wait(&S.full[s], ph, abort_flag, args.err, kErrTimeoutFull);
                    ok = ok && mbar_wait(&S.bu_empty[bb], ((conv >> 1) & 1u) ^ 1u, abort_flag, args.err,
                                         kErrTimeoutEmpty);
                    S.conv_ok = ok ? 1 : 0;
                }
                named_barrier(2, kConverterThreads);
                alive = S.conv_ok != 0;
                if (alive) {
                    if (L::kAPacked) convert_tile<kBM>(sA + s * kAPackedBytes, sAu + bb * kABytes, cthread);
                    if (L::kBPacked) convert_tile<kBN>(sB + s * kBPackedBytes, sBu + bb * kBBytes, cthread);
                    fence_proxy_async_smem();  // generic writes -> visible to the MMA (async proxy)
                }
                named_barrier(2, kConverterThreads);
                if (cthread == 0 && alive) {
                    mbar_arrive(&S.bu_full[bb]);
                    mbar_arrive(&S.empty[s]);  // packed stage consumed
                }
                ++conv;
                if (++s == kStages) {
                    s = 0;
                    ph ^= 1u;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

template __global__ void int8_gemm_kernel<kModeW8A8>(const __grid_constant__ CUtensorMap,
                                                     const __grid_constant__ CUtensorMap, const GemmArgs);
template __global__ void int8_gemm_kernel<kModeW4A8>(const __grid_constant__ CUtensorMap,
                                                     const __grid_constant__ CUtensorMap, const GemmArgs);
template __global__ void int8_gemm_kernel<kModeW4A4>(const __grid_constant__ CUtensorMap,
                                                     const __grid_constant__ CUtensorMap, const GemmArgs);

}  // namespace gemm
}  // namespace ctu
