// W8A8 integer GEMM on the 5th-generation tensor cores (tcgen05, kind::i8) with
// the ConvRot dequant + bias epilogue fused:
//
//   out[m, n] = bf16( ((float(acc[m, n]) * a_scale[m]) * w_scale[n]) + bias[n] )
//   acc[m, n] = sum_k a[m, k] * w[n, k]          (exact int32)
//
// This replaces the reference's CUTLASS SM75 mma.sync GEMM
// (kernel/csrc/turing/w4a8.cu:376-618, entry w4a8.cu:1185-1219) and keeps its
// epilogue order (w4a8.cu:474-525: scale by the activation scale, then the
// weight scale, then add the bias, round to bf16).
//
// Design (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A [128 x 128 B] and B [256 x 128 B] tiles, 128-byte
//               swizzle, into a kStages-deep shared-memory ring (mbarrier per stage)
//   warp 1      MMA issuer: owns the TMEM allocation (512 columns = two 128x256
//               int32 accumulators), issues tcgen05.mma M=128 N=256 K=32, frees
//               smem stages with tcgen05.commit
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time, fused scale/bias/bf16,
//               16-byte global stores; releases the accumulator buffer so the next
//               tile's MMAs overlap this tile's epilogue
// Tiles are visited n-fastest so the CTAs resident at one time share the same A
// rows and the whole weight matrix stays L2-resident.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "gemm_i8.cuh"
#include "ptx.cuh"

namespace ctu {
namespace gemm {

struct Smem {
    uint64_t full[kStages];
    uint64_t empty[kStages];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort_flag;
    float col_scale[kBN];
    float col_bias[kBN];
};

__device__ __forceinline__ void named_barrier_epilogue() {
    asm volatile("bar.sync 1, %0;" ::"n"(kEpilogueThreads) : "memory");
}

__device__ __forceinline__ void store_chunk_bf16(__nv_bfloat16 *dst, const uint32_t (&acc)[32], float a_s,
                                                 const float *ws, const float *bs, int valid_cols) {
    uint32_t packed[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        float v0 = __fmul_rn(__int2float_rn(static_cast<int>(acc[2 * j])), a_s);
        float v1 = __fmul_rn(__int2float_rn(static_cast<int>(acc[2 * j + 1])), a_s);
        v0 = __fadd_rn(__fmul_rn(v0, ws[2 * j]), bs[2 * j]);
        v1 = __fadd_rn(__fmul_rn(v1, ws[2 * j + 1]), bs[2 * j + 1]);
        packed[j] = pack_bf16x2(v0, v1);
    }
    uint4 *d = reinterpret_cast<uint4 *>(dst);
    if (valid_cols >= 32) {
#pragma unroll
        for (int q = 0; q < 4; ++q) d[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
    } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if (8 * q < valid_cols) d[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
        }
    }
}

__device__ __forceinline__ void store_chunk_s32(int32_t *dst, const uint32_t (&acc)[32], int valid_cols) {
    uint4 *d = reinterpret_cast<uint4 *>(dst);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        if (4 * q < valid_cols) d[q] = make_uint4(acc[4 * q], acc[4 * q + 1], acc[4 * q + 2], acc[4 * q + 3]);
    }
}

__global__ void __launch_bounds__(kThreads, 1)
    w8a8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                     const GemmArgs args) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + kStages * kABytes;
    Smem &S = *reinterpret_cast<Smem *>(sB + kStages * kBBytes);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_n = (args.n + kBN - 1) / kBN;
    const int num_m = (args.m + kBM - 1) / kBM;
    const int num_tiles = num_m * num_n;
    const int nk = (args.k + kBK - 1) / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&S.acc_full[b], 1);
            mbar_init(&S.acc_empty[b], kEpilogueWarps);
        }
        mbar_init(&S.drain, 1);
        S.abort_flag = 0;
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
                    mbar_arrive_expect_tx(&S.full[s], kABytes + kBBytes);
                    tma_load_2d(sA + s * kABytes, &tmap_a, kb * kBK, m0, &S.full[s]);
                    tma_load_2d(sB + s * kBBytes, &tmap_b, kb * kBK, n0, &S.full[s]);
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
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sA + s * kABytes);
                    const uint32_t b_addr = smem_u32(sB + s * kBBytes);
#pragma unroll
                    for (int k = 0; k < kBK / kUmmaK; ++k) {
                        mma_i8(d_tmem, smem_desc_sw128(a_addr + k * kUmmaK), smem_desc_sw128(b_addr + k * kUmmaK),
                               idesc, (kb | k) != 0 ? 1u : 0u);
                    }
                    mma_commit(&S.empty[s]);
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
    } else {
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
            named_barrier_epilogue();
            if (args.out_mode == kOutBf16) {
                for (int c = ethread; c < kBN; c += kEpilogueThreads) {
                    const int n = n0 + c;
                    const bool in = n < args.n;
                    S.col_scale[c] = in ? args.w_scale[args.w_scale_count == 1 ? 0 : n] : 0.0f;
                    S.col_bias[c] = (in && args.bias != nullptr) ? args.bias[n] : 0.0f;
                }
            }
            named_barrier_epilogue();
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
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

}  // namespace gemm
}  // namespace ctu
