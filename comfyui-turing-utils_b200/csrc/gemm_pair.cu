// CTA-pair integer GEMMs (tcgen05.mma.cta_group::2, kind::i8) with the same fused
// ConvRot epilogue as the single-CTA kernel:
//
//   out[m, n] = bf16( fma(float(acc[m, n]) * a_scale[m], w_scale[n], bias[n]) )
//
// A cluster of two CTAs (one per SM) owns a 256 x 256 output tile.  CTA r of the pair
// stages activation rows [128 r, 128 r + 128) and weight rows [128 r, 128 r + 128) of
// the tile; the leader (r = 0) issues one M = 256, N = 256, K = 32 MMA per step that
// reads A from each CTA's own shared memory and B from both, and writes each CTA's
// 128 accumulator rows into that CTA's TMEM.  Per SM and per K block this halves the
// weight bytes that cross shared memory (the single-CTA kernel stages the whole
// 256-row weight tile in every CTA), which is what bounds the single-CTA kernel.
//
// Roles per CTA (warp-specialised, persistent over pair tiles, n-fastest):
//   warp 0      TMA producer for this CTA's halves.  W8A8: the copies signal the
//               leader's `full` barrier (.cta_group::2), and only the leader's
//               producer posts the expected byte count for both CTAs.  int4 modes:
//               the packed copies signal this CTA's own `full` barrier.
//   warp 1      pair TMEM allocation (both CTAs); in the leader, the MMA issuer.
//               Its commits arrive on both CTAs' barriers (multicast mask 0b11).
//   warps 2..5  epilogue over this CTA's 128 rows; releases the accumulator buffer
//               on the leader's barrier (8 arrivals: 4 warps x 2 CTAs).
//   warps 6..   (int4 modes) converters, one per ring stage (W4A4: two): sign-extend
//               this CTA's packed tiles of the stage into the stage's 128-byte-swizzled
//               int8 copies, then arrive on the leader's `bu_full[stage]` (one arrival
//               per converter warp of each CTA).
//               (fused ConvRot linear, kGt > 0) quantizer warps: claim bf16 input rows
//               in order, rotate and quantize each with the warp-row pipeline, write its
//               codes and scale, and count it in its 128-row block; the producer loads an
//               activation tile once its block is complete, so quantization of later
//               rows overlaps the MMAs of earlier ones.
// Every wait is bounded; a role that gives up raises the abort flag in both CTAs so
// the pair stops together, and both CTAs stay resident until the final cluster
// barrier, so no remote arrival or copy can target a CTA that has exited.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "convrot_rowwarp.cuh"
#include "gemm_i8.cuh"
#include "gemm_tile.cuh"
#include "ptx.cuh"

namespace ctu {
namespace gemm {

namespace {

struct PairSmem {
    uint64_t full[8];
    uint64_t empty[8];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];  // used in the leader only
    uint64_t bu_full[8];    // int4 modes, leader only: stage s converted in both CTAs
    uint64_t drain;
    uint64_t qbar[kFusedQuantWarps];  // fused linear: row copy of each quantizer warp
    uint32_t tmem_base;
    int abort_flag;
    float col_scale[kBN];
    float col_bias[kBN];
};

__device__ __forceinline__ void st_cluster_u32(uint32_t cluster_addr, uint32_t v) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}

// Abort state of one CTA: its own flag, the peer's flag (cluster address), error word.
struct PairAbort {
    volatile int *flag;
    uint32_t peer_flag;
    uint32_t *err;

    __device__ __forceinline__ void raise() const {
        *flag = 1;
        st_cluster_u32(peer_flag, 1u);
    }
    // Bounded wait on a barrier whose arrivals come from this CTA or from tcgen05
    // commits.  On failure the peer is told to stop as well.
    __device__ __forceinline__ bool wait(uint64_t *bar, uint32_t parity, uint32_t code) const {
        if (mbar_wait(bar, parity, flag, err, code)) return true;
        raise();
        return false;
    }
    // Same, with cluster-scope acquire, for barriers the peer CTA's threads arrive on.
    __device__ __forceinline__ bool wait_cluster(uint64_t *bar, uint32_t parity, uint32_t code) const {
        if (mbar_wait_cluster(bar, parity, flag, err, code)) return true;
        raise();
        return false;
    }
};

// Bounded pause (by %globaltimer) that lets bulk copies already issued land before a
// CTA that gave up leaves; used only on the abort path of the W8A8 pair, whose copies
// complete on the other CTA's barrier and so cannot be waited for one by one.
__device__ __forceinline__ void settle_inflight_copies() {
    const uint64_t start = globaltimer();
    while (globaltimer() - start < 1000000ull) __nanosleep(1000);
}

}  // namespace

template <int kMode, int kGt>
__global__ void __cluster_dims__(2, 1, 1)
    __launch_bounds__(kGt > 0 ? kFusedThreadCount : PairLayout<kMode>::kThreadCount, 1)
    int8_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                          const __grid_constant__ CUtensorMap tmap_b_narrow, const GemmArgs args) {
    using L = PairLayout<kMode>;
    constexpr bool kConvert = L::kConvert;
    constexpr bool kFused = kGt > 0;
    // The fused linear runs a shallower ring so the quantizer warps' row buffers fit.
    constexpr int kStagesP = kFused ? kFusedStages : L::kStages;
    static_assert(kStagesP <= 8, "barrier arrays hold 8 stages");
    static_assert(!kFused || (kMode == kModeW8A8 && kGt <= kFusedMaxGt), "fused linear: W8A8, k <= 5120");
    extern __shared__ uint8_t smem_raw[];
    // Same offset in both CTAs: the MMA addresses the peer's operands at this CTA's offsets.
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem + L::kAOffset;
    uint8_t *sB = smem + (kFused ? kFusedStages * L::kAStageBytes : L::kBOffset);
    uint8_t *sAu = smem + L::kAuOffset;
    uint8_t *sBu = smem + L::kBuOffset;
    PairSmem &S = *reinterpret_cast<PairSmem *>(smem + (kFused ? kFusedStructOffset : L::kStructOffset));

    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int pair = blockIdx.x >> 1;
    const int num_pairs = gridDim.x >> 1;
    const int num_n = (args.n + kBN - 1) / kBN;
    const int num_m = (args.m + kPairBM - 1) / kPairBM;
    const int num_tiles = num_m * num_n;
    const int nk = (args.k + kBK - 1) / kBK;
    // Work items: tiles [0, num_full) whole, then each of the last split_tiles tiles as
    // two 128-column halves (W8A8 only).
    const int split = kConvert ? 0 : args.split_tiles;
    const int num_full = num_tiles - split;
    const int num_work = num_tiles + split;
    // Output tile row index, first column and width of work item w.
    auto work_item = [&](int w, int &m_tile, int &n0, int &ncols) {
        int t = w;
        int half = 0;
        if (w >= num_full) {
            t = num_full + ((w - num_full) >> 1);
            half = (w - num_full) & 1;
        }
        m_tile = t / num_n;
        ncols = w >= num_full ? kHalfBN : kBN;
        n0 = (t - m_tile * num_n) * kBN + half * kHalfBN;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStagesP; ++s) {
            mbar_init(&S.full[s], 1);
            // int4 modes: a stage (packed and converted parts) is free once the MMA
            // has read it and this CTA's converters are done with it.
            mbar_init(&S.empty[s], kConvert ? 1 + L::kConvWarpsPerStage : 1);
            mbar_init(&S.bu_full[s], 2 * L::kConvWarpsPerStage);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&S.acc_full[b], 1);
            mbar_init(&S.acc_empty[b], 2 * kEpilogueWarps);
        }
        mbar_init(&S.drain, 1);
        for (int i = 0; i < kFusedQuantWarps; ++i) mbar_init(&S.qbar[i], 1);
        S.abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(&S.tmem_base, kTmemCols);
        tmem_relinquish_pair();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_b);
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers initialised before any remote arrival
    tc_fence_after();
    const uint32_t tmem_base = S.tmem_base;
    const PairAbort ab_state{&S.abort_flag, mapa_shared(smem_u32(&S.abort_flag), rank ^ 1u), args.err};
    volatile int *abort_flag = &S.abort_flag;

    if (warp == 0) {
        // ------------------------------------------------------------------ producer
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            uint32_t fills = 0;
            bool ok = true;
            for (int t = pair; t < num_work && ok; t += num_pairs) {
                int m_tile, n0, ncols;
                work_item(t, m_tile, n0, ncols);
                const int m0 = m_tile * kPairBM + static_cast<int>(rank) * kBM;
                const bool narrow = ncols != kBN;  // each CTA stages ncols / 2 weight rows
                const int w0 = n0 + static_cast<int>(rank) * (ncols / 2);
                if constexpr (kFused) {
                    // This CTA's activation rows must all be quantized before the tile's
                    // first copy; the proxy fence makes the tensor-map loads read them.
                    const int need = min(kBM, args.m - m0);
                    if (need > 0 && !counter_wait(args.qsync + 1 + (m0 >> 7), static_cast<uint32_t>(need), abort_flag,
                                                  args.err, kErrTimeoutRows)) {
                        ab_state.raise();
                        ok = false;
                        break;
                    }
                    fence_proxy_async_global();
                }
                for (int kb = 0; kb < nk; ++kb) {
                    if (!ab_state.wait(&S.empty[s], ph ^ 1u, kErrTimeoutEmpty)) {
                        ok = false;
                        break;
                    }
                    uint8_t *dst_a = sA + s * L::kAStageBytes;
                    uint8_t *dst_b = sB + s * L::kBStageBytes;
                    if constexpr (kConvert) {
                        mbar_arrive_expect_tx(&S.full[s], L::kAStageBytes + L::kBStageBytes);
                        tma_load_2d(dst_a, &tmap_a, kb * (L::kAPacked ? kBK / 2 : kBK), m0, &S.full[s]);
                        tma_load_2d(dst_b, &tmap_b, kb * (kBK / 2), w0, &S.full[s]);
                    } else {
                        const uint32_t leader_full = mapa_shared(smem_u32(&S.full[s]), 0u);
                        const uint32_t b_bytes = narrow ? L::kBStageBytes / 2 : L::kBStageBytes;
                        if (leader) mbar_arrive_expect_tx(&S.full[s], 2 * (L::kAStageBytes + b_bytes));
                        tma_load_2d_pair(dst_a, &tmap_a, kb * kBK, m0, leader_full);
                        tma_load_2d_pair(dst_b, narrow ? &tmap_b_narrow : &tmap_b, kb * kBK, w0, leader_full);
                    }
                    ++fills;
                    if (++s == kStagesP) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
            }
            if (!ok || *abort_flag) {
                if constexpr (kConvert) {
                    // Own copies signal own barriers: wait for the last fills to land.
                    for (uint32_t i = 0; i < static_cast<uint32_t>(kStagesP) && i < fills; ++i) {
                        const uint32_t fill = fills - 1 - i;
                        mbar_wait(&S.full[fill % kStagesP], (fill / kStagesP) & 1u, nullptr, args.err,
                                  kErrTimeoutDrain);
                    }
                } else {
                    settle_inflight_copies();
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer (leader)
        if (leader && lane == 0) {
            constexpr uint32_t idesc_full = idesc_i8(kPairBM, kBN);
            constexpr uint32_t idesc_half = idesc_i8(kPairBM, kHalfBN);
            int s = 0;
            uint32_t ph = 0;
            int local = 0;
            bool ok = true;
            if (args.inject_timeout) {
                // Test hook: a wait nothing will satisfy must time out and stop both CTAs.
                if (!mbar_wait(&S.drain, 0u, abort_flag, args.err, kErrInjected, args.inject_timeout_ns))
                    ab_state.raise();
                ok = false;
            }
            for (int t = pair; t < num_work && ok; t += num_pairs, ++local) {
                const int ab = local & 1;
                const uint32_t aph = (local >> 1) & 1;
                const uint32_t idesc = t >= num_full ? idesc_half : idesc_full;
                if (!ab_state.wait_cluster(&S.acc_empty[ab], aph ^ 1u, kErrTimeoutAccumFree)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(ab * kBN);
                for (int kb = 0; kb < nk; ++kb) {
                    if constexpr (kConvert) {
                        // Both CTAs' converters arrive only after their stage landed and
                        // their converted tiles are fenced for the async proxy.
                        if (!ab_state.wait_cluster(&S.bu_full[s], ph, kErrTimeoutFull)) {
                            ok = false;
                            break;
                        }
                    } else {
                        if (!ab_state.wait(&S.full[s], ph, kErrTimeoutFull)) {
                            ok = false;
                            break;
                        }
                    }
                    tc_fence_after();
                    const uint32_t a_addr =
                        L::kAPacked ? smem_u32(sAu + s * L::kAuStageBytes) : smem_u32(sA + s * L::kAStageBytes);
                    const uint32_t b_addr =
                        L::kBPacked ? smem_u32(sBu + s * L::kBuStageBytes) : smem_u32(sB + s * L::kBStageBytes);
#pragma unroll
                    for (int k = 0; k < kBK / kUmmaK; ++k) {
                        mma_i8_pair(d_tmem, smem_desc_sw128(a_addr + k * kUmmaK), smem_desc_sw128(b_addr + k * kUmmaK),
                                    idesc, (kb | k) != 0 ? 1u : 0u);
                    }
                    mma_commit_pair_both(&S.empty[s]);
                    if (++s == kStagesP) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
                if (!ok) break;
                mma_commit_pair_both(&S.acc_full[ab]);
            }
            // Everything issued must complete before either CTA releases TMEM or smem.
            mma_commit_pair_local(&S.drain);
            mbar_wait(&S.drain, 0u, nullptr, args.err, kErrTimeoutDrain);
        }
    } else if (warp < 2 + kEpilogueWarps) {
        // ------------------------------------------------------------------ epilogue
        const int quad = warp & 3;
        const int ethread = threadIdx.x - 2 * 32;
        const uint32_t leader_acc_empty0 = mapa_shared(smem_u32(&S.acc_empty[0]), 0u);
        bool alive = true;
        int local = 0;
        for (int t = pair; t < num_work; t += num_pairs, ++local) {
            const int ab = local & 1;
            const uint32_t aph = (local >> 1) & 1;
            int m_tile, n0, ncols;
            work_item(t, m_tile, n0, ncols);
            const int m0 = m_tile * kPairBM + static_cast<int>(rank) * kBM;
            named_barrier(1, kEpilogueThreads);
            if (args.out_mode == kOutBf16) {
                for (int c = ethread; c < ncols; c += kEpilogueThreads) {
                    const int n = n0 + c;
                    const bool in = n < args.n;
                    S.col_scale[c] = in ? args.w_scale[args.w_scale_count == 1 ? 0 : n] : 0.0f;
                    S.col_bias[c] = (in && args.bias != nullptr) ? args.bias[n] : 0.0f;
                }
            }
            named_barrier(1, kEpilogueThreads);
            if (alive) {
                int ok = 1;
                if (lane == 0) ok = ab_state.wait(&S.acc_full[ab], aph, kErrTimeoutAccum) ? 1 : 0;
                alive = __shfl_sync(0xffffffffu, ok, 0) != 0;
            }
            if (!alive) continue;
            tc_fence_after();
            const int row = quad * 32 + lane;
            const int m = m0 + row;
            const bool row_ok = m < args.m;
            float a_s = 0.0f;
            if constexpr (kFused) {
                // The producer saw this block complete before loading it; this acquire
                // orders the scale loads after the quantizer warps' release as well.
                const int need = min(kBM, args.m - m0);
                if (need > 0) counter_wait(args.qsync + 1 + (m0 >> 7), static_cast<uint32_t>(need), abort_flag, args.err,
                                           kErrTimeoutRows);
                if (row_ok) a_s = __ldcg(args.a_scale + m);
            } else {
                a_s = (row_ok && args.out_mode == kOutBf16) ? args.a_scale[m] : 0.0f;
            }
#pragma unroll 1
            for (int c = 0; c < ncols / 32; ++c) {
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
            if (lane == 0) mbar_arrive_remote(leader_acc_empty0 + static_cast<uint32_t>(ab * sizeof(uint64_t)));
        }
    } else if (kConvert) {
        // ------------------------------------------------------------------ int4 converters
        // Converter warp w owns ring stage w % kStages (W4A4: warp w < kStages converts
        // the activation tile, warp w + kStages the weight half-tile) and converts
        // every use of it in order, so each warp waits at most one phase ahead and up
        // to kStages stage conversions -- each a chain of barrier wait, loads, stores,
        // proxy fence and arrival -- run at once.  Stage s's converted copies are free
        // whenever its packed part is: the producer refills stage s only after the MMA
        // that read them has completed.
        const int cwarp = warp - (2 + kEpilogueWarps);
        const int s = cwarp % kStagesP;
        const int part = cwarp / kStagesP;
        const uint32_t leader_bu_full = mapa_shared(smem_u32(&S.bu_full[s]), 0u);
        const int my_tiles = pair < num_tiles ? (num_tiles - 1 - pair) / num_pairs + 1 : 0;
        const int64_t total = static_cast<int64_t>(my_tiles) * nk;  // k blocks of this CTA
        for (int64_t i = s; i < total; i += kStagesP) {
            const uint32_t ph = static_cast<uint32_t>((i / kStagesP) & 1);
            int ok = 1;
            if (lane == 0) ok = ab_state.wait(&S.full[s], ph, kErrTimeoutFull) ? 1 : 0;
            if (__shfl_sync(0xffffffffu, ok, 0) == 0) break;
            if (L::kAPacked && part == 0)
                convert_tile<kBM, 32>(sA + s * L::kAStageBytes, sAu + s * L::kAuStageBytes, lane);
            if (L::kBPacked && part == L::kConvWarpsPerStage - 1)
                convert_tile<kHalfBN, 32>(sB + s * L::kBStageBytes, sBu + s * L::kBuStageBytes, lane);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive_remote(leader_bu_full);
                mbar_arrive(&S.empty[s]);
            }
        }
    } else if constexpr (kFused) {
        // ------------------------------------------------------------------ ConvRot quantizer warps
        // Warp-row pipeline (convrot_rowwarp.cuh): a row is copied into this warp's
        // buffer by one bulk copy, rotated with the halvings folded, and quantized to
        // int8 with the per-row scale absmax / 127; the next claimed row's copy is in
        // flight while the codes are written.
        const int qw = warp - (2 + kEpilogueWarps);
        const int K = args.k;
        const int groups = K / 256;
        const uint32_t row_bytes = static_cast<uint32_t>(K) * 2u;
        const uint32_t buf_bytes = static_cast<uint32_t>(fused_quant_buffer_bytes(K));
        uint8_t *qbuf = smem + kFusedQuantOffset + qw * (buf_bytes + kFusedQuantTransposeBytes);
        const uint32_t buf = smem_u32(qbuf);
        uint64_t *bar = &S.qbar[qw];
        const uint32_t g = static_cast<uint32_t>(lane >> 3);
        const uint32_t q = static_cast<uint32_t>(lane & 7);
        const uint32_t garea = buf + buf_bytes + g * 1024u;
        const uint32_t wbase = garea + 16u * ((4u * q) ^ (q >> 1) ^ (4u * (g & 1u)));
        const uint32_t rbase = garea + 8u * (q & 1u) + 16u * ((q >> 1) ^ (4u * (g & 1u)));
        const ctu::rot::ActLut lut{nullptr, nullptr};
        const uint16_t *x = static_cast<const uint16_t *>(args.qx);
        uint32_t *claim = args.qsync;
        uint32_t *done = args.qsync + 1;

        int row = 0;
        if (lane == 0) {
            row = static_cast<int>(atomicAdd(claim, 1u));
            if (row < args.m) {
                mbar_arrive_expect_tx(bar, row_bytes);
                bulk_load(qbuf, x + static_cast<int64_t>(row) * K, row_bytes, bar);
            }
        }
        row = __shfl_sync(0xffffffffu, row, 0);
        bool pending = row < args.m;  // lane 0: a copy is in flight
        uint32_t it = 0;
        // A row is counted in its block one row later, once its code stores are long
        // complete, so the fence in front of the count does not stall on them.
        int unpublished = -1;
        auto publish = [&](int r) {
            // Codes are read by other SMs' tensor-map loads (async proxy), the scale by
            // their epilogues.  __syncwarp orders every lane's stores before lane 0's
            // release, which is cumulative over them.
            fence_proxy_async_global();
            __syncwarp();
            if (lane == 0) red_release_gpu_add(done + (r >> 7), 1u);
        };
        while (row < args.m) {
            int next = 0;
            if (lane == 0) next = static_cast<int>(atomicAdd(claim, 1u));  // used after the rotation
            int ok = 1;
            if (lane == 0) ok = mbar_wait(bar, it & 1u, abort_flag, args.err, kErrTimeoutFull) ? 1 : 0;
            if (__shfl_sync(0xffffffffu, ok, 0) == 0) {
                ab_state.raise();
                break;
            }
            pending = false;
            uint32_t W[kGt > 0 ? kGt : 1][16];
            bool folded[kGt > 0 ? kGt : 1];
            float amax = 0.0f;
            bool any_nan = false;
            ctu::rot::w8_rotate_row<ctu::rot::kActNone, kGt>(buf, groups, g, q, wbase, rbase, lut, W, folded, amax,
                                                             any_nan);
            next = __shfl_sync(0xffffffffu, next, 0);
            if (lane == 0 && next < args.m) {
                mbar_arrive_expect_tx(bar, row_bytes);
                bulk_load(qbuf, x + static_cast<int64_t>(next) * K, row_bytes, bar);
                pending = true;
            }
            amax = ctu::rot::w8_row_absmax(amax);
            const bool row_nan = __any_sync(0xffffffffu, any_nan);
            const float scale = ctu::rot::row_scale<8>(amax, false);
            if (unpublished >= 0) publish(unpublished);
            if (lane == 0) args.qscales[row] = scale;
            ctu::rot::w8_store_codes<8, kGt>(W, folded, amax, scale, row_nan, groups, g, q,
                                             args.qcodes + static_cast<int64_t>(row) * K);
            unpublished = row;
            row = next;
            ++it;
        }
        if (unpublished >= 0 && row >= args.m) publish(unpublished);  // not after an abort
        if (lane == 0 && pending) {
            // A wait gave up with a copy still in flight: let it land before the CTA exits.
            mbar_wait(bar, it & 1u, nullptr, args.err, kErrTimeoutDrain);
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // neither CTA leaves while the other may still address its memory
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, kTmemCols);
    }
}

template __global__ void int8_gemm_pair_kernel<kModeW8A8>(const __grid_constant__ CUtensorMap,
                                                          const __grid_constant__ CUtensorMap,
                                                          const __grid_constant__ CUtensorMap, const GemmArgs);
template __global__ void int8_gemm_pair_kernel<kModeW4A8>(const __grid_constant__ CUtensorMap,
                                                          const __grid_constant__ CUtensorMap,
                                                          const __grid_constant__ CUtensorMap, const GemmArgs);
template __global__ void int8_gemm_pair_kernel<kModeW4A4>(const __grid_constant__ CUtensorMap,
                                                          const __grid_constant__ CUtensorMap,
                                                          const __grid_constant__ CUtensorMap, const GemmArgs);
#define CTU_FUSED_LINEAR(GT)                                                                                    \
    template __global__ void int8_gemm_pair_kernel<kModeW8A8, GT>(                                              \
        const __grid_constant__ CUtensorMap, const __grid_constant__ CUtensorMap, const __grid_constant__ CUtensorMap, \
        const GemmArgs);
CTU_FUSED_LINEAR(1)
CTU_FUSED_LINEAR(2)
CTU_FUSED_LINEAR(3)
CTU_FUSED_LINEAR(4)
CTU_FUSED_LINEAR(5)
#undef CTU_FUSED_LINEAR

}  // namespace gemm
}  // namespace ctu
