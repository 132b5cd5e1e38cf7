// Per-group (128 along K) integer GEMMs for the asymmetric W4A8 and the W4A4 linears:
//
//   W4A8: t = sum_g fma(w_scale[g][n], float(acc_g[m, n]), t);  out = bf16(fma(t, a_scale[m], bias[n]))
//   W4A4: t = sum_g fma(float(acc_g[m, n]) * a_scale[m][g], w_scale[g][n], t);  out = bf16(t + bias[n])
//
// with acc_g the exact int32 product of group g's 128 columns.  Two tilings share the code:
//   single (kPair = false)  one CTA owns a 128 x 128 output tile (tcgen05.mma.cta_group::1,
//                           M = 128, N = 128) and stages 128 activation and 128 weight rows
//                           of each group;
//   pair   (kPair = true)   a cluster of two CTAs owns a 256 x 128 tile (cta_group::2,
//                           M = 256): CTA r stages activation rows [128 r, 128 r + 128)
//                           and weight rows [64 r, 64 r + 64) of each group.
// One ring stage is one group (four K = 32 MMAs).  Each group's partial lands in its own
// 128-column TMEM buffer, and there are four, so the MMA runs up to four groups ahead of
// the epilogue that converts and scales them.  The single tiling stages twice the weight
// bytes per MMA, but each buffer goes back to the MMA through a CTA-local barrier; the
// pair's non-leader must relay its releases to the leader (see the roles below).
//
// Conversion without I2F.  The group's first MMA overwrites the buffer, so it holds the
// exact int32 partial acc, |acc| <= 128 * 128 * 15 < 2^22.  For such acc the bit pattern
// (acc & 0x7FFFFF) ^ 0x4B400000 is the float 1.5 * 2^23 + acc (floats in [2^23, 2^24) are
// the integers; bits 0..21 are acc's, bit 22 is the complement of its sign-extension
// bit, the exponent is the constant's), so float(acc) is one bitwise operation and one
// exact packed subtract of 1.5 * 2^23.  TMEM is only read: writing a pattern back costs
// more TMEM bandwidth than the MMAs leave.
//
// Throughput.  Per group and CTA the epilogue does one ALU and 2 (W4A8) or 3 (W4A4) fp32
// operations on each of 128 x 128 partials: 256 cycles of the ALU pipe and 256 or 384 of
// the 128-lane FMA pipe, against about 262 cycles for the group's MMAs (M = 256, N = 128,
// K = 128 on two SMs, or M = 128 on one).  So the
// per-group control work is kept to a few instructions per warp, each warp reads its
// partials of a group with one TMEM load (one load latency per group) straight into
// register pairs, the scales arrive as pairs next to their use, and 16 epilogue warps (4
// per scheduler) keep enough of these latency-bound chains in flight.
//
// Roles per CTA (persistent over tiles, n-fastest):
//   warp 0      producer: the stage's A and B tiles (completing on the leader's `full`
//               barrier), and the group's 128 fp32 weight scales into this CTA's scale
//               ring (completing on its own `sc_full`).
//   warp 1      TMEM allocation.  Single CTA: the MMA issuer, which waits for each buffer's
//               release on `acc_free`.  Pair leader: the MMA issuer; non-leader: forwards its
//               epilogue's buffer releases to the leader's `acc_empty` (one remote
//               arrival per release instead of one per epilogue warp).  The four buffers
//               are released in pairs (groups 2i and 2i + 1 together): a remote arrival
//               with cluster-scope release keeps the forwarding thread about a microsecond
//               (a globaltimer trace; a relaxed or CTA-scope arrival is faster but let the
//               MMA overwrite partials the peer had not finished reading), so one per two
//               groups halves the time the forwarder paces the pair at.
//   warps 2..   epilogue (kGroupedEpilogueWarps): warp w reads TMEM lanes 32 (w % 4) ..
//               +31 (its rows) and kGroupedEpilogueCols columns from
//               kGroupedEpilogueCols ((w - 2) / 4); one fp32 running sum per column.
// Every wait is bounded; a role that gives up raises the abort flag in both CTAs, and
// both CTAs stay resident until the final cluster barrier.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "gemm_i8.cuh"
#include "gemm_tile.cuh"
#include "ptx.cuh"

namespace ctu {
namespace gemm {

namespace {

constexpr uint32_t kMagicBits = 0x4B400000u;  // 1.5 * 2^23
constexpr uint32_t kAccMask = 0x007FFFFFu;
constexpr float kMagic = 12582912.0f;
constexpr int kGroupedTmemCols = kGroupedBuffers * kGroupedBN;  // 512
constexpr int kLoadCols = 32;  // TMEM columns per epilogue load
static_assert(kGroupedTmemCols == 512, "four 128-column buffers fill TMEM");
static_assert(kGroupedBuffers < GroupedLayout<true>::kStages && kGroupedBuffers < GroupedLayout<false>::kStages,
              "the epilogue identifies a group's MMA completion by stage parity");
static_assert(GroupedLayout<true>::kStages <= kGroupedMaxStages && GroupedLayout<false>::kStages <= kGroupedMaxStages,
              "ring barriers");

struct GroupedSmem {
    uint64_t full[kGroupedMaxStages];
    uint64_t empty[kGroupedMaxStages];
    // Pair: buffer pairs {0, 1} and {2, 3}, each released once both of its groups are read.
    uint64_t acc_empty[kGroupedBuffers / 2];  // leader: its epilogue warps (x2) + 1 forwarded peer release
    uint64_t acc_local[kGroupedBuffers / 2];  // non-leader: its epilogue warps (x2)
    uint64_t acc_free[kGroupedBuffers];       // single CTA: its epilogue warps, per buffer
    uint64_t sc_full[kGroupedScaleSlots];
    uint64_t sc_empty[kGroupedScaleSlots];
    uint64_t drain;
    uint32_t tmem_base;
    int abort_flag;
    alignas(16) float scale_ring[kGroupedScaleSlots][kGroupedBN];
    alignas(16) float col_bias[kGroupedBN];
};
static_assert(sizeof(GroupedSmem) <= kGroupedBookkeepingBytes, "grouped GEMM bookkeeping exceeds its reservation");

__device__ __forceinline__ void st_cluster_u32(uint32_t cluster_addr, uint32_t v) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}

struct GroupedAbort {
    volatile int *flag;
    uint32_t peer_flag;  // the pair's other CTA's flag; 0 for a single CTA
    uint32_t *err;

    __device__ __forceinline__ void raise() const {
        *flag = 1;
        if (peer_flag != 0u) st_cluster_u32(peer_flag, 1u);
    }
    __device__ __forceinline__ bool wait(uint64_t *bar, uint32_t parity, uint32_t code) const {
        if (mbar_wait(bar, parity, flag, err, code)) return true;
        raise();
        return false;
    }
    __device__ __forceinline__ bool wait_cluster(uint64_t *bar, uint32_t parity, uint32_t code) const {
        if (mbar_wait_cluster(bar, parity, flag, err, code)) return true;
        raise();
        return false;
    }
};

// Four fp32 of shared memory, as a volatile load: it stays where it is written (after the
// TMEM read it pairs with) instead of being hoisted to the loop head, which would hold
// every scale of the group in registers at once.
// Returned as two packed pairs, so they feed the packed arithmetic without moves.
__device__ __forceinline__ void lds_f32x2x2(uint32_t addr, f32x2 &a, f32x2 &b) {
    asm volatile("ld.shared.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "r"(addr));
}

// Two int32 partials -> the bit patterns of 1.5 * 2^23 + acc (see the file comment): one
// three-input logic operation, (acc & mask) ^ pattern, per partial.
__device__ __forceinline__ f32x2 to_magic_pair(u32x2 v) {
    f32x2 r;
    asm("{\n\t.reg .b32 lo, hi;\n\t"
        "mov.b64 {lo, hi}, %1;\n\t"
        "lop3.b32 lo, lo, %2, %3, 0x6A;\n\t"
        "lop3.b32 hi, hi, %2, %3, 0x6A;\n\t"
        "mov.b64 %0, {lo, hi};\n\t}"
        : "=l"(r)
        : "l"(v), "r"(kAccMask), "r"(kMagicBits));
    return r;
}

__device__ __forceinline__ void settle_inflight_copies_grouped() {
    const uint64_t start = globaltimer();
    while (globaltimer() - start < 1000000ull) __nanosleep(1000);
}

}  // namespace

template <int kGroupMode, bool kPair>
__global__ void __maxnreg__(kGroupedMaxRegisters)
    int8_gemm_grouped_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                             const GroupedArgs args) {
    using L = GroupedLayout<kPair>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + L::kStages * kGroupedAStage;
    GroupedSmem &S = *reinterpret_cast<GroupedSmem *>(smem + L::kStages * (kGroupedAStage + L::kBStage));

    const uint32_t rank = kPair ? cluster_ctarank() : 0u;
    const bool leader = rank == 0;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // "pair": this tile's owner -- a CTA pair, or a single CTA.
    const int pair = kPair ? blockIdx.x >> 1 : blockIdx.x;
    const int num_pairs = kPair ? gridDim.x >> 1 : gridDim.x;
    const int num_n = (args.n + kGroupedBN - 1) / kGroupedBN;
    const int num_m = (args.m + L::kTileM - 1) / L::kTileM;
    const int num_tiles = num_m * num_n;
    const int nk = args.k / kGroupK;
    const int my_tiles = pair < num_tiles ? (num_tiles - 1 - pair) / num_pairs + 1 : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < L::kStages; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], 1);
        }
        if constexpr (kPair) {
            for (int b = 0; b < kGroupedBuffers / 2; ++b) {
                mbar_init(&S.acc_empty[b], 2 * kGroupedEpilogueWarps + 1);
                mbar_init(&S.acc_local[b], 2 * kGroupedEpilogueWarps);
            }
        } else {
            for (int b = 0; b < kGroupedBuffers; ++b) mbar_init(&S.acc_free[b], kGroupedEpilogueWarps);
        }
        for (int r = 0; r < kGroupedScaleSlots; ++r) {
            mbar_init(&S.sc_full[r], 1);
            mbar_init(&S.sc_empty[r], kGroupedEpilogueWarps);
        }
        mbar_init(&S.drain, 1);
        S.abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        if constexpr (kPair) {
            tmem_alloc_pair(&S.tmem_base, kGroupedTmemCols);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(&S.tmem_base, kGroupedTmemCols);
            tmem_relinquish();
        }
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_b);
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (kPair) cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = S.tmem_base;
    const GroupedAbort ab{&S.abort_flag, kPair ? mapa_shared(smem_u32(&S.abort_flag), rank ^ 1u) : 0u, args.err};
    volatile int *abort_flag = &S.abort_flag;

    if (warp == 0) {
        // ------------------------------------------------------------------ producer
        if (lane == 0) {
            const uint32_t leader_full0 = kPair ? mapa_shared(smem_u32(&S.full[0]), 0u) : 0u;
            uint32_t j = 0;  // group steps of this pair, over all its tiles
            bool ok = true;
            for (int t = pair; t < num_tiles && ok; t += num_pairs) {
                const int m_tile = t / num_n;
                const int n0 = (t - m_tile * num_n) * kGroupedBN;
                const int m0 = m_tile * L::kTileM + static_cast<int>(rank) * kBM;
                const int w0 = n0 + static_cast<int>(rank) * (kGroupedBN / 2);  // rank 0 for a single CTA
                const uint32_t sc_bytes = static_cast<uint32_t>(min(kGroupedBN, args.n - n0)) * 4u;
                for (int kb = 0; kb < nk; ++kb, ++j) {
                    const uint32_t s = j % L::kStages;
                    const uint32_t ph = (j / L::kStages) & 1u;
                    const uint32_t r = j % kGroupedScaleSlots;
                    const uint32_t rph = (j / kGroupedScaleSlots) & 1u;
                    if (!ab.wait(&S.sc_empty[r], rph ^ 1u, kErrTimeoutEmpty)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&S.sc_full[r], sc_bytes);
                    bulk_load(&S.scale_ring[r][0], args.w_scale_gn + static_cast<int64_t>(kb) * args.n + n0, sc_bytes,
                              &S.sc_full[r]);
                    if (!ab.wait(&S.empty[s], ph ^ 1u, kErrTimeoutEmpty)) {
                        ok = false;
                        break;
                    }
                    if constexpr (kPair) {
                        if (leader) mbar_arrive_expect_tx(&S.full[s], 2 * (kGroupedAStage + L::kBStage));
                        const uint32_t leader_full = leader_full0 + s * static_cast<uint32_t>(sizeof(uint64_t));
                        tma_load_2d_pair(sA + s * kGroupedAStage, &tmap_a, kb * kGroupK, m0, leader_full);
                        tma_load_2d_pair(sB + s * L::kBStage, &tmap_b, kb * kGroupK, w0, leader_full);
                    } else {
                        mbar_arrive_expect_tx(&S.full[s], kGroupedAStage + L::kBStage);
                        tma_load_2d(sA + s * kGroupedAStage, &tmap_a, kb * kGroupK, m0, &S.full[s]);
                        tma_load_2d(sB + s * L::kBStage, &tmap_b, kb * kGroupK, w0, &S.full[s]);
                    }
                }
            }
            if (!ok || *abort_flag) settle_inflight_copies_grouped();
        }
    } else if (warp == 1) {
        if (leader) {
            // -------------------------------------------------------------- MMA issuer
            if (lane == 0) {
                constexpr uint32_t idesc = idesc_i8(L::kTileM, kGroupedBN);
                uint32_t j = 0;
                bool ok = true;
                for (int t = pair; t < num_tiles && ok; t += num_pairs) {
                    for (int kb = 0; kb < nk; ++kb, ++j) {
                        const uint32_t pb = j % kGroupedBuffers;
                        const uint32_t use = j / kGroupedBuffers;
                        // Completion `use - 1` of the buffer's release barrier: the epilogue's
                        // release of the buffer's previous group (in both CTAs of a pair; a fresh
                        // barrier passes use 0).  A pair releases buffers in pairs: the first of
                        // a pair waits for both.
                        if constexpr (kPair) {
                            if ((pb & 1u) == 0u &&
                                !ab.wait_cluster(&S.acc_empty[pb >> 1], (use & 1u) ^ 1u, kErrTimeoutAccumFree)) {
                                ok = false;
                                break;
                            }
                        } else if (!ab.wait(&S.acc_free[pb], (use & 1u) ^ 1u, kErrTimeoutAccumFree)) {
                            ok = false;
                            break;
                        }
                        const uint32_t s = j % L::kStages;
                        if (!ab.wait(&S.full[s], (j / L::kStages) & 1u, kErrTimeoutFull)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t a_addr = smem_u32(sA + s * kGroupedAStage);
                        const uint32_t b_addr = smem_u32(sB + s * L::kBStage);
                        const uint32_t d_tmem = tmem_base + pb * kGroupedBN;
#pragma unroll
                        for (int k = 0; k < kGroupK / kUmmaK; ++k) {  // the first overwrites the buffer
                            const uint64_t a_desc = smem_desc_sw128(a_addr + k * kUmmaK);
                            const uint64_t b_desc = smem_desc_sw128(b_addr + k * kUmmaK);
                            if constexpr (kPair) {
                                mma_i8_pair(d_tmem, a_desc, b_desc, idesc, k != 0 ? 1u : 0u);
                            } else {
                                mma_i8(d_tmem, a_desc, b_desc, idesc, k != 0 ? 1u : 0u);
                            }
                        }
                        // One commit per group: its arrival on empty[s] (both CTAs of a pair)
                        // frees the stage for the producer and tells the epilogue the partial
                        // is ready.
                        if constexpr (kPair) {
                            mma_commit_pair_both(&S.empty[s]);
                        } else {
                            mma_commit(&S.empty[s]);
                        }
                    }
                }
                if constexpr (kPair) {
                    mma_commit_pair_local(&S.drain);
                } else {
                    mma_commit(&S.drain);
                }
                mbar_wait(&S.drain, 0u, nullptr, args.err, kErrTimeoutDrain);
            }
        } else if (kPair && lane == 0) {
            // -------------------------------------------------------------- release forwarder
            const uint32_t leader_acc_empty0 = mapa_shared(smem_u32(&S.acc_empty[0]), 0u);
            const uint32_t releases = static_cast<uint32_t>(my_tiles) * static_cast<uint32_t>(nk);
            // Groups i and i + 1 (i even) share a buffer pair; an unpaired last group is
            // never waited for by the MMA, so it is not forwarded.
            for (uint32_t i = 0; i + 1 < releases; i += 2) {
                const uint32_t pp = (i % kGroupedBuffers) >> 1;
                if (!ab.wait(&S.acc_local[pp], (i / kGroupedBuffers) & 1u, kErrTimeoutAccumFree)) break;
                mbar_arrive_remote(leader_acc_empty0 + pp * static_cast<uint32_t>(sizeof(uint64_t)));
            }
        }
    } else {
        // ------------------------------------------------------------------ epilogue
        const int quad = warp & 3;  // TMEM lanes this warp may access
        const int col0 = ((warp - 2) >> 2) * kGroupedEpilogueCols;
        const int row = quad * 32 + lane;
        const uint32_t col_base = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(col0);
        uint64_t *release0 = !kPair ? &S.acc_free[0] : leader ? &S.acc_empty[0] : &S.acc_local[0];
        const f32x2 magic2 = pk2(kMagic, kMagic);

        bool alive = true;
        uint32_t j = 0;
        uint32_t r = 0, rph = 0;  // scale ring slot of step j and its phase parity
        for (int t = pair; t < num_tiles; t += num_pairs) {
            const int m_tile = t / num_n;
            const int n0 = (t - m_tile * num_n) * kGroupedBN;
            const int m = m_tile * L::kTileM + static_cast<int>(rank) * kBM + row;
            const bool row_ok = m < args.m;
            named_barrier(1, 32 * kGroupedEpilogueWarps);  // the previous tile's bias reads are done
            for (int c = threadIdx.x - 64; c < kGroupedBN; c += 32 * kGroupedEpilogueWarps) {
                const int n = n0 + c;
                S.col_bias[c] = (n < args.n && args.bias != nullptr) ? args.bias[n] : 0.0f;
            }
            named_barrier(1, 32 * kGroupedEpilogueWarps);
            if (!alive) {
                j += static_cast<uint32_t>(nk);
                continue;
            }

            f32x2 acc[kGroupedEpilogueCols / 2];
#pragma unroll
            for (int i = 0; i < kGroupedEpilogueCols / 2; ++i) acc[i] = pk2(0.0f, 0.0f);
            // W4A4: this row's activation scales, fetched two groups ahead.
            const float *a_row = args.a_scale + static_cast<int64_t>(row_ok ? m : 0) * nk;
            float gs0 = 0.0f, gs1 = 0.0f;
            if constexpr (kGroupMode == kGroupW4A4) {
                gs0 = row_ok ? a_row[0] : 0.0f;
                gs1 = (row_ok && nk > 1) ? a_row[1] : 0.0f;
            }
            for (int kb = 0; kb < nk; ++kb, ++j) {
                const uint32_t pb = j % kGroupedBuffers;
                float gs2 = 0.0f;
                if constexpr (kGroupMode == kGroupW4A4) gs2 = (row_ok && kb + 2 < nk) ? a_row[kb + 2] : 0.0f;
                // The group's MMAs are complete when stage j % kStages completes its phase
                // j / kStages.  The MMA runs at most kGroupedBuffers groups ahead of this
                // loop, fewer than the ring depth, so that phase is the current or the
                // previous one of the barrier and its parity identifies it.
                const bool ok = mbar_wait(&S.empty[j % L::kStages], (j / L::kStages) & 1u, abort_flag, args.err,
                                          kErrTimeoutAccum) &&
                                mbar_wait(&S.sc_full[r], rph, abort_flag, args.err, kErrTimeoutFull);
                alive = __all_sync(0xffffffffu, ok);
                if (!alive) {
                    ab.raise();
                    break;
                }
                tc_fence_after();
                // Read this warp's columns (kLoadCols per TMEM load) and release the buffer
                // once all are read, accumulating as they arrive.
                static_assert(kGroupedEpilogueCols % kLoadCols == 0, "whole TMEM loads per warp and group");
                const uint32_t sc = smem_u32(&S.scale_ring[r][col0]);
                const f32x2 g2 = pk2(gs0, gs0);  // W4A4: this row's activation scale of the group
#pragma unroll
                for (int h = 0; h < kGroupedEpilogueCols / kLoadCols; ++h) {
                    u32x2 v[kLoadCols / 2];
                    tmem_ld_32x32b_x32_pairs(col_base + pb * kGroupedBN + kLoadCols * h, v);
                    if (h == kGroupedEpilogueCols / kLoadCols - 1) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(release0 + (kPair ? pb >> 1 : pb));
                    }
#pragma unroll
                    for (int i = 0; i < kLoadCols / 4; ++i) {
                        f32x2 s01, s23;
                        lds_f32x2x2(sc + 16u * (i + h * kLoadCols / 4), s01, s23);
                        const f32x2 d0 = fsub2(to_magic_pair(v[2 * i]), magic2);
                        const f32x2 d1 = fsub2(to_magic_pair(v[2 * i + 1]), magic2);
                        f32x2 &t0 = acc[2 * i + h * kLoadCols / 2];
                        f32x2 &t1 = acc[2 * i + 1 + h * kLoadCols / 2];
                        if constexpr (kGroupMode == kGroupW4A4) {
                            t0 = ffma2(fmul2(d0, g2), s01, t0);
                            t1 = ffma2(fmul2(d1, g2), s23, t1);
                        } else {
                            t0 = ffma2(s01, d0, t0);
                            t1 = ffma2(s23, d1, t1);
                        }
                    }
                }
                if constexpr (kGroupMode == kGroupW4A4) {
                    gs0 = gs1;
                    gs1 = gs2;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.sc_empty[r]);
                if (++r == kGroupedScaleSlots) {
                    r = 0;
                    rph ^= 1u;
                }
            }
            if (!alive) continue;

            // Tile done: bias (and the per-token scale) and the bf16 store of this warp's columns.
            if (row_ok) {
                const float a_s = kGroupMode == kGroupAsymW4A8 ? args.a_scale[m] : 0.0f;
                __nv_bfloat16 *dst = static_cast<__nv_bfloat16 *>(args.out) + static_cast<int64_t>(m) * args.n + n0 + col0;
#pragma unroll
                for (int c = 0; c < kGroupedEpilogueCols / 8; ++c) {
                    uint32_t w[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        float lo, hi;
                        unpk2(acc[4 * c + i], lo, hi);
                        const float b0 = S.col_bias[col0 + 8 * c + 2 * i];
                        const float b1 = S.col_bias[col0 + 8 * c + 2 * i + 1];
                        if constexpr (kGroupMode == kGroupAsymW4A8) {
                            lo = __fmaf_rn(lo, a_s, b0);
                            hi = __fmaf_rn(hi, a_s, b1);
                        } else {
                            lo = __fadd_rn(lo, b0);
                            hi = __fadd_rn(hi, b1);
                        }
                        w[i] = pack_bf16x2(lo, hi);
                    }
                    if (n0 + col0 + 8 * c < args.n) {
                        *reinterpret_cast<uint4 *>(dst + 8 * c) = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if constexpr (kPair) cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        if constexpr (kPair) {
            tmem_dealloc_pair(tmem_base, kGroupedTmemCols);
        } else {
            tmem_dealloc(tmem_base, kGroupedTmemCols);
        }
    }
}

#define CTU_GROUPED_GEMM(mode, pair)                                                                      \
    template __global__ void int8_gemm_grouped_kernel<mode, pair>(const __grid_constant__ CUtensorMap,  \
                                                                  const __grid_constant__ CUtensorMap,  \
                                                                  const GroupedArgs);
CTU_GROUPED_GEMM(kGroupAsymW4A8, false)
CTU_GROUPED_GEMM(kGroupAsymW4A8, true)
CTU_GROUPED_GEMM(kGroupW4A4, false)
CTU_GROUPED_GEMM(kGroupW4A4, true)
#undef CTU_GROUPED_GEMM

}  // namespace gemm
}  // namespace ctu
