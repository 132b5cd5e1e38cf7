// Tile geometry and launch arguments of the tcgen05 int8 GEMM.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace ctu {
namespace gemm {

constexpr int kBM = 128;       // tile rows (tokens)      = UMMA M
constexpr int kBN = 256;       // tile columns (channels) = UMMA N
constexpr int kBK = 128;       // K bytes per stage = one 128-byte swizzle row
constexpr int kUmmaK = 32;     // K per tcgen05.mma kind::i8
constexpr int kStages = 4;     // shared-memory ring depth
constexpr int kABytes = kBM * kBK;
constexpr int kBBytes = kBN * kBK;
constexpr int kAPackedBytes = kBM * kBK / 2;  // W4A4: two signed 4-bit activations per byte
constexpr int kBPackedBytes = kBN * kBK / 2;  // W4: two signed 4-bit weights per byte
constexpr int kTmemCols = 512; // two 256-column int32 accumulators
constexpr int kEpilogueWarps = 4;
constexpr int kEpilogueThreads = kEpilogueWarps * 32;
constexpr int kConverterThreads = 256;  // int4 modes: 8 warps that sign-extend packed tiles
constexpr int kThreads = 64 + kEpilogueThreads;
constexpr int kThreadsW4 = kThreads + kConverterThreads;
constexpr int kSmemBytes = 1024 + kStages * (kABytes + kBBytes) + 4096;
constexpr int kSmemBytesW4 = 1024 + kStages * (kABytes + kBPackedBytes) + 2 * kBBytes + 4096;
constexpr int kSmemBytesW4A4 = 1024 + kStages * (kAPackedBytes + kBPackedBytes) + 2 * (kABytes + kBBytes) + 4096;

// Operand formats: int8 x int8, int8 activations x packed signed int4 weights, packed
// signed int4 activations x packed signed int4 weights.
enum Mode : int { kModeW8A8 = 0, kModeW4A8 = 1, kModeW4A4 = 2 };

enum OutMode : int { kOutBf16 = 0, kOutS32 = 1 };

struct GemmArgs {
    const float *a_scale;   // [m]
    const float *w_scale;   // [n] or [1]
    const float *bias;      // [n] or null
    void *out;              // bf16 [m, ldc] or int32 [m, ldc]
    uint32_t *err;          // device error word
    int m, n, k;
    int ldc;
    int w_scale_count;
    int out_mode;
    int inject_timeout;           // test hook (0 in production)
    unsigned long long inject_timeout_ns;
    // CTA-pair W8A8 kernel: the last `split_tiles` 256 x 256 tiles run as two 256 x 128
    // halves each, so a last wave that would leave most pairs idle is spread over twice
    // as many work items (0: every tile whole).
    int split_tiles;
    // Fused ConvRot linear (int8_gemm_pair_kernel<kModeW8A8, kGt> with kGt > 0): the bf16
    // input rows [m, k], the int8 codes [m, k] and per-row scales [m] its quantizer warps
    // write (the A operand and `a_scale` of the GEMM), and the progress counters --
    // qsync[0] the next unclaimed row, qsync[1 + b] the finished rows of 128-row block b --
    // which must be zero at launch.
    const void *qx;
    int8_t *qcodes;
    float *qscales;
    uint32_t *qsync;
};

// kModeW8A8: a int8 [m, k], w int8 [n, k]; kModeW4A8: w packed signed int4 [n, k/2];
// kModeW4A4: a and w packed signed int4 ([m, k/2], [n, k/2]).
template <int kMode>
__global__ void int8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                                 const GemmArgs args);

// ---------------------------------------------------------------------------
// CTA-pair variant: a cluster of two CTAs computes a 256 x 256 output tile with one
// tcgen05.mma.cta_group::2 (M = 256) per K step.  Each CTA stages its 128 activation
// rows and half (128 rows) of the weight tile; the pair's tensor cores read both
// halves of the weight tile, so every weight byte crosses shared memory once per
// pair instead of once per CTA.
constexpr int kPairBM = 2 * kBM;    // output rows per CTA pair
constexpr int kHalfBN = kBN / 2;    // weight rows staged by each CTA of a pair

template <int kMode>
struct PairLayout {
    static constexpr bool kAPacked = kMode == kModeW4A4;
    static constexpr bool kBPacked = kMode != kModeW8A8;
    static constexpr bool kConvert = kAPacked || kBPacked;
    static constexpr int kAStageBytes = kAPacked ? kBM * kBK / 2 : kBM * kBK;          // TMA'd activation tile
    static constexpr int kBStageBytes = kBPacked ? kHalfBN * kBK / 2 : kHalfBN * kBK;  // TMA'd weight half-tile
    // int4 modes: every ring stage has its own sign-extended (int8, 128-byte swizzled)
    // copies, so conversion runs as far ahead of the MMA as the TMA ring does.
    static constexpr int kAuStageBytes = kAPacked ? kBM * kBK : 0;
    static constexpr int kBuStageBytes = kBPacked ? kHalfBN * kBK : 0;
    static constexpr int kStageBytes = kAStageBytes + kBStageBytes + kAuStageBytes + kBuStageBytes;
    static constexpr int kStages = kMode == kModeW8A8 ? 6 : (kMode == kModeW4A8 ? 5 : 4);
    static constexpr int kAOffset = 0;
    static constexpr int kBOffset = kAOffset + kStages * kAStageBytes;
    static constexpr int kAuOffset = kBOffset + kStages * kBStageBytes;
    static constexpr int kBuOffset = kAuOffset + kStages * kAuStageBytes;
    static constexpr int kStructOffset = kBuOffset + kStages * kBuStageBytes;
    static constexpr int kSmemBytes = 1024 + kStructOffset + 4096;
    // Converter warps: each owns one ring stage (W4A4: two per stage, one for the
    // activation tile and one for the weight half-tile).
    static constexpr int kConvWarpsPerStage = kAPacked ? 2 : 1;
    static constexpr int kConvWarps = kConvert ? kStages * kConvWarpsPerStage : 0;
    static constexpr int kThreadCount = kThreads + 32 * kConvWarps;
    static_assert(kSmemBytes <= 232448, "CTA-pair GEMM exceeds the shared memory of one SM");
};

// Fused ConvRot linear: the W8A8 pair kernel with kFusedQuantWarps more warps per CTA
// that rotate and quantize the bf16 input rows (the warp-row pipeline of the stand-alone
// quantizer; rows claimed in order from a global counter) while the tensor cores work on
// the rows already finished.  A CTA's producer loads an activation tile only once its
// 128-row block is complete.  Each quantizer warp stages one row in its own buffer of
// shared memory after the ring and the bookkeeping area: kGt = groups per team =
// ceil(k / 1024), so k <= 256 * 4 * kFusedMaxGt.
#ifndef CTU_FUSED_QUANT_WARPS
#define CTU_FUSED_QUANT_WARPS 4
#endif
#ifndef CTU_FUSED_STAGES
#define CTU_FUSED_STAGES 5
#endif
constexpr int kFusedQuantWarps = CTU_FUSED_QUANT_WARPS;
constexpr int kFusedStages = CTU_FUSED_STAGES;  // ring depth: the quantizer buffers take the rest
constexpr int kFusedMaxGt = 5;
constexpr int kFusedStructOffset =
    kFusedStages * (PairLayout<kModeW8A8>::kAStageBytes + PairLayout<kModeW8A8>::kBStageBytes);
constexpr int kFusedQuantOffset = kFusedStructOffset + 4096;
constexpr int kFusedQuantTransposeBytes = 4096;  // 1 KB per team
constexpr int kFusedThreadCount = PairLayout<kModeW8A8>::kThreadCount + 32 * kFusedQuantWarps;
__host__ __device__ inline int fused_quant_buffer_bytes(int k) { return ((2 * k + 1023) / 1024) * 1024; }
inline int fused_smem_bytes(int k) {
    return 1024 + kFusedQuantOffset + kFusedQuantWarps * (fused_quant_buffer_bytes(k) + kFusedQuantTransposeBytes);
}
static_assert(1024 + kFusedQuantOffset + kFusedQuantWarps * (2 * 256 * 4 * kFusedMaxGt + kFusedQuantTransposeBytes) <=
                  232448,
              "fused ConvRot linear exceeds the shared memory of one SM");

// `tmap_b_narrow` is the weight map with a kHalfBN / 2-row box: the per-CTA weight rows of
// a 128-column half tile (W8A8 only; the int4 modes never split tiles).  kGt > 0 (W8A8
// only): the fused ConvRot linear above.
template <int kMode, int kGt = 0>
__global__ void int8_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a,
                                      const __grid_constant__ CUtensorMap tmap_b,
                                      const __grid_constant__ CUtensorMap tmap_b_narrow, const GemmArgs args);

// ---------------------------------------------------------------------------
// Per-group (128 along K) linears: every 128-column group of K has its own weight scale
// (and, for W4A4, its own activation scale per token), so each group's int32 partial is
// converted and scaled on its own.  One ring stage is one group; four 128-column TMEM
// buffers hold the partials of four consecutive groups, so the MMA runs up to four groups
// ahead of the epilogue.  Two tilings: a single CTA per 128 x 128 output tile
// (cta_group::1, each buffer released by its own epilogue warps), or a CTA pair per
// 256 x 128 tile (cta_group::2, buffers freed in pairs through the peer's relay).
//
//   kGroupAsymW4A8: t += w_scale[g][n] * float(acc_g);  out = bf16(fma(t, a_scale[m], bias[n]))
//   kGroupW4A4:     t += (float(acc_g) * a_scale[m][g]) * w_scale[g][n];  out = bf16(t + bias[n])
//
// (each += one fused multiply-add, groups in order).  The operands are int8: the
// asymmetric uint4 weights arrive widened to (nibble - zero), the int4 activations
// sign-extended.
enum GroupMode : int { kGroupAsymW4A8 = 0, kGroupW4A4 = 1 };

constexpr int kGroupK = kBK;           // K columns per group = one ring stage
constexpr int kGroupedBN = 128;        // output columns per tile
constexpr int kGroupedBuffers = 4;     // TMEM partial buffers of kGroupedBN columns
constexpr int kGroupedScaleSlots = 12; // weight-scale ring (one group's kGroupedBN scales per slot)
#ifndef CTU_GROUPED_EPILOGUE_WARPS
#define CTU_GROUPED_EPILOGUE_WARPS 16
#endif
// Epilogue warps per CTA: 4 per TMEM lane quadrant, 32 columns each, so every scheduler
// has four of them to hide the latency of the per-group convert-and-accumulate chains.
constexpr int kGroupedEpilogueWarps = CTU_GROUPED_EPILOGUE_WARPS;
constexpr int kGroupedEpilogueCols = kGroupedBN / (kGroupedEpilogueWarps / 4);
constexpr int kGroupedThreads = 64 + 32 * kGroupedEpilogueWarps;
// A warp's registers come from its scheduler's quarter of the register file (16384), and
// the busiest scheduler holds ceil(warps / 4) warps (18 warps: 5, so 96 registers a thread).
constexpr int kGroupedMaxRegisters = (16384 / (((kGroupedThreads / 32 + 3) / 4) * 32)) / 8 * 8;
constexpr int kGroupedAStage = kBM * kGroupK;  // 16 KB: 128 activation rows of one group
constexpr int kGroupedBookkeepingBytes = 12288;

// Per-tiling layout: output rows per tile, ring depth and weight rows staged per CTA.
template <bool kPair>
struct GroupedLayout {
    static constexpr int kTileM = kPair ? kPairBM : kBM;
    static constexpr int kBStage = (kPair ? kGroupedBN / 2 : kGroupedBN) * kGroupK;  // 8 KB (half each) or 16 KB
    static constexpr int kStages = kPair ? 8 : 6;
    static constexpr int kSmemBytes = 1024 + kStages * (kGroupedAStage + kBStage) + kGroupedBookkeepingBytes;
    static_assert(kSmemBytes <= 232448, "grouped GEMM exceeds the shared memory of one SM");
};
constexpr int kGroupedMaxStages = 8;

struct GroupedArgs {
    const float *a_scale;     // kGroupAsymW4A8: [m]; kGroupW4A4: [m, k / 128]
    const float *w_scale_gn;  // [k / 128, n] fp32, group-major
    const float *bias;        // [n] or null
    void *out;                // bf16 [m, n]
    uint32_t *err;            // device error word
    int m, n, k;
};

// a int8 [m, k], w int8 [n, k] (tensor maps with a 128 x 128 box for A and a
// (kGroupedBN or kGroupedBN / 2) x 128 box for B, 128-byte swizzle).  kPair: launched as
// clusters of two CTAs; otherwise one CTA per SM.  kGroupedThreads threads per CTA.
template <int kGroupMode, bool kPair>
__global__ void int8_gemm_grouped_kernel(const __grid_constant__ CUtensorMap tmap_a,
                                         const __grid_constant__ CUtensorMap tmap_b, const GroupedArgs args);

}  // namespace gemm
}  // namespace ctu
