// Launch arguments and shared-memory budget of the fused ConvRot quantizer.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace ctu {
namespace rot {

enum Act : int { kActNone = 0, kActSwiGLU = 1, kActGelu = 2 };

constexpr int kMaxThreads = 256;   // 8 warps = 128 lane pairs = 128 groups in flight
constexpr int kMaxBoxRows = 64;    // 128-byte slices per TMA copy (8 KiB)

struct QuantArgs {
    const void *x;       // input rows (read by the warp-row kernel's bulk copies)
    int8_t *codes;       // [m, k] int8 or [m, k/2] packed int4
    float *scales;       // [m] (output; unused when given_scales is set)
    // Optional caller-supplied per-row scales (int8 only): the codes use them instead
    // of the row's own absmax, and no scale is written.
    const float *given_scales;
    uint32_t *err;       // device error word
    int m;               // rows
    int k;               // rotated width (the SwiGLU input is 2k wide)
    int rows_per_batch;  // rows per shared-memory batch
    int box_rows;        // 128-byte slices per TMA copy (a multiple of 8: 1024-byte aligned copies)
    int copies;          // TMA copies per batch; copies * box_rows >= rows_per_batch * k_in / 64
    int scale_mul;       // 1: the staged quantizers' scale (absmax * (1/qmax)); 0: absmax / qmax
    // Activation tables (act_lut_fill_kernel), set for the SwiGLU and GELU quantizers.
    const float *silu_lut;       // [65536] fp32, bf16-indexed
    const uint16_t *gelu_lut;    // [65536] bf16 bits, bf16-indexed
    const float *silu16_lut;     // [65536] fp32, fp16-indexed
    const uint16_t *gelu16_lut;  // [65536] fp16 bits, fp16-indexed
    // Per-token-per-128-column int4 scales [m, k/128] (output of the group-scale
    // quantizer; the per-row `scales` is then unused).
    float *group_scales;
};

// Fills the activation tables: launch 256 blocks of 256 threads.
__global__ void act_lut_fill_kernel(float *silu, uint16_t *gelu, float *silu16, uint16_t *gelu16);

// Slices (128 bytes = 64 bf16) per TMA copy and copies per batch.  Every copy
// starts on a 1024-byte boundary, as the 128-byte swizzle pattern requires.
inline void quant_copy_plan(int rows, int k, int act, int *box_rows, int *copies) {
    const long long k_in = act == kActSwiGLU ? 2LL * k : k;
    const long long slices = rows * k_in / 64;
    const long long box = slices >= kMaxBoxRows ? kMaxBoxRows : ((slices + 7) / 8) * 8;
    *box_rows = static_cast<int>(box);
    *copies = static_cast<int>((slices + box - 1) / box);
}

// Dynamic shared memory for a batch of `rows` rows.
inline size_t quant_smem_bytes(int rows, int k, int act, int bits) {
    int box = 0, copies = 0;
    quant_copy_plan(rows, k, act, &box, &copies);
    const size_t k_out = bits == 4 ? k / 2 : k;
    const size_t in_bytes = static_cast<size_t>(box) * copies * 128;
    const size_t code_bytes = (static_cast<size_t>(rows) * k_out + 15) & ~size_t(15);
    return 1024 + 2 * in_bytes + code_bytes + 16 * static_cast<size_t>(rows) + 64;
}

// kHalf: fp16 rows (the staged quantizers' other input type); instantiated for the
// SwiGLU and GELU activations only.
template <int Act, int Bits, bool kHalf = false>
__global__ void convrot_quant_kernel(const __grid_constant__ CUtensorMap tmap_x, const QuantArgs args);

// Register-resident variant: one lane pair per 256-column group and whole rows per
// batch, so a row may have at most kRegMaxGroups groups (a CTA of at most
// kRegMaxThreads threads).
constexpr int kRegMaxThreads = 256;
constexpr int kRegMaxGroups = kRegMaxThreads / 2;

// Dynamic shared memory of the register-resident variant for a batch of `rows` rows:
// one input buffer, two slots of per-row absmax and NaN flags, one mbarrier.
inline size_t quant_reg_smem_bytes(int rows, int k, int act) {
    int box = 0, copies = 0;
    quant_copy_plan(rows, k, act, &box, &copies);
    const size_t in_bytes = static_cast<size_t>(box) * copies * 128;
    return 1024 + in_bytes + 16 * static_cast<size_t>(rows) + 8;
}

template <int Act, int Bits>
__global__ void convrot_quant_reg_kernel(const __grid_constant__ CUtensorMap tmap_x, const QuantArgs args);

// Four-lane variant with a shared-memory transpose between rotation stages 2 and 3:
// 8 groups per warp, whole rows per batch, at most kT4MaxThreads threads (168 registers:
// at 128 it spills).
constexpr int kT4MaxThreads = 384;

// Dynamic shared memory of the four-lane variant for a batch of `rows` rows and `warps`
// warps: input buffer, 8 KB of transpose area per warp, row statistics, one mbarrier.
inline size_t quant_t4_smem_bytes(int rows, int k, int act, int warps) {
    int box = 0, copies = 0;
    quant_copy_plan(rows, k, act, &box, &copies);
    const size_t in_bytes = static_cast<size_t>(box) * copies * 128;
    return 1024 + in_bytes + 8192 * static_cast<size_t>(warps) + 16 * static_cast<size_t>(rows) + 8;
}

template <int Act, int Bits>
__global__ void convrot_quant_t4_kernel(const __grid_constant__ CUtensorMap tmap_x, const QuantArgs args);

// Eight-lane variant: 32 values per lane, a 1 KB shared-memory transpose per group between
// rotation stages 2 and 3, 4 groups per warp, whole rows per batch, at most kK8MaxThreads
// threads.
constexpr int kK8MaxThreads = 512;
constexpr int kK8Registers = 96;
constexpr int kK8GroupBytes = 1024;
constexpr int kK8WarpBytes = 4 * kK8GroupBytes;

// Dynamic shared memory of the eight-lane variant for a batch of `rows` rows and `warps`
// warps: input buffer, 4 KB of transpose area per warp, row statistics, one mbarrier.
inline size_t quant_k8_smem_bytes(int rows, int k, int act, int warps) {
    int box = 0, copies = 0;
    quant_copy_plan(rows, k, act, &box, &copies);
    const size_t in_bytes = static_cast<size_t>(box) * copies * 128;
    return 1024 + in_bytes + static_cast<size_t>(kK8WarpBytes) * warps + 16 * static_cast<size_t>(rows) + 8;
}

template <int Act, int Bits>
__global__ void convrot_quant_k8_kernel(const __grid_constant__ CUtensorMap tmap_x, const QuantArgs args);

// Multi-group eight-lane variant: each 8-lane team rotates G groups per batch, the batch
// input is double-buffered (one CTA barrier per batch), and plain / GELU rows run the
// rotation with the per-stage halvings folded into the quantization.
constexpr int kG8MaxThreads = 512;

// Dynamic shared memory of the multi-group variant for a batch of `rows` rows and `warps`
// warps: two input buffers, 4 KB of transpose area per warp, three slots of row
// statistics, two mbarriers.
inline size_t quant_g8_smem_bytes(int rows, int k, int act, int warps) {
    int box = 0, copies = 0;
    quant_copy_plan(rows, k, act, &box, &copies);
    const size_t in_bytes = static_cast<size_t>(box) * copies * 128;
    return 1024 + 2 * in_bytes + static_cast<size_t>(kK8WarpBytes) * warps + 24 * static_cast<size_t>(rows) + 24;
}

// Warp-row variant (plain and GELU rows of at most 4 * kW8MaxGroupsPerTeam groups): each
// warp owns whole rows -- one bulk copy of the row into its shared-memory buffer, its
// four 8-lane teams rotating kGt groups each with the halvings folded, a warp-level row
// absmax -- so no CTA barrier is ever taken; the next row's copy is issued as soon as
// the row's input has been consumed, overlapping its quantization.
constexpr int kW8MaxGroupsPerTeam = 6;
constexpr int kW8Warps = 4;

// Shared memory of one warp: its row buffer (1024-byte aligned) and 4 KB of transpose
// area; the CTA adds alignment slack and one mbarrier per warp.
inline size_t quant_w8_warp_bytes(int k) {
    return ((static_cast<size_t>(k) * 2 + 1023) & ~size_t(1023)) + static_cast<size_t>(kK8WarpBytes);
}
inline size_t quant_w8_smem_bytes(int k, int warps) {
    return 1024 + static_cast<size_t>(warps) * quant_w8_warp_bytes(k) + 8 * static_cast<size_t>(warps);
}

// kBlock128 (plain rows, int8 only): the block-128 rotation (radix-2 last stage) in the
// halved order; see ctu_convrot_quantize_b128.
template <int Act, int Bits, int kGt, bool kBlock128 = false>
__global__ void convrot_quant_w8_kernel(const __grid_constant__ CUtensorMap tmap_x, const QuantArgs args);

// kGroupScales (plain rows, int4 only): every 128 columns of a rotated row get their own
// scale (args.group_scales) and codes; no row statistics are exchanged.  kBlock128 as above.
template <int Act, int Bits, int G, bool kGroupScales = false, bool kBlock128 = false>
__global__ void convrot_quant_g8_kernel(const __grid_constant__ CUtensorMap tmap_x, const QuantArgs args);

}  // namespace rot
}  // namespace ctu
