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
};

// kModeW8A8: a int8 [m, k], w int8 [n, k]; kModeW4A8: w packed signed int4 [n, k/2];
// kModeW4A4: a and w packed signed int4 ([m, k/2], [n, k/2]).
template <int kMode>
__global__ void int8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                                 const GemmArgs args);

}  // namespace gemm
}  // namespace ctu
