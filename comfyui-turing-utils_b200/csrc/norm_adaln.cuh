// Affine RMSNorm + segmented AdaLN and LayerNorm + AdaLN (the norm step in front of the
// quantized linears; reference: kernel/csrc/turing/segmented_rms_adaln.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace ctu {
namespace norm {

// Storage type of every floating tensor of one call (input, weight, scale, shift, output).
enum NormType : int { kNormBf16 = 0, kNormFp16 = 1, kNormFp32 = 2 };

constexpr int kRowThreads = 256;     // threads per row: fixes the reduction order
constexpr int kRmsCacheVectors = 8;  // 16-byte vectors a thread keeps in registers
constexpr int kLnSmemBytes = 48 * 1024;  // LayerNorm rows up to this size are staged in shared memory
constexpr int kLnSteps = 96;              // Welford steps a thread takes with a compile-time reciprocal
                                          // (every step of a staged row)

struct RmsArgs {
    const void *x;         // [rows, hidden]
    const void *weight;    // [hidden]
    const void *scale;     // [param_rows, *], rows scale_stride elements apart
    const void *shift;     // [param_rows, *], rows shift_stride elements apart
    const int32_t *segments;  // [segment_count, 3] = (start, stop, modulation_row)
    void *out;             // [rows, hidden]
    int64_t scale_stride;
    int64_t shift_stride;
    int rows;
    int hidden;
    int param_rows;
    int segment_count;
    float epsilon;
    int vector_store;      // 1 when `out` is 16-byte aligned (vectorized order only)
};

struct LnArgs {
    const void *x;      // [batch, sequence, hidden]
    const void *scale;  // [batch, modulation_steps, hidden]
    const void *shift;  // [batch, modulation_steps, hidden]
    void *out;          // [batch, sequence, hidden]
    int64_t rows;       // batch * sequence
    int sequence;
    int hidden;
    int modulation_steps;
    float epsilon;
    int vector_in;      // 1 when x rows may be read as 16-byte vectors (set by the launcher)
    int vector_out;     // 1 when scale / shift / out may use 16-byte vectors (set by the launcher)
    uint32_t *err;      // device error word (bounded-wait timeouts)
};

// True when the reference launch takes its 16-byte vector path
// (segmented_rms_adaln.cu:308-313; the output there is always a fresh allocation).
bool rms_vectorized(const RmsArgs &a, int type);

cudaError_t launch_segmented_rms_adaln(const RmsArgs &a, int type, cudaStream_t stream);
cudaError_t launch_layer_norm_adaln(const LnArgs &a, int type, int num_sms, cudaStream_t stream);

}  // namespace norm
}  // namespace ctu
