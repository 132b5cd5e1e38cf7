// Device arithmetic of the RMSNorm + segmented AdaLN step, shared by the standalone
// norm kernel and the quantizer's fused norm prologue so both give the same bits
// (reference: kernel/csrc/turing/segmented_rms_adaln.cu:114-131, 216-219).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace ctu {
namespace norm {

// The first segment (start, stop, row) whose stop exceeds `row`; -1 when the row falls
// in no segment.
__device__ __forceinline__ int find_modulation_row(const int32_t *segments, int count, int row) {
    int low = 0;
    int high = count;
    while (low < high) {
        const int mid = low + (high - low) / 2;
        if (row < segments[mid * 3 + 1]) {
            high = mid;
        } else {
            low = mid + 1;
        }
    }
    if (low >= count || row < segments[low * 3]) return -1;
    return segments[low * 3 + 2];
}

// The modulation row the reference uses: the segment's row, or row 0 when the row is
// in no segment or the segment names a row outside [0, param_rows).
__device__ __forceinline__ int modulation_row_of(const int32_t *segments, int count, int param_rows, int row) {
    const int mapped = find_modulation_row(segments, count, row);
    return mapped >= 0 && mapped < param_rows ? mapped : 0;
}

// 1 / rms from the row's sum of squares (IEEE division by the width, then epsilon).
__device__ __forceinline__ float inverse_rms(float sum_squares, int hidden, float epsilon) {
    return rsqrtf(__fadd_rn(__fdiv_rn(sum_squares, static_cast<float>(hidden)), epsilon));
}

// One output element: ((x * inv) * w) * (1 + s) + shift, the last multiply-add fused.
__device__ __forceinline__ float rms_output(float x, float inv, float w, float s, float h) {
    return __fmaf_rn(__fmul_rn(__fmul_rn(x, inv), w), __fadd_rn(1.0f, s), h);
}

// rms_output with 1 + s already formed (as the fp32 value __fadd_rn(1, s)).
__device__ __forceinline__ float rms_output_staged(float x, float inv, float w, float one_plus_s, float h) {
    return __fmaf_rn(__fmul_rn(__fmul_rn(x, inv), w), one_plus_s, h);
}

}  // namespace norm
}  // namespace ctu
