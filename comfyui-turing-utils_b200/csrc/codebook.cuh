// Grouped-codebook W4 weight decode (int8 workspace for the W8A8 tensor-core GEMM).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace ctu {
namespace cb {

// out[n, c] = clamp(rint(codebook[code(n, c)] * e4m3(group_scale[n, c / group_size])), -127, 127)
// for rows [0, rows) of a packed [rows, k/2] weight; 16 columns per work item.
__global__ void codebook_decode_kernel(const int8_t *packed, const uint8_t *group_scale, const float *codebook,
                                       int8_t *out, int64_t items, int k, int group_size);

}  // namespace cb
}  // namespace ctu
