// int32 -> bf16 dequantization kernels (see dequant.cu).
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

namespace ctu {
namespace deq {

__global__ void dequant_vec8_kernel(const int32_t *__restrict__ acc, int64_t acc_stride, const float *__restrict__ a_scale,
                                    const float *__restrict__ w_scale, int w_scale_count, __nv_bfloat16 *__restrict__ out,
                                    int64_t rows, int64_t cols);
__global__ void dequant_scalar_kernel(const int32_t *__restrict__ acc, int64_t acc_stride,
                                      const float *__restrict__ a_scale, const float *__restrict__ w_scale,
                                      int w_scale_count, __nv_bfloat16 *__restrict__ out, int64_t rows, int64_t cols);

}  // namespace deq
}  // namespace ctu
