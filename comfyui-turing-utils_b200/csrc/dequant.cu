// int32 accumulator -> bf16 dequantization (no bias): out = bf16((float(acc) * a_s[m]) * w_s[n]).
// Replaces kernel/csrc/turing/bf16_epilogue.cu:46-217 of the reference with the same
// operation order (bf16_epilogue.cu:105-113).  HBM-bound: 4 bytes in, 2 bytes out per value.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "dequant.cuh"
#include "ptx.cuh"

namespace ctu {
namespace deq {

__global__ void __launch_bounds__(256) dequant_vec8_kernel(const int32_t *__restrict__ acc, int64_t acc_stride,
                                                           const float *__restrict__ a_scale,
                                                           const float *__restrict__ w_scale, int w_scale_count,
                                                           __nv_bfloat16 *__restrict__ out, int64_t rows, int64_t cols) {
    const int64_t vec_per_row = cols / 8;
    const int64_t total = rows * vec_per_row;
    for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < total;
         v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = v / vec_per_row;
        const int64_t c = (v - r * vec_per_row) * 8;
        const int4 q0 = __ldg(reinterpret_cast<const int4 *>(acc + r * acc_stride + c));
        const int4 q1 = __ldg(reinterpret_cast<const int4 *>(acc + r * acc_stride + c + 4));
        const float as = __ldg(a_scale + r);
        float ws[8];
        if (w_scale_count == 1) {
            const float w = __ldg(w_scale);
#pragma unroll
            for (int i = 0; i < 8; ++i) ws[i] = w;
        } else {
            const float4 w0 = __ldg(reinterpret_cast<const float4 *>(w_scale + c));
            const float4 w1 = __ldg(reinterpret_cast<const float4 *>(w_scale + c + 4));
            ws[0] = w0.x; ws[1] = w0.y; ws[2] = w0.z; ws[3] = w0.w;
            ws[4] = w1.x; ws[5] = w1.y; ws[6] = w1.z; ws[7] = w1.w;
        }
        const int qa[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        uint32_t p[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float v0 = __fmul_rn(__fmul_rn(__int2float_rn(qa[2 * i]), as), ws[2 * i]);
            const float v1 = __fmul_rn(__fmul_rn(__int2float_rn(qa[2 * i + 1]), as), ws[2 * i + 1]);
            p[i] = pack_bf16x2(v0, v1);
        }
        *reinterpret_cast<uint4 *>(out + r * cols + c) = make_uint4(p[0], p[1], p[2], p[3]);
    }
}

__global__ void __launch_bounds__(256) dequant_scalar_kernel(const int32_t *__restrict__ acc, int64_t acc_stride,
                                                             const float *__restrict__ a_scale,
                                                             const float *__restrict__ w_scale, int w_scale_count,
                                                             __nv_bfloat16 *__restrict__ out, int64_t rows,
                                                             int64_t cols) {
    const int64_t total = rows * cols;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / cols;
        const int64_t c = i - r * cols;
        const float w = w_scale[w_scale_count == 1 ? 0 : c];
        const float v = __fmul_rn(__fmul_rn(__int2float_rn(acc[r * acc_stride + c]), a_scale[r]), w);
        out[i] = __float2bfloat16_rn(v);
    }
}

}  // namespace deq
}  // namespace ctu
