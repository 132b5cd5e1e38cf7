// Decode of the grouped-codebook W4 weight format (kitchen's AsymW4A8Int8Layout as the
// reference consumes it, kernel/csrc/turing/w4a8.cu:75-80, 216-240, 903-976) into int8
// weights for the tcgen05 W8A8 GEMM:
//
//   w[n, c] = clamp(rint(codebook[code] * s), -127, 127)
//
// code = 4-bit value of column c (even column in the low nibble), s = float8 e4m3fn
// scale of group c / group_size in row n, the product in fp32, rint ties-to-even (a NaN
// product gives 0, infinities saturate).  The decode is a streaming pass (0.5 byte +
// scale in, 1 byte out per weight); the GEMM then runs at the W8A8 rate, which a decode
// inside the GEMM's converter warps (several instructions per weight for every M tile)
// cannot match at long sequence lengths.
#include <cuda_runtime.h>

#include <cstdint>

#include "codebook.cuh"

namespace ctu {
namespace cb {

namespace {

// float8 e4m3fn -> fp32, exact: 1 sign, 4 exponent bits (bias 7), 3 mantissa bits, no
// infinities, S.1111.111 is NaN; exponent 0 encodes m * 2^-9.
__device__ __forceinline__ float e4m3fn_to_f32(uint32_t v) {
    const uint32_t sign = (v & 0x80u) << 24;
    const uint32_t e = (v >> 3) & 0xFu;
    const uint32_t m = v & 0x7u;
    if (e == 0xFu && m == 0x7u) return __uint_as_float(0x7FC00000u);
    if (e == 0u) return __uint_as_float(sign | __float_as_uint(static_cast<float>(m) * 0.001953125f));
    return __uint_as_float(sign | ((e + 120u) << 23) | (m << 20));
}

__device__ __forceinline__ uint32_t decode_byte(float value) {
    // __float2int_rn: ties to even, NaN -> 0, out-of-range saturates; then +-127.
    const int q = max(-127, min(127, __float2int_rn(value)));
    return static_cast<uint32_t>(q) & 0xFFu;
}

}  // namespace

__global__ void __launch_bounds__(256) codebook_decode_kernel(const int8_t *packed, const uint8_t *group_scale,
                                                              const float *codebook, int8_t *out, int64_t items,
                                                              int k, int group_size) {
    __shared__ float lut[16];
    if (threadIdx.x < 16) lut[threadIdx.x] = codebook[threadIdx.x];
    __syncthreads();
    const int items_per_row = k / 16;
    const int groups_per_row = k / group_size;
    for (int64_t item = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; item < items;
         item += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t row = item / items_per_row;
        const int col = static_cast<int>(item - row * items_per_row) * 16;
        const uint2 p = *reinterpret_cast<const uint2 *>(packed + row * (k / 2) + col / 2);
        const uint8_t *scales = group_scale + row * groups_per_row;
        uint32_t words[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            // group_size is a multiple of 4: the 4 columns of a word share one scale.
            const float s = e4m3fn_to_f32(scales[(col + 4 * w) / group_size]);
            const uint32_t bits = (w < 2 ? p.x : p.y) >> (16 * (w & 1));
            uint32_t word = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const uint32_t code = (bits >> (4 * e)) & 0xFu;
                word |= decode_byte(lut[code] * s) << (8 * e);
            }
            words[w] = word;
        }
        *reinterpret_cast<uint4 *>(out + row * k + col) = make_uint4(words[0], words[1], words[2], words[3]);
    }
}

}  // namespace cb
}  // namespace ctu
