// Packed signed int4 -> int8 (sign-extended), for the W4 linears at long sequences: once
// the weight (and, for W4A4, the activation) is widened, the W8A8 CTA-pair GEMM runs at
// its full rate, and the widening is a streaming pass of 0.5 byte in + 1 byte out per value
// (w4a8.cu:34-72 packing: even column in the low nibble, two's complement nibbles).
#include <cuda_runtime.h>

#include <cstdint>

#include "gemm_tile.cuh"
#include "unpack_s4.cuh"

namespace ctu {
namespace w4 {

__global__ void __launch_bounds__(256) unpack_s4_kernel(const int8_t *packed, int8_t *out, int64_t items) {
    // One item = 16 packed bytes -> 32 int8 values; rows are contiguous, so the items of
    // the whole [rows, k/2] tensor are one flat range (k % 32 == 0).
    for (int64_t item = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; item < items;
         item += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const uint4 p = *reinterpret_cast<const uint4 *>(packed + item * 16);
        const uint2 w0 = gemm::unpack_s4x8(p.x), w1 = gemm::unpack_s4x8(p.y);
        const uint2 w2 = gemm::unpack_s4x8(p.z), w3 = gemm::unpack_s4x8(p.w);
        uint4 *dst = reinterpret_cast<uint4 *>(out + item * 32);
        dst[0] = make_uint4(w0.x, w0.y, w1.x, w1.y);
        dst[1] = make_uint4(w2.x, w2.y, w3.x, w3.y);
    }
}

__global__ void __launch_bounds__(256) widen_u4_zero_kernel(const uint8_t *packed, const uint8_t *zeros, int8_t *out,
                                                          int64_t items) {
    // One item = 16 packed bytes = 32 values of one row; a 128-column group is 4 items and
    // k % 128 == 0, so the flat item index / 4 is the flat [rows, k/128] zero-point index.
    for (int64_t item = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; item < items;
         item += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const uint4 p = *reinterpret_cast<const uint4 *>(packed + item * 16);
        const uint32_t z = static_cast<uint32_t>(zeros[item >> 2]) * 0x01010101u;
        const uint32_t words[4] = {p.x, p.y, p.z, p.w};
        uint32_t widened[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t even = words[i] & 0x0F0F0F0Fu;         // values 0, 2, 4, 6 of the word
            const uint32_t odd = (words[i] >> 4) & 0x0F0F0F0Fu;   // values 1, 3, 5, 7
            const uint32_t lo = __byte_perm(even, odd, 0x5140);   // values 0..3 in order
            const uint32_t hi = __byte_perm(even, odd, 0x7362);   // values 4..7
            // Bytewise (v - z) for v, z in [0, 15]: bias every byte by 128 so no borrow
            // crosses a byte, then flip the bias bit back (two's complement result).
            widened[2 * i] = ((lo | 0x80808080u) - z) ^ 0x80808080u;
            widened[2 * i + 1] = ((hi | 0x80808080u) - z) ^ 0x80808080u;
        }
        uint4 *dst = reinterpret_cast<uint4 *>(out + item * 32);
        dst[0] = make_uint4(widened[0], widened[1], widened[2], widened[3]);
        dst[1] = make_uint4(widened[4], widened[5], widened[6], widened[7]);
    }
}

}  // namespace w4
}  // namespace ctu
