// Device helpers shared by the single-CTA and CTA-pair integer GEMMs: the fused
// dequant/bias epilogue stores and the signed-int4 tile converter.
#pragma once

#include <cuda_bf16.h>

#include <cstdint>

#include "gemm_i8.cuh"
#include "ptx.cuh"

namespace ctu {
namespace gemm {

__device__ __forceinline__ void named_barrier(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// 32 columns of one row: bf16(fma(float(acc) * a_s, w_s, bias)).  The reference's
// epilogue visitor tree (w4a8.cu:474-525: activation scale, weight scale, bias add, each
// rounded to nearest) is built without -fmad=false, and nvcc contracts the weight-scale
// multiply and the bias add into one fma; its outputs match this form on every element
// (about 2 in 10^5 differ from a separately rounded multiply and add).  A null bias is
// +0.0 here as in the reference, and fma(x, w, +0) equals the rounded product.
__device__ __forceinline__ void store_chunk_bf16(__nv_bfloat16 *dst, const uint32_t (&acc)[32], float a_s,
                                                 const float *ws, const float *bs, int valid_cols) {
    uint32_t packed[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        float v0 = __fmul_rn(__int2float_rn(static_cast<int>(acc[2 * j])), a_s);
        float v1 = __fmul_rn(__int2float_rn(static_cast<int>(acc[2 * j + 1])), a_s);
        v0 = __fmaf_rn(v0, ws[2 * j], bs[2 * j]);
        v1 = __fmaf_rn(v1, ws[2 * j + 1], bs[2 * j + 1]);
        packed[j] = pack_bf16x2(v0, v1);
    }
    uint4 *d = reinterpret_cast<uint4 *>(dst);
    if (valid_cols >= 32) {
#pragma unroll
        for (int q = 0; q < 4; ++q) d[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
    } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if (8 * q < valid_cols) d[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
        }
    }
}

__device__ __forceinline__ void store_chunk_s32(int32_t *dst, const uint32_t (&acc)[32], int valid_cols) {
    uint4 *d = reinterpret_cast<uint4 *>(dst);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        if (4 * q < valid_cols) d[q] = make_uint4(acc[4 * q], acc[4 * q + 1], acc[4 * q + 2], acc[4 * q + 3]);
    }
}

// Eight signed 4-bit values (one packed word, even k in each byte's low nibble) to
// eight int8 values in k order.  A nibble's sign is bit 3 of its byte position;
// prmt's sign-replicate selectors (8..b) turn each byte's top bit into 0x00/0xff.
__device__ __forceinline__ uint2 unpack_s4x8(uint32_t w) {
    const uint32_t zero = 0;
    uint32_t se, so, lo, hi;
    // Sign masks: odd nibbles' signs are the bytes' top bits; even nibbles' signs are
    // bit 3 of each byte, moved to the top by a 4-bit shift.
    asm("prmt.b32 %0, %1, %2, 0xBA98;" : "=r"(so) : "r"(w), "r"(zero));
    asm("prmt.b32 %0, %1, %2, 0xBA98;" : "=r"(se) : "r"(w << 4), "r"(zero));
    // (nibble & 0x0f) | (sign & 0xf0) per byte.
    const uint32_t even = (w & 0x0F0F0F0Fu) | (se & 0xF0F0F0F0u);
    const uint32_t odd = ((w >> 4) & 0x0F0F0F0Fu) | (so & 0xF0F0F0F0u);
    // Interleave to k order: (e0, o0, e1, o1) and (e2, o2, e3, o3).
    asm("prmt.b32 %0, %1, %2, 0x5140;" : "=r"(lo) : "r"(even), "r"(odd));
    asm("prmt.b32 %0, %1, %2, 0x7362;" : "=r"(hi) : "r"(even), "r"(odd));
    return make_uint2(lo, hi);
}

// Sign-extend `kRows` x 64 packed bytes (ring stage `src`) into `kRows` x 128 int8
// bytes laid out as a 128-byte-swizzled TMA tile (`dst`).  Thread q of the kThreadsT
// threads taking part takes 16-byte packed chunks q, q + kThreadsT, ...: row =
// chunk / 4, chunk % 4 -> k bytes [32c, 32c + 32) = swizzled 16-byte chunks 2c and
// 2c+1 of the row.  Consecutive threads read consecutive 16-byte chunks, and each
// group of eight threads (two rows) writes eight distinct 16-byte bank groups.
template <int kRows, int kThreadsT = kConverterThreads>
__device__ __forceinline__ void convert_tile(const uint8_t *src, uint8_t *dst, int cthread) {
    static_assert((kRows * 4) % kThreadsT == 0, "converter threads must divide the tile's chunks");
#pragma unroll 4
    for (int i = 0; i < kRows * 4 / kThreadsT; ++i) {
        const int q = i * kThreadsT + cthread;
        const int row = q >> 2;
        const int c = q & 3;
        const uint4 p = *reinterpret_cast<const uint4 *>(src + row * 64 + c * 16);
        const uint2 w0 = unpack_s4x8(p.x), w1 = unpack_s4x8(p.y);
        const uint2 w2 = unpack_s4x8(p.z), w3 = unpack_s4x8(p.w);
        const uint32_t r7 = static_cast<uint32_t>(row & 7);
        *reinterpret_cast<uint4 *>(dst + row * 128 + (((2 * c) ^ r7) << 4)) = make_uint4(w0.x, w0.y, w1.x, w1.y);
        *reinterpret_cast<uint4 *>(dst + row * 128 + (((2 * c + 1) ^ r7) << 4)) = make_uint4(w2.x, w2.y, w3.x, w3.y);
    }
}

}  // namespace gemm
}  // namespace ctu
