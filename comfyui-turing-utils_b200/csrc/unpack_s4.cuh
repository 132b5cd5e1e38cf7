// Packed signed int4 -> int8 widening pass.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace ctu {
namespace w4 {

// out[i] = sign-extended nibble i of packed (even index in the low nibble) for
// items * 32 values.
__global__ void unpack_s4_kernel(const int8_t *packed, int8_t *out, int64_t items);

// Asymmetric uint4 weights with a uint4 zero point per 128 columns:
// out[r][c] = nibble c of row r (even column in the low nibble) - zeros[r][c / 128], as
// int8 in [-15, 15], for items * 32 values (rows of k values, k % 128 == 0).
__global__ void widen_u4_zero_kernel(const uint8_t *packed, const uint8_t *zeros, int8_t *out, int64_t items);

}  // namespace w4
}  // namespace ctu
