// Packed signed int4 -> int8 widening pass.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace ctu {
namespace w4 {

// out[i] = sign-extended nibble i of packed (even index in the low nibble) for
// items * 32 values.
__global__ void unpack_s4_kernel(const int8_t *packed, int8_t *out, int64_t items);

}  // namespace w4
}  // namespace ctu
