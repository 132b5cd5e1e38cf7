// Host-side helpers shared by the C ABI translation units (not exported).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace ctu {
namespace host {

struct DeviceQuery {
    int device = 0;
    int num_sms = 0;
    int smem_optin = 0;
};

// Record a message for ctu_last_error() and return `code`.
int fail(int code, const char *fmt, ...);
int cuda_fail(cudaError_t e, const char *what);
bool aligned16(const void *p);

// Current device's SM count and shared-memory limit; rejects anything but sm_100.
// Performs no allocation.
int device_query(DeviceQuery *q);

// Validated launches of the two kernels with an explicit error word.  Neither
// allocates device memory.
int run_quantize(const void *x, int64_t rows, int64_t k, int act, int bits, int8_t *codes, float *scales,
                 uint32_t *err, const DeviceQuery &q, cudaStream_t stream, const float *given_scales = nullptr,
                 bool staged_scale = false, bool half_input = false);
int run_int8_linear(const int8_t *a, const int8_t *w, const float *a_scale, const float *w_scale,
                    int64_t w_scale_count, const float *bias, void *out, int64_t m, int64_t n, int64_t k,
                    uint32_t *err, const DeviceQuery &q, cudaStream_t stream);

// Error flags recorded by the no-allocation entry point on `device` (0 when it was
// never used there).  Defined next to that entry point.
int static_scratch_error(int device, uint32_t *flags, bool clear);

}  // namespace host
}  // namespace ctu
