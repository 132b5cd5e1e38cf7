// One-call ConvRot W8A8 linear for callers that cannot allocate device memory.
//
// The two-step path (ctu_convrot_quantize, then ctu_int8_linear) needs an
// intermediate buffer for the quantized activation (int8 codes plus one fp32 scale
// per token) that the caller allocates, and the library itself allocates a small
// device error word on first use.  Some callers cannot do either: code that runs
// inside a region where cudaMalloc is forbidden or would break their memory
// accounting (a pre-reserved memory pool, an allocator-less C host, work recorded
// between their own allocation phases).  This entry point keeps all of that working
// memory in one file-scope device array instead, so it never allocates.
//
// Limits and sharing rules:
//   * the array holds kCodeBytes (16 MiB) of codes, kMaxRows (65536) scales and an
//     error word; every GPU that loads libctu_b200.so keeps it until process exit;
//   * problems with m * k > 16 MiB or m > 65536 are rejected (split the rows);
//   * every call on a device uses the same array: calls that may overlap on the
//     GPU (different streams without ordering) race on it and must be serialized;
//   * the first call on each device resolves the array's address with
//     cudaGetSymbolAddress and clears the error word on the caller's stream; make
//     that first call before any stream capture.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "../../include/ctu_b200.h"
#include "host.cuh"

namespace {

constexpr size_t kCodeBytes = size_t(16) << 20;
constexpr int64_t kMaxRows = 65536;
constexpr size_t kScaleOffset = kCodeBytes;
constexpr size_t kErrOffset = kScaleOffset + kMaxRows * sizeof(float);
constexpr size_t kScratchBytes = kErrOffset + 256;
// The narrowest accepted width (256) at the row limit fills the code area exactly.
static_assert(kCodeBytes == static_cast<size_t>(kMaxRows) * 256, "code area = row limit x narrowest width");
static_assert(kScaleOffset % 256 == 0 && kErrOffset % 256 == 0, "scale and error areas start 256-byte aligned");

// Codes [m, k] int8 | scales [m] fp32 | error word.
static __device__ __align__(256) uint8_t g_static_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
uint8_t *g_scratch_ptr[kMaxDevices] = {};

// Resolve the array's device address once per device (the host-side symbol is not
// a device address).  Clears the error word on the caller's stream, so the clear is
// ordered before the kernels this call launches next on that stream (a memset on the
// legacy default stream would not be ordered against a non-blocking stream).  Must
// run with `device` current.
int setup(int device, cudaStream_t stream, uint8_t **out) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (g_scratch_ptr[device] == nullptr) {
        void *ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&ptr, g_static_scratch);
        if (e != cudaSuccess) return ctu::host::cuda_fail(e, "cudaGetSymbolAddress(static scratch)");
        const cudaError_t z =
            cudaMemsetAsync(static_cast<uint8_t *>(ptr) + kErrOffset, 0, sizeof(uint32_t), stream);
        if (z != cudaSuccess) return ctu::host::cuda_fail(z, "clearing the static-scratch error word");
        g_scratch_ptr[device] = static_cast<uint8_t *>(ptr);
    }
    *out = g_scratch_ptr[device];
    return CTU_OK;
}

}  // namespace

namespace ctu {
namespace host {

int static_scratch_error(int device, uint32_t *flags, bool clear) {
    *flags = 0;
    uint8_t *base = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_setup_mutex);
        if (device < 0 || device >= kMaxDevices) return CTU_OK;
        base = g_scratch_ptr[device];
    }
    if (base == nullptr) return CTU_OK;  // never used on this device
    int prev = 0;
    cudaError_t e = cudaGetDevice(&prev);
    if (e == cudaSuccess) e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(flags, base + kErrOffset, sizeof(uint32_t), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && clear) e = cudaMemset(base + kErrOffset, 0, sizeof(uint32_t));
    cudaSetDevice(prev);
    if (e != cudaSuccess) return cuda_fail(e, "reading the static-scratch error word");
    return CTU_OK;
}

}  // namespace host
}  // namespace ctu

extern "C" {

int ctu_convrot_w8a8_linear_static_scratch(const void *x, const int8_t *w, const float *w_scale,
                                           int64_t w_scale_count, const float *bias, void *out, int64_t m,
                                           int64_t n, int64_t k, void *stream) {
    using ctu::host::fail;
    if (m < 0 || n < 0 || k <= 0 || k % 256 != 0)
        return fail(CTU_ERR_INVALID_ARGUMENT, "ConvRot width must be positive and divisible by 256 (got %lld)",
                    static_cast<long long>(k));
    if (m == 0 || n == 0) return CTU_OK;
    if (m > kMaxRows || m * k > static_cast<int64_t>(kCodeBytes))
        return fail(CTU_ERR_INVALID_ARGUMENT,
                    "static-scratch ConvRot linear holds at most %lld rows and %lld activation bytes (m*k); "
                    "got m=%lld, k=%lld: split the rows or use ctu_convrot_quantize + ctu_int8_linear",
                    static_cast<long long>(kMaxRows), static_cast<long long>(kCodeBytes), static_cast<long long>(m),
                    static_cast<long long>(k));
    ctu::host::DeviceQuery q;
    if (int rc = ctu::host::device_query(&q)) return rc;
    if (q.device < 0 || q.device >= kMaxDevices) return fail(CTU_ERR_UNSUPPORTED, "device index out of range");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint8_t *base = nullptr;
    if (int rc = setup(q.device, s, &base)) return rc;
    int8_t *codes = reinterpret_cast<int8_t *>(base);
    float *scales = reinterpret_cast<float *>(base + kScaleOffset);
    uint32_t *err = reinterpret_cast<uint32_t *>(base + kErrOffset);
    // The codes and scales are rewritten in full by the quantizer on every call; the
    // error word keeps flags until ctu_get_device_error reads and clears it.
    if (int rc = ctu::host::run_quantize(x, m, k, CTU_ACT_NONE, 8, codes, scales, err, q, s)) return rc;
    return ctu::host::run_int8_linear(codes, w, scales, w_scale, w_scale_count, bias, out, m, n, k, err, q, s);
}

}  // extern "C"
