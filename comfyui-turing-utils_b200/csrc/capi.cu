// C ABI of libctu_b200.so (declared in include/ctu_b200.h): argument checks,
// TMA tensor-map encoding, launch geometry and the per-device error word.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <tuple>
#include <atomic>
#include <mutex>
#include <string>

#include "../../include/ctu_b200.h"
#include "codebook.cuh"
#include "convrot_quant.cuh"
#include "dequant.cuh"
#include "gemm_i8.cuh"
#include "host.cuh"
#include "norm_adaln.cuh"
#include "unpack_s4.cuh"
#include "ptx.cuh"

namespace ctu {
namespace host {

thread_local std::string g_last_error;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char *what) {
    return fail(CTU_ERR_CUDA, "CUDA error in %s: %s", what, cudaGetErrorString(e));
}

#define CTU_CUDA(call)                                  \
    do {                                                \
        cudaError_t e_ = (call);                        \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call); \
    } while (0)

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int device_query(DeviceQuery *q) {
    CTU_CUDA(cudaGetDevice(&q->device));
    int major = 0, minor = 0;
    CTU_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, q->device));
    CTU_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, q->device));
    if (major != 10 || minor != 0) {
        return fail(CTU_ERR_UNSUPPORTED, "libctu_b200 targets sm_100a (B200); device %d is sm_%d%d", q->device, major,
                    minor);
    }
    CTU_CUDA(cudaDeviceGetAttribute(&q->num_sms, cudaDevAttrMultiProcessorCount, q->device));
    CTU_CUDA(cudaDeviceGetAttribute(&q->smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, q->device));
    return CTU_OK;
}

// ---------------------------------------------------------------------------- device state
constexpr int kMaxDevices = 64;
std::mutex g_mutex;
uint32_t *g_err_word[kMaxDevices] = {};
int g_num_sms[kMaxDevices] = {};
int g_smem_optin[kMaxDevices] = {};

struct DeviceInfo {
    int device;
    uint32_t *err;
    int num_sms;
    int smem_optin;
};

int device_info(DeviceInfo *info) {
    int dev = 0;
    CTU_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(CTU_ERR_UNSUPPORTED, "device index %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_mutex);
    if (g_err_word[dev] == nullptr) {
        cudaDeviceProp prop;
        CTU_CUDA(cudaGetDeviceProperties(&prop, dev));
        if (prop.major != 10 || prop.minor != 0) {
            return fail(CTU_ERR_UNSUPPORTED, "libctu_b200 targets sm_100a (B200); device %d is sm_%d%d", dev,
                        prop.major, prop.minor);
        }
        uint32_t *w = nullptr;
        CTU_CUDA(cudaMalloc(&w, sizeof(uint32_t)));
        CTU_CUDA(cudaMemset(w, 0, sizeof(uint32_t)));
        g_err_word[dev] = w;
        g_num_sms[dev] = prop.multiProcessorCount;
        g_smem_optin[dev] = static_cast<int>(prop.sharedMemPerBlockOptin);
    }
    info->device = dev;
    info->err = g_err_word[dev];
    info->num_sms = g_num_sms[dev];
    info->smem_optin = g_smem_optin[dev];
    return CTU_OK;
}

// ---------------------------------------------------------------------------- tensor maps
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int get_encoder(EncodeTiledFn *out) {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    static cudaError_t status = cudaSuccess;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        status = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
        if (status == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    if (fn == nullptr) return fail(CTU_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    *out = fn;
    return CTU_OK;
}

// 2D row-major tensor [outer, inner] of `elem_bytes`-byte elements, 128-byte swizzle.
int encode_2d(CUtensorMap *map, CUtensorMapDataType type, int elem_bytes, const void *base, uint64_t inner,
              uint64_t outer, uint32_t box_inner, uint32_t box_outer,
              CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
    EncodeTiledFn enc;
    if (int rc = get_encoder(&enc)) return rc;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {inner * static_cast<uint64_t>(elem_bytes)};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(map, type, 2, const_cast<void *>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(CTU_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return CTU_OK;
}

// ---------------------------------------------------------------------------- quantizer geometry
enum QuantKind : int { kQuantTwoPass = 0, kQuantReg = 1, kQuantT4 = 2, kQuantK8 = 3, kQuantG8 = 4, kQuantW8 = 5 };

struct QuantPlan {
    int kind;  // QuantKind
    int rows_per_batch;
    int warps;
    int box_rows;
    int copies;
    size_t smem;
    int groups_per_team = 1;  // kQuantG8: groups each 8-lane team rotates per batch
};

// Registers a thread of the multi-group eight-lane kernel uses, by groups per team
// (ptxas, no spills).
constexpr int kG8Registers[3] = {100, 128, 128};

// Which ConvRot quantizer runs: 0 chooses per width, 1 forces the two-pass kernel,
// 2 the register-resident (two lanes per group) kernel, 3 the four-lane and 4 the
// eight-lane transpose kernel, 5 the multi-group eight-lane kernel (groups per team
// chosen per width), 6 / 7 that kernel with 1 / 2 groups per team, 8 the warp-row
// kernel, where the width allows them (test hook ctu_debug_set_quant_kernel).
std::atomic<int> g_quant_kernel{0};

// Whole-row plans: W warps hold `per_warp` x W groups, i.e. floor(per_warp W / groups)
// rows; an SM holds floor(max_warps / W) such CTAs (register-limited) when their shared
// memory fits.  The plan maximises the share of the SM's lane slots holding a group.
bool plan_quant_rows(int64_t k, int act, int smem_optin, int kind, QuantPlan *plan, int g8_groups = 1) {
    const int groups = static_cast<int>(k / 256);
    const int per_warp = kind == kQuantG8 ? 4 * g8_groups : kind == kQuantK8 ? 4 : (kind == kQuantT4 ? 8 : 16);
    const int max_threads = kind == kQuantG8   ? ctu::rot::kG8MaxThreads
                            : kind == kQuantK8 ? ctu::rot::kK8MaxThreads
                            : kind == kQuantT4 ? ctu::rot::kT4MaxThreads
                                               : ctu::rot::kRegMaxThreads;
    // Warps per SM at 96 / 168 / 255 registers a thread (multi-group: per groups per team).
    const int max_warps = kind == kQuantG8   ? 65536 / (kG8Registers[g8_groups - 1] * 32)
                          : kind == kQuantK8 ? 65536 / (ctu::rot::kK8Registers * 32)
                                             : (kind == kQuantT4 ? 12 : 8);
    if (groups > per_warp * max_threads / 32) return false;
    double best = -1.0;
    for (int w = 1; w <= max_threads / 32; ++w) {
        const int b = per_warp * w / groups;
        if (b < 1) continue;
        const size_t smem = kind == kQuantG8   ? ctu::rot::quant_g8_smem_bytes(b, static_cast<int>(k), act, w)
                            : kind == kQuantK8 ? ctu::rot::quant_k8_smem_bytes(b, static_cast<int>(k), act, w)
                            : kind == kQuantT4 ? ctu::rot::quant_t4_smem_bytes(b, static_cast<int>(k), act, w)
                                               : ctu::rot::quant_reg_smem_bytes(b, static_cast<int>(k), act);
        if (smem > static_cast<size_t>(smem_optin)) continue;
        const int ctas = std::min(max_warps / w, static_cast<int>((228 * 1024) / (smem + 1024)));
        if (ctas < 1) continue;
        const double score = static_cast<double>(b * groups) / (per_warp * w) * (ctas * w) / max_warps;
        if (score > best + 1e-9) {
            best = score;
            plan->rows_per_batch = b;
            plan->warps = w;
            plan->smem = smem;
        }
    }
    if (best < 0.0) return false;
    plan->kind = kind;
    plan->groups_per_team = kind == kQuantG8 ? g8_groups : 1;
    ctu::rot::quant_copy_plan(plan->rows_per_batch, static_cast<int>(k), act, &plan->box_rows, &plan->copies);
    return true;
}

// Warp-row plan: plain and GELU rows of at most 4 * kW8MaxGroupsPerTeam groups whose
// per-warp buffers fit (kW8Warps rows per CTA and batch).
bool plan_quant_w8(int64_t k, int act, int smem_optin, QuantPlan *plan) {
    const int groups = static_cast<int>(k / 256);
    if (act == CTU_ACT_SWIGLU || groups > 4 * ctu::rot::kW8MaxGroupsPerTeam) return false;
    const size_t smem = ctu::rot::quant_w8_smem_bytes(static_cast<int>(k), ctu::rot::kW8Warps);
    if (smem > static_cast<size_t>(smem_optin)) return false;
    plan->kind = kQuantW8;
    plan->warps = ctu::rot::kW8Warps;
    plan->rows_per_batch = ctu::rot::kW8Warps;
    plan->smem = smem;
    plan->groups_per_team = (groups + 3) / 4;
    plan->box_rows = 8;
    plan->copies = 1;
    return true;
}

int plan_quant(int64_t k, int act, int bits, int smem_optin, QuantPlan *plan, bool two_pass_only = false) {
    const int forced = two_pass_only ? 1 : g_quant_kernel.load(std::memory_order_relaxed);
    // Measured on B200 (M = 32760, activations from the tables, int8 and int4, plain and
    // fused): the eight-lane kernel is fastest at K = 5120 (20 groups: one row per 5-warp
    // CTA, 20 warps per SM; 2-11 % ahead), the four-lane kernel at K <= 4096 and K = 8192
    // (5-11 % ahead), the two-lane kernel at K = 13824 (9-13 % ahead of the others).
    const bool prefer_k8 = k > 4096 && k <= 6144;
    const bool prefer_t4 = k <= 8192;
    // The multi-group eight-lane kernel for plain and GELU rows (whose rotation folds the
    // halvings): one group per team up to 24 groups a row, two beyond.  Measured at
    // M = 32760: K = 5120 164 us against 197 us for the eight-lane kernel, K = 13824
    // 498 us against 573 us for the two-lane kernel (GELU 648 against 838 us).
    const int g8_default = k / 256 <= 24 ? 1 : 2;
    const bool prefer_g8 = act != CTU_ACT_SWIGLU && k > 4096;
    // The warp-row kernel for plain and GELU rows of 4096 < K <= 6144: no CTA barrier and
    // 21 % fewer instructions than the multi-group kernel, at 12 instead of 20 warps per
    // SM.  Measured at M = 32760, K = 5120: 137.2 us (statistics per lane, one warp
    // reduction per row) against 145.4 us back to back.
    const bool prefer_w8 = act != CTU_ACT_SWIGLU && k > 4096 && k <= 6144;
    if ((forced == 8 || (forced == 0 && prefer_w8)) && plan_quant_w8(k, act, smem_optin, plan)) return CTU_OK;
    if ((forced >= 5 && forced <= 7) || (forced == 0 && prefer_g8)) {
        const int g8_groups = forced == 6 ? 1 : forced == 7 ? 2 : g8_default;
        if (plan_quant_rows(k, act, smem_optin, kQuantG8, plan, g8_groups)) return CTU_OK;
    }
    if ((forced == 4 || (forced == 0 && prefer_k8)) && plan_quant_rows(k, act, smem_optin, kQuantK8, plan))
        return CTU_OK;
    if ((forced == 3 || (forced == 0 && prefer_t4)) && plan_quant_rows(k, act, smem_optin, kQuantT4, plan))
        return CTU_OK;
    if (forced != 1 && plan_quant_rows(k, act, smem_optin, kQuantReg, plan)) return CTU_OK;
    plan->kind = kQuantTwoPass;
    const int groups = static_cast<int>(k / 256);
    const int64_t k_in = act == CTU_ACT_SWIGLU ? 2 * k : k;
    // Rows per batch: keep every lane pair busy (a warp owns 16 groups), at most 4
    // warps per CTA so two CTAs share an SM, and the double-buffered batch in budget.
    const size_t budget = std::min<size_t>(static_cast<size_t>(smem_optin), 110 * 1024);
    double best_util = -1.0;
    int best_b = 0;
    for (int b = 1; b <= 16; ++b) {
        const int tasks = b * groups;
        const int warps = (tasks + 15) / 16;
        if (warps > 4 && b > 1) break;
        if (ctu::rot::quant_smem_bytes(b, static_cast<int>(k), act, bits) > budget && b > 1) break;
        const double util = static_cast<double>(tasks) / (16.0 * warps);
        if (util > best_util + 1e-9) {
            best_util = util;
            best_b = b;
        }
    }
    if (best_b == 0) best_b = 1;
    plan->rows_per_batch = best_b;
    plan->warps = std::min(8, (best_b * groups + 15) / 16);
    plan->smem = ctu::rot::quant_smem_bytes(best_b, static_cast<int>(k), act, bits);
    if (plan->smem > static_cast<size_t>(smem_optin)) {
        return fail(CTU_ERR_UNSUPPORTED, "ConvRot width %lld needs %zu bytes of shared memory (limit %d)",
                    static_cast<long long>(k), plan->smem, smem_optin);
    }
    ctu::rot::quant_copy_plan(best_b, static_cast<int>(k), act, &plan->box_rows, &plan->copies);
    (void)k_in;
    return CTU_OK;
}

// Per (kernel, device, block, shared memory): CTAs per SM.  Filled on first use, so
// repeated calls of one shape launch without runtime queries (and the first call of a
// shape should come before any stream capture).
std::map<std::tuple<const void *, int, int, size_t>, int> g_quant_occupancy;

using QuantKernel = void (*)(const CUtensorMap, const ctu::rot::QuantArgs);

int launch_quant_kernel(QuantKernel kernel, const CUtensorMap &map, const ctu::rot::QuantArgs &args,
                        const QuantPlan &plan, const DeviceQuery &q, cudaStream_t stream) {
    const int threads = plan.warps * 32;
    const auto key = std::make_tuple(reinterpret_cast<const void *>(kernel), q.device, threads, plan.smem);
    int per_sm = 0;
    {
        std::lock_guard<std::mutex> lock(g_mutex);
        auto it = g_quant_occupancy.find(key);
        if (it != g_quant_occupancy.end()) per_sm = it->second;
    }
    if (per_sm == 0) {
        CTU_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, q.smem_optin));
        CTU_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, plan.smem));
        if (per_sm < 1) return fail(CTU_ERR_UNSUPPORTED, "ConvRot quantizer does not fit on an SM");
        std::lock_guard<std::mutex> lock(g_mutex);
        g_quant_occupancy[key] = per_sm;
    }
    const int64_t batches = (args.m + plan.rows_per_batch - 1) / plan.rows_per_batch;
    const int grid = static_cast<int>(std::min<int64_t>(batches, static_cast<int64_t>(q.num_sms) * per_sm));
    kernel<<<grid, threads, plan.smem, stream>>>(map, args);
    CTU_CUDA(cudaGetLastError());
    return CTU_OK;
}

template <int Act, int Bits>
QuantKernel w8_kernel(int groups_per_team) {
    if constexpr (Act == ctu::rot::kActSwiGLU) {
        return nullptr;
    } else {
        switch (groups_per_team) {
        case 1: return ctu::rot::convrot_quant_w8_kernel<Act, Bits, 1>;
        case 2: return ctu::rot::convrot_quant_w8_kernel<Act, Bits, 2>;
        case 3: return ctu::rot::convrot_quant_w8_kernel<Act, Bits, 3>;
        case 4: return ctu::rot::convrot_quant_w8_kernel<Act, Bits, 4>;
        case 5: return ctu::rot::convrot_quant_w8_kernel<Act, Bits, 5>;
        case 6: return ctu::rot::convrot_quant_w8_kernel<Act, Bits, 6>;
        default: return nullptr;
        }
    }
}

template <int Act, int Bits>
int launch_quant(const CUtensorMap &map, const ctu::rot::QuantArgs &args, const QuantPlan &plan,
                 const DeviceQuery &q, cudaStream_t stream) {
    if (plan.kind == kQuantW8) {
        const QuantKernel kernel = w8_kernel<Act, Bits>(plan.groups_per_team);
        if (kernel == nullptr) return fail(CTU_ERR_UNSUPPORTED, "no warp-row quantizer for this activation and width");
        return launch_quant_kernel(kernel, map, args, plan, q, stream);
    }
    const QuantKernel kernel =
        plan.kind == kQuantG8    ? (plan.groups_per_team == 2 ? ctu::rot::convrot_quant_g8_kernel<Act, Bits, 2>
                                                              : ctu::rot::convrot_quant_g8_kernel<Act, Bits, 1>)
        : plan.kind == kQuantK8  ? ctu::rot::convrot_quant_k8_kernel<Act, Bits>
        : plan.kind == kQuantT4  ? ctu::rot::convrot_quant_t4_kernel<Act, Bits>
        : plan.kind == kQuantReg ? ctu::rot::convrot_quant_reg_kernel<Act, Bits>
                                 : ctu::rot::convrot_quant_kernel<Act, Bits>;
    return launch_quant_kernel(kernel, map, args, plan, q, stream);
}

// ---------------------------------------------------------------------------- GEMM launch
// Which GEMM kernel runs: 0 chooses per problem, 1 forces the single-CTA kernel,
// 2 forces the CTA-pair kernel (test hook ctu_debug_set_gemm_kernel).
std::atomic<int> g_gemm_kernel{0};

// Clusters of two CTAs that can be resident at once, per device and kernel variant.
int g_pair_clusters[kMaxDevices][3] = {};

// Tiles of the CTA-pair W8A8 kernel that run as two 128-column halves.  With P pairs
// resident, T tiles take ceil(T / P) rounds; when the last round holds r = T mod P
// tiles and 2 r <= P, splitting those r tiles into 2 r halves lets the last round take
// half as long (e.g. a 4095-row shard at N = 5120: 320 tiles on 74 pairs, 4.5 rounds
// instead of 5).  A test hook can force a split count (ctu_debug_set_gemm_split).
std::atomic<int> g_gemm_split{-1};

int64_t split_tail_tiles(int64_t tiles, int64_t pairs, bool allowed) {
    if (!allowed || pairs <= 0) return 0;
    const int forced = g_gemm_split.load(std::memory_order_relaxed);
    if (forced >= 0) return std::min<int64_t>(forced, tiles);
    const int64_t rem = tiles % pairs;
    return (rem != 0 && 2 * rem <= pairs) ? rem : 0;
}

template <int kMode, bool kPair>
int launch_gemm_t(const int8_t *a, const int8_t *w, const ctu::gemm::GemmArgs &args, int device, int num_sms,
                  cudaStream_t stream) {
    using ctu::gemm::kBK;
    using ctu::gemm::kBM;
    using ctu::gemm::kBN;
    constexpr bool a_packed = kMode == ctu::gemm::kModeW4A4;
    constexpr bool w_packed = kMode != ctu::gemm::kModeW8A8;
    // The pair kernel stages half of the weight tile in each CTA of the pair.
    constexpr uint32_t w_box_rows = kPair ? ctu::gemm::kHalfBN : kBN;
    // Packed int4 tiles are read by the converter warps with plain loads (no swizzle);
    // int8 tiles feed the MMA directly (128-byte swizzle).
    CUtensorMap map_a, map_b, map_b_narrow;
    if (int rc = encode_2d(&map_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a, a_packed ? args.k / 2 : args.k, args.m,
                           a_packed ? kBK / 2 : kBK, kBM,
                           a_packed ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B))
        return rc;
    if (int rc = encode_2d(&map_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w, w_packed ? args.k / 2 : args.k, args.n,
                           w_packed ? kBK / 2 : kBK, w_box_rows,
                           w_packed ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B))
        return rc;
    if constexpr (kPair && !w_packed) {
        // Half tiles (256 x 128) stage kHalfBN / 2 weight rows per CTA.
        if (int rc = encode_2d(&map_b_narrow, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w, args.k, args.n, kBK,
                               ctu::gemm::kHalfBN / 2, CU_TENSOR_MAP_SWIZZLE_128B))
            return rc;
    } else {
        map_b_narrow = map_b;
    }
    using PL = ctu::gemm::PairLayout<kMode>;
    constexpr int smem = kPair                                ? PL::kSmemBytes
                         : kMode == ctu::gemm::kModeW8A8     ? ctu::gemm::kSmemBytes
                         : kMode == ctu::gemm::kModeW4A8     ? ctu::gemm::kSmemBytesW4
                                                             : ctu::gemm::kSmemBytesW4A4;
    constexpr int threads = kPair ? PL::kThreadCount
                                  : (kMode == ctu::gemm::kModeW8A8 ? ctu::gemm::kThreads : ctu::gemm::kThreadsW4);
    constexpr auto single_kernel = ctu::gemm::int8_gemm_kernel<kMode>;
    constexpr auto pair_kernel = ctu::gemm::int8_gemm_pair_kernel<kMode>;
    // Function attributes belong to a device's context: set once per device.
    static bool attr_set[kMaxDevices] = {};
    bool need_attr = false;
    {
        std::lock_guard<std::mutex> lock(g_mutex);
        need_attr = !attr_set[device];
    }
    if (need_attr) {
        if constexpr (kPair) {
            CTU_CUDA(cudaFuncSetAttribute(pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        } else {
            CTU_CUDA(cudaFuncSetAttribute(single_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        }
        std::lock_guard<std::mutex> lock(g_mutex);
        attr_set[device] = true;
    }
    if constexpr (!kPair) {
        constexpr auto kernel = single_kernel;
        const int64_t tiles = ((args.m + kBM - 1) / kBM) * static_cast<int64_t>((args.n + kBN - 1) / kBN);
        const int grid = static_cast<int>(std::min<int64_t>(tiles, num_sms));
        kernel<<<grid, threads, smem, stream>>>(map_a, map_b, args);
        CTU_CUDA(cudaGetLastError());
        return CTU_OK;
    } else {
        constexpr auto kernel = pair_kernel;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cudaLaunchConfig_t cfg{};
        cfg.blockDim = dim3(threads, 1, 1);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = stream;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int clusters = 0;
        {
            std::lock_guard<std::mutex> lock(g_mutex);
            clusters = g_pair_clusters[device][kMode];
        }
        if (clusters == 0) {
            cfg.gridDim = dim3(2 * (num_sms / 2), 1, 1);
            CTU_CUDA(cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg));
            if (clusters <= 0) return fail(CTU_ERR_UNSUPPORTED, "no CTA pair of the GEMM fits on device %d", device);
            std::lock_guard<std::mutex> lock(g_mutex);
            g_pair_clusters[device][kMode] = clusters;
        }
        const int64_t tiles =
            ((args.m + ctu::gemm::kPairBM - 1) / ctu::gemm::kPairBM) * static_cast<int64_t>((args.n + kBN - 1) / kBN);
        ctu::gemm::GemmArgs run = args;
        run.split_tiles = static_cast<int>(split_tail_tiles(tiles, clusters, !w_packed));
        const int64_t work = tiles + run.split_tiles;
        cfg.gridDim = dim3(2 * static_cast<unsigned>(std::min<int64_t>(work, clusters)), 1, 1);
        CTU_CUDA(cudaLaunchKernelEx(&cfg, kernel, map_a, map_b, map_b_narrow, run));
        return CTU_OK;
    }
}

// The pair kernel halves the shared-memory traffic of the weight tile per SM; below
// one pair tile of rows it would leave half of every pair idle.
bool use_pair_kernel(const ctu::gemm::GemmArgs &args) {
    const int forced = g_gemm_kernel.load(std::memory_order_relaxed);
    if (forced == 1) return false;
    if (forced == 2) return true;
    return args.m > ctu::gemm::kBM;
}

template <int kMode>
int launch_gemm_mode(const int8_t *a, const int8_t *w, const ctu::gemm::GemmArgs &args, int device, int num_sms,
                     cudaStream_t stream) {
    return use_pair_kernel(args) ? launch_gemm_t<kMode, true>(a, w, args, device, num_sms, stream)
                                 : launch_gemm_t<kMode, false>(a, w, args, device, num_sms, stream);
}

int launch_gemm(const int8_t *a, const int8_t *w, const ctu::gemm::GemmArgs &args, int device, int num_sms,
                cudaStream_t stream, int mode = ctu::gemm::kModeW8A8) {
    switch (mode) {
    case ctu::gemm::kModeW4A8:
        return launch_gemm_mode<ctu::gemm::kModeW4A8>(a, w, args, device, num_sms, stream);
    case ctu::gemm::kModeW4A4:
        return launch_gemm_mode<ctu::gemm::kModeW4A4>(a, w, args, device, num_sms, stream);
    default:
        return launch_gemm_mode<ctu::gemm::kModeW8A8>(a, w, args, device, num_sms, stream);
    }
}

int check_gemm_shapes(const int8_t *a, const int8_t *w, const void *out, int64_t m, int64_t n, int64_t k) {
    if (m < 0 || n < 0 || k < 0) return fail(CTU_ERR_INVALID_ARGUMENT, "GEMM dimensions must be non-negative");
    if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX)
        return fail(CTU_ERR_INVALID_ARGUMENT, "GEMM dimensions exceed the kernel range");
    if (k % 16 != 0 || n % 8 != 0)
        return fail(CTU_ERR_INVALID_ARGUMENT, "INT8 linear requires K%%16=0 and N%%8=0 (got K=%lld, N=%lld)",
                    static_cast<long long>(k), static_cast<long long>(n));
    if (m == 0 || n == 0) return CTU_OK;
    if (!a || !w || !out) return fail(CTU_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (!aligned16(a) || !aligned16(w) || !aligned16(out))
        return fail(CTU_ERR_INVALID_ARGUMENT, "activation, weight and output must be 16-byte aligned");
    return CTU_OK;
}

int check_quantize_args(const void *x, int64_t rows, int64_t k, int act, int bits, const int8_t *codes,
                        const float *scales) {
    if (rows < 0 || k <= 0 || k % 256 != 0)
        return fail(CTU_ERR_INVALID_ARGUMENT, "ConvRot width must be positive and divisible by 256 (got %lld)",
                    static_cast<long long>(k));
    if (bits != 8 && bits != 4) return fail(CTU_ERR_INVALID_ARGUMENT, "bits must be 8 or 4");
    if (act != CTU_ACT_NONE && act != CTU_ACT_SWIGLU && act != CTU_ACT_GELU_TANH)
        return fail(CTU_ERR_INVALID_ARGUMENT, "unknown activation %d", act);
    if (rows > INT32_MAX || k > (1 << 20)) return fail(CTU_ERR_INVALID_ARGUMENT, "ConvRot dimensions exceed range");
    if (rows == 0) return CTU_OK;
    if (!x || !codes || !scales) return fail(CTU_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (!aligned16(x) || !aligned16(codes)) return fail(CTU_ERR_INVALID_ARGUMENT, "x and codes must be 16-byte aligned");
    return CTU_OK;
}

// Per device: the activation tables of the SwiGLU / GELU quantizers (bf16- and
// fp16-indexed, 768 KiB), filled on the first activation call on that device and kept
// until exit.  That call synchronizes its stream once, so it must not be made during
// stream capture.
struct ActTables {
    float *silu = nullptr;
    uint16_t *gelu = nullptr;
    float *silu16 = nullptr;
    uint16_t *gelu16 = nullptr;
};
ActTables g_act_tables[kMaxDevices];

int act_tables(int device, cudaStream_t stream, ActTables *out) {
    std::lock_guard<std::mutex> lock(g_mutex);
    ActTables &t = g_act_tables[device];
    if (t.silu == nullptr) {
        void *p = nullptr;
        CTU_CUDA(cudaMalloc(&p, 2 * 65536 * (sizeof(float) + sizeof(uint16_t))));
        float *f = static_cast<float *>(p);
        uint16_t *u = reinterpret_cast<uint16_t *>(f + 2 * 65536);
        ActTables fresh{f, u, f + 65536, u + 65536};
        ctu::rot::act_lut_fill_kernel<<<256, 256, 0, stream>>>(fresh.silu, fresh.gelu, fresh.silu16, fresh.gelu16);
        cudaError_t e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaStreamSynchronize(stream);  // other streams may read the tables next
        if (e != cudaSuccess) {
            cudaFree(p);
            return cuda_fail(e, "activation table fill");
        }
        t = fresh;
    }
    *out = t;
    return CTU_OK;
}

int run_quantize(const void *x, int64_t rows, int64_t k, int act, int bits, int8_t *codes, float *scales,
                 uint32_t *err, const DeviceQuery &q, cudaStream_t stream, const float *given_scales,
                 bool staged_scale, bool half_input) {
    if (int rc = check_quantize_args(x, rows, k, act, bits, codes, given_scales ? given_scales : scales)) return rc;
    if (rows == 0) return CTU_OK;
    if (half_input && act == CTU_ACT_NONE)
        return fail(CTU_ERR_UNSUPPORTED, "fp16 rows are taken by the SwiGLU / GELU staged quantizers only");
    QuantPlan plan;
    if (int rc = plan_quant(k, act, bits, q.smem_optin, &plan, half_input)) return rc;
    const int64_t k_in = act == CTU_ACT_SWIGLU ? 2 * k : k;
    CUtensorMap map;
    if (int rc = encode_2d(&map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, x, 64, static_cast<uint64_t>(rows) * k_in / 64, 64,
                           static_cast<uint32_t>(plan.box_rows)))
        return rc;
    ctu::rot::QuantArgs args{};
    args.x = x;
    args.codes = codes;
    args.scales = scales;
    args.given_scales = given_scales;
    args.err = err;
    args.m = static_cast<int>(rows);
    args.k = static_cast<int>(k);
    args.rows_per_batch = plan.rows_per_batch;
    args.box_rows = plan.box_rows;
    args.copies = plan.copies;
    args.scale_mul = staged_scale ? 1 : 0;
    if (act != CTU_ACT_NONE) {
        ActTables tables;
        if (int rc = act_tables(q.device, stream, &tables)) return rc;
        args.silu_lut = tables.silu;
        args.gelu_lut = tables.gelu;
        args.silu16_lut = tables.silu16;
        args.gelu16_lut = tables.gelu16;
    }
    if (half_input) {  // the two-pass kernel carries the fp16 variant
        using ctu::rot::convrot_quant_kernel;
        const QuantKernel kernel =
            act == CTU_ACT_SWIGLU
                ? (bits == 8 ? convrot_quant_kernel<ctu::rot::kActSwiGLU, 8, true>
                             : convrot_quant_kernel<ctu::rot::kActSwiGLU, 4, true>)
                : (bits == 8 ? convrot_quant_kernel<ctu::rot::kActGelu, 8, true>
                             : convrot_quant_kernel<ctu::rot::kActGelu, 4, true>);
        return launch_quant_kernel(kernel, map, args, plan, q, stream);
    }
    using ctu::rot::kActGelu;
    using ctu::rot::kActNone;
    using ctu::rot::kActSwiGLU;
    if (act == CTU_ACT_NONE) {
        return bits == 8 ? launch_quant<kActNone, 8>(map, args, plan, q, stream)
                         : launch_quant<kActNone, 4>(map, args, plan, q, stream);
    }
    if (act == CTU_ACT_SWIGLU) {
        return bits == 8 ? launch_quant<kActSwiGLU, 8>(map, args, plan, q, stream)
                         : launch_quant<kActSwiGLU, 4>(map, args, plan, q, stream);
    }
    return bits == 8 ? launch_quant<kActGelu, 8>(map, args, plan, q, stream)
                     : launch_quant<kActGelu, 4>(map, args, plan, q, stream);
}

// Rotation block 128 (plain int8 rows): the warp-row kernel up to 4 * kW8MaxGroupsPerTeam
// groups a row, the multi-group kernel beyond, both in their block-128 form.
int run_quantize_b128(const void *x, int64_t rows, int64_t k, int8_t *codes, float *scales, uint32_t *err,
                      const DeviceQuery &q, cudaStream_t stream) {
    if (int rc = check_quantize_args(x, rows, k, CTU_ACT_NONE, 8, codes, scales)) return rc;
    if (rows == 0) return CTU_OK;
    using ctu::rot::kActNone;
    QuantPlan plan;
    QuantKernel kernel = nullptr;
    const int groups = static_cast<int>(k / 256);
    if (groups <= 4 * ctu::rot::kW8MaxGroupsPerTeam && plan_quant_w8(k, CTU_ACT_NONE, q.smem_optin, &plan)) {
        switch (plan.groups_per_team) {
        case 1: kernel = ctu::rot::convrot_quant_w8_kernel<kActNone, 8, 1, true>; break;
        case 2: kernel = ctu::rot::convrot_quant_w8_kernel<kActNone, 8, 2, true>; break;
        case 3: kernel = ctu::rot::convrot_quant_w8_kernel<kActNone, 8, 3, true>; break;
        case 4: kernel = ctu::rot::convrot_quant_w8_kernel<kActNone, 8, 4, true>; break;
        case 5: kernel = ctu::rot::convrot_quant_w8_kernel<kActNone, 8, 5, true>; break;
        default: kernel = ctu::rot::convrot_quant_w8_kernel<kActNone, 8, 6, true>; break;
        }
    } else if (plan_quant_rows(k, CTU_ACT_NONE, q.smem_optin, kQuantG8, &plan, groups <= 24 ? 1 : 2)) {
        kernel = plan.groups_per_team == 2 ? ctu::rot::convrot_quant_g8_kernel<kActNone, 8, 2, false, true>
                                           : ctu::rot::convrot_quant_g8_kernel<kActNone, 8, 1, false, true>;
    } else {
        return fail(CTU_ERR_UNSUPPORTED, "the block-128 ConvRot quantizer takes rows of at most %d columns",
                    256 * 4 * 2 * (ctu::rot::kG8MaxThreads / 32));
    }
    CUtensorMap map;
    if (int rc = encode_2d(&map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, x, 64, static_cast<uint64_t>(rows) * k / 64, 64,
                           static_cast<uint32_t>(plan.box_rows)))
        return rc;
    ctu::rot::QuantArgs args{};
    args.x = x;
    args.codes = codes;
    args.scales = scales;
    args.err = err;
    args.m = static_cast<int>(rows);
    args.k = static_cast<int>(k);
    args.rows_per_batch = plan.rows_per_batch;
    args.box_rows = plan.box_rows;
    args.copies = plan.copies;
    return launch_quant_kernel(kernel, map, args, plan, q, stream);
}

int run_int8_linear(const int8_t *a, const int8_t *w, const float *a_scale, const float *w_scale,
                    int64_t w_scale_count, const float *bias, void *out, int64_t m, int64_t n, int64_t k,
                    uint32_t *err, const DeviceQuery &q, cudaStream_t stream) {
    if (int rc = check_gemm_shapes(a, w, out, m, n, k)) return rc;
    if (m == 0 || n == 0) return CTU_OK;
    if (!a_scale || !w_scale) return fail(CTU_ERR_INVALID_ARGUMENT, "null scale pointer");
    if (w_scale_count != 1 && w_scale_count != n)
        return fail(CTU_ERR_INVALID_ARGUMENT, "weight_scale must be scalar or contain one value per output channel");
    if (k == 0) return fail(CTU_ERR_UNSUPPORTED, "K = 0 is not supported");
    ctu::gemm::GemmArgs args{};
    args.a_scale = a_scale;
    args.w_scale = w_scale;
    args.bias = bias;
    args.out = out;
    args.err = err;
    args.m = static_cast<int>(m);
    args.n = static_cast<int>(n);
    args.k = static_cast<int>(k);
    args.ldc = static_cast<int>(n);
    args.w_scale_count = static_cast<int>(w_scale_count);
    args.out_mode = ctu::gemm::kOutBf16;
    return launch_gemm(a, w, args, q.device, q.num_sms, stream);
}

// ---------------------------------------------------------------------------- fused ConvRot linear
// Whether ctu_convrot_int8_linear runs the fused kernel: 0 chooses per problem, 1 forces
// the separate quantizer and GEMM, 2 the fused kernel wherever it applies (test hook
// ctu_debug_set_fused_linear).
std::atomic<int> g_fused_linear{0};

// Clusters of the fused kernel resident at once, per device and groups per team.
int g_fused_clusters[kMaxDevices][ctu::gemm::kFusedMaxGt + 1] = {};

// The fused kernel is the CTA-pair W8A8 GEMM with quantizer warps whose row buffers fit
// beside the ring: rows of at most 4 * kFusedMaxGt groups, more than one row tile (the
// single-CTA GEMM keeps the separate quantizer).  Per problem it runs where it measured
// faster than the quantizer and GEMM back to back on power-capped B200s: N <= 8192 and
// M >= 16384 (5120 x 5120 at 16384 and 32760 rows: 2-7 % faster).  With fewer rows the
// first row blocks' quantization delays the tensor cores (8192 rows: 3 % slower, 4095:
// 6-10 %), and at N = 13824 the quantizer's extra power lowers the clock of a GEMM that is
// already at the power cap (0-3 % slower).
bool use_fused_linear(int64_t m, int64_t n, int64_t k) {
    const int sel = g_fused_linear.load(std::memory_order_relaxed);
    if (sel == 1) return false;
    if (k > 1024 * ctu::gemm::kFusedMaxGt) return false;
    const int forced = g_gemm_kernel.load(std::memory_order_relaxed);
    if (forced == 1) return false;
    if (sel == 2) return forced == 2 || m > ctu::gemm::kBM;
    return m >= 16384 && n <= 8192;
}

template <int kGt>
int launch_fused_linear(const int8_t *w, const ctu::gemm::GemmArgs &base, int device, cudaStream_t stream) {
    using ctu::gemm::kBK;
    using ctu::gemm::kBM;
    using ctu::gemm::kBN;
    using ctu::gemm::kHalfBN;
    CUtensorMap map_a, map_b, map_b_narrow;
    if (int rc = encode_2d(&map_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, base.qcodes, base.k, base.m, kBK, kBM,
                           CU_TENSOR_MAP_SWIZZLE_128B))
        return rc;
    if (int rc = encode_2d(&map_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w, base.k, base.n, kBK, kHalfBN,
                           CU_TENSOR_MAP_SWIZZLE_128B))
        return rc;
    if (int rc = encode_2d(&map_b_narrow, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w, base.k, base.n, kBK, kHalfBN / 2,
                           CU_TENSOR_MAP_SWIZZLE_128B))
        return rc;
    constexpr auto kernel = ctu::gemm::int8_gemm_pair_kernel<ctu::gemm::kModeW8A8, kGt>;
    // The attribute covers the widest rows of this kGt, so one setting serves every k.
    constexpr int max_smem = 1024 + ctu::gemm::kFusedQuantOffset +
                             ctu::gemm::kFusedQuantWarps * (2 * 1024 * kGt + ctu::gemm::kFusedQuantTransposeBytes);
    static bool attr_set[kMaxDevices] = {};
    bool need_attr = false;
    {
        std::lock_guard<std::mutex> lock(g_mutex);
        need_attr = !attr_set[device];
    }
    if (need_attr) {
        CTU_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem));
        std::lock_guard<std::mutex> lock(g_mutex);
        attr_set[device] = true;
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg{};
    cfg.blockDim = dim3(ctu::gemm::kFusedThreadCount, 1, 1);
    cfg.dynamicSmemBytes = max_smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    {
        std::lock_guard<std::mutex> lock(g_mutex);
        clusters = g_fused_clusters[device][kGt];
    }
    if (clusters == 0) {
        DeviceInfo dev;
        if (int rc = device_info(&dev)) return rc;
        cfg.gridDim = dim3(2 * (dev.num_sms / 2), 1, 1);
        CTU_CUDA(cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg));
        if (clusters <= 0) return fail(CTU_ERR_UNSUPPORTED, "no CTA pair of the fused linear fits on device %d", device);
        std::lock_guard<std::mutex> lock(g_mutex);
        g_fused_clusters[device][kGt] = clusters;
    }
    cfg.dynamicSmemBytes = static_cast<size_t>(ctu::gemm::fused_smem_bytes(base.k));
    const int64_t tiles = ((base.m + ctu::gemm::kPairBM - 1) / ctu::gemm::kPairBM) *
                          static_cast<int64_t>((base.n + kBN - 1) / kBN);
    ctu::gemm::GemmArgs run = base;
    run.split_tiles = static_cast<int>(split_tail_tiles(tiles, clusters, true));
    const int64_t work = tiles + run.split_tiles;
    cfg.gridDim = dim3(2 * static_cast<unsigned>(std::min<int64_t>(work, clusters)), 1, 1);
    CTU_CUDA(cudaMemsetAsync(base.qsync, 0, sizeof(uint32_t) * ctu_convrot_int8_linear_sync_words(base.m), stream));
    CTU_CUDA(cudaLaunchKernelEx(&cfg, kernel, map_a, map_b, map_b_narrow, run));
    return CTU_OK;
}

// ---------------------------------------------------------------------------- per-group linears
// Tiles of the per-group GEMM resident at once (CTA pairs, or single CTAs), per device,
// mode and tiling.
int g_grouped_units[kMaxDevices][2][2] = {};

template <int kGroupMode, bool kPair>
int launch_grouped_tiling(const int8_t *a, const int8_t *w, const ctu::gemm::GroupedArgs &args, int device,
                          cudaStream_t stream) {
    using L = ctu::gemm::GroupedLayout<kPair>;
    using ctu::gemm::kGroupedBN;
    using ctu::gemm::kGroupK;
    CUtensorMap map_a, map_b;
    if (int rc = encode_2d(&map_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a, args.k, args.m, kGroupK, ctu::gemm::kBM))
        return rc;
    if (int rc = encode_2d(&map_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w, args.k, args.n, kGroupK,
                           kPair ? kGroupedBN / 2 : kGroupedBN))
        return rc;
    constexpr auto kernel = ctu::gemm::int8_gemm_grouped_kernel<kGroupMode, kPair>;
    constexpr int smem = L::kSmemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg{};
    cfg.blockDim = dim3(ctu::gemm::kGroupedThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = kPair ? 1 : 0;
    int units = 0;
    {
        std::lock_guard<std::mutex> lock(g_mutex);
        units = g_grouped_units[device][kGroupMode][kPair ? 1 : 0];
    }
    if (units == 0) {
        int num_sms = 0;
        CTU_CUDA(cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, device));
        CTU_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        if (kPair) {
            cfg.gridDim = dim3(2 * (num_sms / 2), 1, 1);
            CTU_CUDA(cudaOccupancyMaxActiveClusters(&units, kernel, &cfg));
        } else {
            int per_sm = 0;
            CTU_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, ctu::gemm::kGroupedThreads, smem));
            units = per_sm * num_sms;
        }
        if (units <= 0) return fail(CTU_ERR_UNSUPPORTED, "no CTA of the grouped GEMM fits on device %d", device);
        std::lock_guard<std::mutex> lock(g_mutex);
        g_grouped_units[device][kGroupMode][kPair ? 1 : 0] = units;
    }
    const int64_t tiles = ((args.m + L::kTileM - 1) / L::kTileM) *
                          static_cast<int64_t>((args.n + kGroupedBN - 1) / kGroupedBN);
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(tiles, units));
    cfg.gridDim = dim3(kPair ? 2 * grid : grid, 1, 1);
    CTU_CUDA(cudaLaunchKernelEx(&cfg, kernel, map_a, map_b, args));
    return CTU_OK;
}

// The per-group GEMM's tiling: single CTAs (128 x 128 tiles whose TMEM buffers return to
// the MMA through a CTA-local barrier; the default) or CTA pairs (256 x 128 tiles whose
// weight rows are staged once for both CTAs).  Bit-identical outputs; the single tiling
// measured 8-15 % faster for the asymmetric W4A8 linear and 0-10 % for W4A4 at
// M = 4096..32760, K, N in {5120, 13824}.  ctu_debug_set_gemm_kernel forces one: 1 single,
// 2 pair.
template <int kGroupMode>
int launch_grouped_gemm(const int8_t *a, const int8_t *w, const ctu::gemm::GroupedArgs &args, int device,
                        cudaStream_t stream) {
    const int forced = g_gemm_kernel.load(std::memory_order_relaxed);
    const bool pair = forced == 2;
    return pair ? launch_grouped_tiling<kGroupMode, true>(a, w, args, device, stream)
                : launch_grouped_tiling<kGroupMode, false>(a, w, args, device, stream);
}

// Shapes of the per-group linears: K a multiple of the 128-column group, N of 8 (16-byte
// rows of the bf16 output and of the fp32 scale rows' 32-byte copies).
int check_grouped_shapes(const char *name, int64_t m, int64_t n, int64_t k) {
    if (m < 0 || n < 0 || k < 0) return fail(CTU_ERR_INVALID_ARGUMENT, "%s dimensions must be non-negative", name);
    if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX)
        return fail(CTU_ERR_INVALID_ARGUMENT, "%s dimensions exceed the kernel range", name);
    if (k % 128 != 0 || n % 8 != 0)
        return fail(CTU_ERR_INVALID_ARGUMENT, "%s requires K%%128=0 and N%%8=0 (got K=%lld, N=%lld)", name,
                    static_cast<long long>(k), static_cast<long long>(n));
    if (m > 0 && n > 0 && k == 0) return fail(CTU_ERR_UNSUPPORTED, "K = 0 is not supported");
    return CTU_OK;
}

int launch_widen(bool zero_points, const void *packed, const uint8_t *zeros, int8_t *out, int64_t rows, int64_t k,
                 int num_sms, cudaStream_t stream) {
    const int64_t items = rows * (k / 32);
    if (items == 0) return CTU_OK;
    const int threads = 256;
    const int grid = static_cast<int>(std::min<int64_t>((items + threads - 1) / threads, static_cast<int64_t>(num_sms) * 8));
    if (zero_points) {
        ctu::w4::widen_u4_zero_kernel<<<grid, threads, 0, stream>>>(static_cast<const uint8_t *>(packed), zeros, out,
                                                                      items);
    } else {
        ctu::w4::unpack_s4_kernel<<<grid, threads, 0, stream>>>(static_cast<const int8_t *>(packed), out, items);
    }
    CTU_CUDA(cudaGetLastError());
    return CTU_OK;
}

}  // namespace host
}  // namespace ctu

using namespace ctu::host;

// ============================================================================ C ABI
extern "C" {

int ctu_version(void) { return (0 << 16) | (1 << 8) | 0; }

const char *ctu_last_error(void) { return g_last_error.c_str(); }

int ctu_get_device_error(int device, uint32_t *flags, int clear) {
    if (device < 0 || device >= kMaxDevices || flags == nullptr)
        return fail(CTU_ERR_INVALID_ARGUMENT, "invalid device or flags pointer");
    uint32_t *w = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_mutex);
        w = g_err_word[device];
    }
    uint32_t regular = 0;
    *flags = 0;
    uint32_t static_flags = 0;
    if (int rc = static_scratch_error(device, &static_flags, clear != 0)) return rc;
    *flags = static_flags;
    if (w == nullptr) return CTU_OK;  // no other launch on this device yet
    int prev = 0;
    CTU_CUDA(cudaGetDevice(&prev));
    CTU_CUDA(cudaSetDevice(device));
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(&regular, w, sizeof(uint32_t), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && clear) e = cudaMemset(w, 0, sizeof(uint32_t));
    cudaSetDevice(prev);
    if (e != cudaSuccess) return cuda_fail(e, "ctu_get_device_error");
    *flags |= regular;
    return CTU_OK;
}

int ctu_convrot_quantize(const void *x, int64_t rows, int64_t k, int act, int bits, int8_t *codes, float *scales,
                         void *stream) {
    if (int rc = check_quantize_args(x, rows, k, act, bits, codes, scales)) return rc;
    if (rows == 0) return CTU_OK;
    DeviceInfo dev;
    if (int rc = device_info(&dev)) return rc;
    DeviceQuery q{dev.device, dev.num_sms, dev.smem_optin};
    return run_quantize(x, rows, k, act, bits, codes, scales, dev.err, q, static_cast<cudaStream_t>(stream));
}

int ctu_convrot_quantize_b128(const void *x, int64_t rows, int64_t k, int8_t *codes, float *scales, void *stream) {
    if (int rc = check_quantize_args(x, rows, k, CTU_ACT_NONE, 8, codes, scales)) return rc;
    if (rows == 0) return CTU_OK;
    DeviceInfo dev;
    if (int rc = device_info(&dev)) return rc;
    DeviceQuery q{dev.device, dev.num_sms, dev.smem_optin};
    return run_quantize_b128(x, rows, k, codes, scales, dev.err, q, static_cast<cudaStream_t>(stream));
}

int ctu_convrot_quantize_staged(const void *x, int64_t rows, int64_t k, int act, int bits, int dtype, int8_t *codes,
                                float *scales, void *stream) {
    if (dtype != CTU_DTYPE_BF16 && dtype != CTU_DTYPE_FP16)
        return fail(CTU_ERR_INVALID_ARGUMENT, "staged ConvRot requires float16 or bfloat16 input");
    if (int rc = check_quantize_args(x, rows, k, act, bits, codes, scales)) return rc;
    if (rows == 0) return CTU_OK;
    DeviceInfo dev;
    if (int rc = device_info(&dev)) return rc;
    DeviceQuery q{dev.device, dev.num_sms, dev.smem_optin};
    return run_quantize(x, rows, k, act, bits, codes, scales, dev.err, q, static_cast<cudaStream_t>(stream), nullptr,
                        true, dtype == CTU_DTYPE_FP16);
}

int ctu_swiglu_int8_convrot_quantize_scaled(const void *x, int64_t rows, int64_t k, int dtype, const float *scales,
                                            int8_t *codes, void *stream) {
    if (dtype != CTU_DTYPE_BF16 && dtype != CTU_DTYPE_FP16)
        return fail(CTU_ERR_INVALID_ARGUMENT, "scaled SwiGLU ConvRot requires float16 or bfloat16 input");
    if (rows > 0 && scales == nullptr) return fail(CTU_ERR_INVALID_ARGUMENT, "null scale pointer");
    if (int rc = check_quantize_args(x, rows, k, CTU_ACT_SWIGLU, 8, codes, scales)) return rc;
    if (rows == 0) return CTU_OK;
    DeviceInfo dev;
    if (int rc = device_info(&dev)) return rc;
    DeviceQuery q{dev.device, dev.num_sms, dev.smem_optin};
    return run_quantize(x, rows, k, CTU_ACT_SWIGLU, 8, codes, nullptr, dev.err, q, static_cast<cudaStream_t>(stream),
                        scales, false, dtype == CTU_DTYPE_FP16);
}

int ctu_int8_linear(const int8_t *a, const int8_t *w, const float *a_scale, const float *w_scale,
                    int64_t w_scale_count, const float *bias, void *out, int64_t m, int64_t n, int64_t k,
                    void *stream) {
    if (int rc = check_gemm_shapes(a, w, out, m, n, k)) return rc;
    if (m == 0 || n == 0) return CTU_OK;
    DeviceInfo dev;
    if (int rc = device_info(&dev)) return rc;
    DeviceQuery q{dev.device, dev.num_sms, dev.smem_optin};
    return run_int8_linear(a, w, a_scale, w_scale, w_scale_count, bias, out, m, n, k, dev.err, q,
                           static_cast<cudaStream_t>(stream));
}

int64_t ctu_convrot_int8_linear_sync_words(int64_t m) { return m <= 0 ? 1 : 1 + (m + 127) / 128; }

int ctu_convrot_int8_linear(const void *x, const int8_t *w, const float *w_scale, int64_t w_scale_count,
                            const float *bias, void *out, int8_t *codes, float *scales, uint32_t *sync, int64_t m,
                            int64_t n, int64_t k, void *stream) {
    if (int rc = check_quantize_args(x, m, k, CTU_ACT_NONE, 8, codes, scales)) return rc;
    if (int rc = check_gemm_shapes(codes, w, out, m, n, k)) return rc;
    if (m == 0 || n == 0) return CTU_OK;
    if (!w_scale) return fail(CTU_ERR_INVALID_ARGUMENT, "null scale pointer");
    if (w_scale_count != 1 && w_scale_count != n)
        return fail(CTU_ERR_INVALID_ARGUMENT, "weight_scale must be scalar or contain one value per output channel");
    DeviceInfo dev;
    if (int rc = device_info(&dev)) return rc;
    DeviceQuery q{dev.device, dev.num_sms, dev.smem_optin};
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!use_fused_linear(m, n, k)) {
        if (int rc = run_quantize(x, m, k, CTU_ACT_NONE, 8, codes, scales, dev.err, q, s, nullptr, false, false))
            return rc;
        return run_int8_linear(codes, w, scales, w_scale, w_scale_count, bias, out, m, n, k, dev.err, q, s);
    }
    if (!sync || reinterpret_cast<uintptr_t>(sync) % 4 != 0)
        return fail(CTU_ERR_INVALID_ARGUMENT, "sync must be a 4-byte aligned array of ctu_convrot_int8_linear_sync_words(m) words");
    ctu::gemm::GemmArgs args{};
    args.a_scale = scales;
    args.w_scale = w_scale;
    args.bias = bias;
    args.out = out;
    args.err = dev.err;
    args.m = static_cast<int>(m);
    args.n = static_cast<int>(n);
    args.k = static_cast<int>(k);
    args.ldc = static_cast<int>(n);
    args.w_scale_count = static_cast<int>(w_scale_count);
    args.out_mode = ctu::gemm::kOutBf16;
    args.qx = x;
    args.qcodes = codes;
    args.qscales = scales;
    args.qsync = sync;
    switch ((k / 256 + 3) / 4) {
    case 1: return launch_fused_linear<1>(w, args, dev.device, s);
    case 2: return launch_fused_linear<2>(w, args, dev.device, s);
    case 3: return launch_fused_linear<3>(w, args, dev.device, s);
    case 4: return launch_fused_linear<4>(w, args, dev.device, s);
    default: return launch_fused_linear<5>(w, args, dev.device, s);
    }
}

int ctu_debug_set_fused_linear(int which) {
    if (which < 0 || which > 2) return fail(CTU_ERR_INVALID_ARGUMENT, "fused linear selector must be 0, 1 or 2");
    return g_fused_linear.exchange(which);
}

static int int4_linear(int mode, const int8_t *a, const int8_t *w_packed, const float *a_scale, const float *w_scale,
                       int64_t w_scale_count, const float *bias, void *out, int64_t m, int64_t n, int64_t k,
                       void *stream) {
    const char *name = mode == ctu::gemm::kModeW4A4 ? "W4A4" : "W4A8";
    if (m < 0 || n < 0 || k < 0) return fail(CTU_ERR_INVALID_ARGUMENT, "GEMM dimensions must be non-negative");
    if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX)
        return fail(CTU_ERR_INVALID_ARGUMENT, "GEMM dimensions exceed the kernel range");
    if (k % 32 != 0 || n % 8 != 0)
        return fail(CTU_ERR_INVALID_ARGUMENT, "%s linear requires K%%32=0 and N%%8=0 (got K=%lld, N=%lld)", name,
                    static_cast<long long>(k), static_cast<long long>(n));
    if (m == 0 || n == 0) return CTU_OK;
    if (k == 0) return fail(CTU_ERR_UNSUPPORTED, "K = 0 is not supported");
    if (!a || !w_packed || !out || !a_scale || !w_scale) return fail(CTU_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (!aligned16(a) || !aligned16(w_packed) || !aligned16(out))
        return fail(CTU_ERR_INVALID_ARGUMENT, "activation, weight and output must be 16-byte aligned");
    if (w_scale_count != 1 && w_scale_count != n)
        return fail(CTU_ERR_INVALID_ARGUMENT, "weight_scale must be scalar or contain one value per output channel");
    DeviceInfo dev;
    if (int rc = device_info(&dev)) return rc;
    ctu::gemm::GemmArgs args{};
    args.a_scale = a_scale;
    args.w_scale = w_scale;
    args.bias = bias;
    args.out = out;
    args.err = dev.err;
    args.m = static_cast<int>(m);
    args.n = static_cast<int>(n);
    args.k = static_cast<int>(k);
    args.ldc = static_cast<int>(n);
    args.w_scale_count = static_cast<int>(w_scale_count);
    args.out_mode = ctu::gemm::kOutBf16;
    return launch_gemm(a, w_packed, args, dev.device, dev.num_sms, static_cast<cudaStream_t>(stream), mode);
}

int ctu_w4a8_linear(const int8_t *a, const int8_t *w_packed, const float *a_scale, const float *w_scale,
                    int64_t w_scale_count, const float *bias, void *out, int64_t m, int64_t n, int64_t k,
                    void *stream) {
    return int4_linear(ctu::gemm::kModeW4A8, a, w_packed, a_scale, w_scale, w_scale_count, bias, out, m, n, k,
                       stream);
}

int ctu_w4a4_linear(const int8_t *a_packed, const int8_t *w_packed, const float *a_scale, const float *w_scale,
                    int64_t w_scale_count, const float *bias, void *out, int64_t m, int64_t n, int64_t k,
                    void *stream) {
    return int4_linear(ctu::gemm::kModeW4A4, a_packed, w_packed, a_scale, w_scale, w_scale_count, bias, out, m, n,
                       k, stream);
}

// ---------------------------------------------------------------- grouped-codebook W4A8
static bool codebook_group_size_ok(int64_t k, int64_t group_size) {
    // bindings.cpp:304-307
    return group_size >= 4 && k % group_size == 0 && (16 % group_size == 0 || group_size % 16 == 0);
}

static int launch_codebook_decode(const int8_t *w_packed, const uint8_t *group_scale, const float *codebook,
                                  int8_t *out, int64_t rows, int64_t k, int64_t group_size, int num_sms,
                                  cudaStream_t stream) {
    const int64_t items = rows * (k / 16);
    if (items == 0) return CTU_OK;
    const int threads = 256;
    const int grid = static_cast<int>(std::min<int64_t>((items + threads - 1) / threads, static_cast<int64_t>(num_sms) * 8));
    ctu::cb::codebook_decode_kernel<<<grid, threads, 0, stream>>>(w_packed, group_scale, codebook, out, items,
                                                                  static_cast<int>(k), static_cast<int>(group_size));
    CTU_CUDA(cudaGetLastError());
    return CTU_OK;
}

int ctu_codebook_decode_s8(const int8_t *w_packed, const uint8_t *group_scale, const float *codebook, int8_t *out,
                           int64_t rows, int64_t k, int64_t group_size, void *stream) {
    if (rows < 0 || k < 0 || rows > INT32_MAX || k > INT32_MAX)
        return fail(CTU_ERR_INVALID_ARGUMENT, "codebook decode dimensions out of range");
    if (k % 16 != 0) return fail(CTU_ERR_INVALID_ARGUMENT, "codebook decode requires K divisible by 16");
    if (!codebook_group_size_ok(k, group_size)) return fail(CTU_ERR_INVALID_ARGUMENT, "unsupported codebook group_size");
    if (rows == 0 || k == 0) return CTU_OK;
    if (!w_packed || !group_scale || !codebook || !out) return fail(CTU_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (!aligned16(w_packed) || !aligned16(out))
        return fail(CTU_ERR_INVALID_ARGUMENT, "packed weight and output must be 16-byte aligned");
    DeviceInfo dev;
    if (int rc = device_info(&dev)) return rc;
    return launch_codebook_decode(w_packed, group_scale, codebook, out, rows, k, group_size, dev.num_sms,
                                  static_cast<cudaStream_t>(stream));
}

int ctu_codebook_w4a8_linear(const int8_t *a, const int8_t *w_packed, const float *a_scale, const uint8_t *group_scale,
                             const float *channel_scale, const float *codebook, const float *bias, void *out,
                             int8_t *workspace, int64_t workspace_rows, int64_t m, int64_t n, int64_t k,
                             int64_t group_size, void *stream) {
    if (m <= 0 || n <= 0 || k <= 0) return fail(CTU_ERR_INVALID_ARGUMENT, "codebook W4A8 dimensions must be positive");
    if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX)
        return fail(CTU_ERR_INVALID_ARGUMENT, "codebook W4A8 dimensions exceed the CUDA kernel range");
    if (k % 16 != 0 || n % 8 != 0)
        return fail(CTU_ERR_INVALID_ARGUMENT, "codebook W4A8 requires K divisible by 16 and N divisible by 8");
    if (!codebook_group_size_ok(k, group_size)) return fail(CTU_ERR_INVALID_ARGUMENT, "unsupported codebook W4A8 group_size");
    if (workspace_rows <= 0 || workspace_rows % 8 != 0)
        return fail(CTU_ERR_INVALID_ARGUMENT, "codebook W4A8 needs an 8-row-aligned workspace");
    if (!a || !w_packed || !a_scale || !group_scale || !channel_scale || !codebook || !out || !workspace)
        return fail(CTU_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (!aligned16(a) || !aligned16(w_packed) || !aligned16(out) || !aligned16(workspace))
        return fail(CTU_ERR_INVALID_ARGUMENT, "activation, weight, output and workspace must be 16-byte aligned");
    DeviceInfo dev;
    if (int rc = device_info(&dev)) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t groups = k / group_size;
    // w4a8.cu:1154-1181: decode a chunk of output channels, then the W8A8 GEMM writes
    // those columns of the output (row stride n).
    for (int64_t row = 0; row < n; row += workspace_rows) {
        const int64_t rows = std::min(workspace_rows, n - row);
        if (int rc = launch_codebook_decode(w_packed + row * (k / 2), group_scale + row * groups, codebook, workspace,
                                            rows, k, group_size, dev.num_sms, s))
            return rc;
        ctu::gemm::GemmArgs args{};
        args.a_scale = a_scale;
        args.w_scale = channel_scale + row;
        args.bias = bias ? bias + row : nullptr;
        args.out = static_cast<__nv_bfloat16 *>(out) + row;
        args.err = dev.err;
        args.m = static_cast<int>(m);
        args.n = static_cast<int>(rows);
        args.k = static_cast<int>(k);
        args.ldc = static_cast<int>(n);
        args.w_scale_count = static_cast<int>(rows);
        args.out_mode = ctu::gemm::kOutBf16;
        if (int rc = launch_gemm(a, workspace, args, dev.device, dev.num_sms, s)) return rc;
    }
    return CTU_OK;
}

// ---------------------------------------------------------------- per-group W4A8 / W4A4
static int quantize_int4_g128(const void *x, int64_t rows, int64_t k, int8_t *codes, float *group_scales,
                              void *stream, bool block128) {
    if (int rc = check_quantize_args(x, rows, k, CTU_ACT_NONE, 4, codes, group_scales)) return rc;
    if (rows == 0) return CTU_OK;
    DeviceInfo dev;
    if (int rc = device_info(&dev)) return rc;
    QuantPlan plan;
    const int g8_groups = k / 256 <= 24 ? 1 : 2;
    if (!plan_quant_rows(k, CTU_ACT_NONE, dev.smem_optin, kQuantG8, &plan, g8_groups))
        return fail(CTU_ERR_UNSUPPORTED, "no per-group int4 quantizer plan for width %lld", static_cast<long long>(k));
    CUtensorMap map;
    if (int rc = encode_2d(&map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, x, 64, static_cast<uint64_t>(rows) * k / 64, 64,
                           static_cast<uint32_t>(plan.box_rows)))
        return rc;
    ctu::rot::QuantArgs args{};
    args.codes = codes;
    args.group_scales = group_scales;
    args.err = dev.err;
    args.m = static_cast<int>(rows);
    args.k = static_cast<int>(k);
    args.rows_per_batch = plan.rows_per_batch;
    args.box_rows = plan.box_rows;
    args.copies = plan.copies;
    DeviceQuery q{dev.device, dev.num_sms, dev.smem_optin};
    using ctu::rot::kActNone;
    const QuantKernel kernel =
        block128 ? (g8_groups == 2 ? ctu::rot::convrot_quant_g8_kernel<kActNone, 4, 2, true, true>
                                   : ctu::rot::convrot_quant_g8_kernel<kActNone, 4, 1, true, true>)
                 : (g8_groups == 2 ? ctu::rot::convrot_quant_g8_kernel<kActNone, 4, 2, true>
                                   : ctu::rot::convrot_quant_g8_kernel<kActNone, 4, 1, true>);
    return launch_quant_kernel(kernel, map, args, plan, q, static_cast<cudaStream_t>(stream));
}

int ctu_convrot_quantize_int4_g128(const void *x, int64_t rows, int64_t k, int8_t *codes, float *group_scales,
                                   void *stream) {
    return quantize_int4_g128(x, rows, k, codes, group_scales, stream, false);
}

int ctu_convrot_quantize_int4_g128_b128(const void *x, int64_t rows, int64_t k, int8_t *codes, float *group_scales,
                                        void *stream) {
    return quantize_int4_g128(x, rows, k, codes, group_scales, stream, true);
}

int ctu_asym_w4a8_g128_linear(const int8_t *a, const uint8_t *w_packed, const float *a_scale,
                              const float *w_scale_gn, const uint8_t *w_zero, const float *bias, void *out,
                              int8_t *w_workspace, int64_t m, int64_t n, int64_t k, void *stream) {
    if (int rc = check_grouped_shapes("asymmetric W4A8", m, n, k)) return rc;
    if (m == 0 || n == 0) return CTU_OK;
    if (!a || !w_packed || !a_scale || !w_scale_gn || !w_zero || !out || !w_workspace)
        return fail(CTU_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (!aligned16(a) || !aligned16(w_packed) || !aligned16(out) || !aligned16(w_workspace) || !aligned16(w_scale_gn))
        return fail(CTU_ERR_INVALID_ARGUMENT, "activation, weight, scales, output and workspace must be 16-byte aligned");
    DeviceInfo dev;
    if (int rc = device_info(&dev)) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (int rc = launch_widen(true, w_packed, w_zero, w_workspace, n, k, dev.num_sms, s)) return rc;
    ctu::gemm::GroupedArgs args{a_scale, w_scale_gn, bias, out, dev.err, static_cast<int>(m), static_cast<int>(n),
                                static_cast<int>(k)};
    return launch_grouped_gemm<ctu::gemm::kGroupAsymW4A8>(a, w_workspace, args, dev.device, s);
}

int ctu_w4a4_g128_linear(const int8_t *a_packed, const int8_t *w_packed, const float *a_scale_mg,
                         const float *w_scale_gn, const float *bias, void *out, int8_t *a_workspace,
                         int8_t *w_workspace, int64_t m, int64_t n, int64_t k, void *stream) {
    if (int rc = check_grouped_shapes("W4A4", m, n, k)) return rc;
    if (m == 0 || n == 0) return CTU_OK;
    if (!a_packed || !w_packed || !a_scale_mg || !w_scale_gn || !out || !a_workspace || !w_workspace)
        return fail(CTU_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (!aligned16(a_packed) || !aligned16(w_packed) || !aligned16(out) || !aligned16(a_workspace) ||
        !aligned16(w_workspace) || !aligned16(w_scale_gn))
        return fail(CTU_ERR_INVALID_ARGUMENT, "activation, weight, scales, output and workspaces must be 16-byte aligned");
    DeviceInfo dev;
    if (int rc = device_info(&dev)) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (int rc = launch_widen(false, a_packed, nullptr, a_workspace, m, k, dev.num_sms, s)) return rc;
    if (int rc = launch_widen(false, w_packed, nullptr, w_workspace, n, k, dev.num_sms, s)) return rc;
    ctu::gemm::GroupedArgs args{a_scale_mg, w_scale_gn, bias, out, dev.err, static_cast<int>(m), static_cast<int>(n),
                                static_cast<int>(k)};
    return launch_grouped_gemm<ctu::gemm::kGroupW4A4>(a_workspace, w_workspace, args, dev.device, s);
}

int ctu_int4_unpack_s8(const int8_t *packed, int8_t *out, int64_t rows, int64_t k, void *stream) {
    if (rows < 0 || k < 0) return fail(CTU_ERR_INVALID_ARGUMENT, "int4 unpack dimensions must be non-negative");
    if (k % 32 != 0) return fail(CTU_ERR_INVALID_ARGUMENT, "int4 unpack requires K divisible by 32");
    if (rows == 0 || k == 0) return CTU_OK;
    if (!packed || !out) return fail(CTU_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (!aligned16(packed) || !aligned16(out)) return fail(CTU_ERR_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
    DeviceInfo dev;
    if (int rc = device_info(&dev)) return rc;
    const int64_t items = rows * (k / 32);
    const int threads = 256;
    const int grid = static_cast<int>(std::min<int64_t>((items + threads - 1) / threads, static_cast<int64_t>(dev.num_sms) * 8));
    ctu::w4::unpack_s4_kernel<<<grid, threads, 0, static_cast<cudaStream_t>(stream)>>>(packed, out, items);
    CTU_CUDA(cudaGetLastError());
    return CTU_OK;
}

int ctu_int8_gemm_s32(const int8_t *a, const int8_t *w, int32_t *acc, int64_t ldc, int64_t m, int64_t n, int64_t k,
                      void *stream) {
    if (int rc = check_gemm_shapes(a, w, acc, m, n, k)) return rc;
    if (m == 0 || n == 0) return CTU_OK;
    if (ldc < n || ldc % 4 != 0) return fail(CTU_ERR_INVALID_ARGUMENT, "ldc must be >= N and a multiple of 4");
    if (k == 0) return fail(CTU_ERR_UNSUPPORTED, "K = 0 is not supported");
    DeviceInfo dev;
    if (int rc = device_info(&dev)) return rc;
    ctu::gemm::GemmArgs args{};
    args.out = acc;
    args.err = dev.err;
    args.m = static_cast<int>(m);
    args.n = static_cast<int>(n);
    args.k = static_cast<int>(k);
    args.ldc = static_cast<int>(ldc);
    args.w_scale_count = 1;
    args.out_mode = ctu::gemm::kOutS32;
    return launch_gemm(a, w, args, dev.device, dev.num_sms, static_cast<cudaStream_t>(stream));
}

int ctu_debug_gemm_injected_timeout(const int8_t *a, const int8_t *w, int32_t *acc, int64_t m, int64_t n, int64_t k,
                                    uint64_t timeout_ns, void *stream) {
    if (int rc = check_gemm_shapes(a, w, acc, m, n, k)) return rc;
    if (m == 0 || n == 0 || k == 0) return fail(CTU_ERR_INVALID_ARGUMENT, "empty problem");
    if (timeout_ns == 0 || timeout_ns > 5000000000ull)
        return fail(CTU_ERR_INVALID_ARGUMENT, "timeout must be in (0, 5 s]");
    DeviceInfo dev;
    if (int rc = device_info(&dev)) return rc;
    ctu::gemm::GemmArgs args{};
    args.out = acc;
    args.err = dev.err;
    args.m = static_cast<int>(m);
    args.n = static_cast<int>(n);
    args.k = static_cast<int>(k);
    args.ldc = static_cast<int>(n);
    args.w_scale_count = 1;
    args.out_mode = ctu::gemm::kOutS32;
    args.inject_timeout = 1;
    args.inject_timeout_ns = timeout_ns;
    return launch_gemm(a, w, args, dev.device, dev.num_sms, static_cast<cudaStream_t>(stream));
}

int ctu_debug_set_quant_kernel(int which) {
    if (which < 0 || which > 8) return fail(CTU_ERR_INVALID_ARGUMENT, "kernel selector must be between 0 and 8");
    return g_quant_kernel.exchange(which);
}

int ctu_debug_quant_plan(int64_t k, int act, int bits, int smem_optin, int *kind, int *warps, int *rows_per_batch) {
    if (!kind || !warps || !rows_per_batch) return fail(CTU_ERR_INVALID_ARGUMENT, "null output pointer");
    if (k <= 0 || k % 256 != 0) return fail(CTU_ERR_INVALID_ARGUMENT, "width must be a positive multiple of 256");
    if (act < CTU_ACT_NONE || act > CTU_ACT_GELU_TANH || (bits != 4 && bits != 8))
        return fail(CTU_ERR_INVALID_ARGUMENT, "invalid activation or bit width");
    QuantPlan plan{};
    if (int rc = plan_quant(k, act, bits, smem_optin, &plan)) return rc;
    *kind = plan.kind;
    *warps = plan.warps;
    *rows_per_batch = plan.rows_per_batch;
    return CTU_OK;
}

int ctu_debug_set_gemm_split(int tiles) {
    if (tiles < -1) return fail(CTU_ERR_INVALID_ARGUMENT, "split count must be -1 (automatic) or >= 0");
    return g_gemm_split.exchange(tiles);
}

int ctu_debug_set_gemm_kernel(int which) {
    if (which < 0 || which > 2) return fail(CTU_ERR_INVALID_ARGUMENT, "kernel selector must be 0, 1 or 2");
    return g_gemm_kernel.exchange(which);
}

int ctu_dequantize_int8_bf16(const int32_t *acc, int64_t acc_stride, const float *a_scale, const float *w_scale,
                             int64_t w_scale_count, void *out, int64_t rows, int64_t cols, void *stream) {
    if (rows < 0 || cols < 0 || acc_stride < cols)
        return fail(CTU_ERR_INVALID_ARGUMENT, "invalid accumulator shape or stride");
    if (rows == 0 || cols == 0) return CTU_OK;
    if (!acc || !a_scale || !w_scale || !out) return fail(CTU_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (w_scale_count != 1 && w_scale_count != cols)
        return fail(CTU_ERR_INVALID_ARGUMENT, "weight_scale must be scalar or contain one value per output column");
    DeviceInfo dev;
    if (int rc = device_info(&dev)) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool vec = cols % 8 == 0 && acc_stride % 4 == 0 && aligned16(acc) && aligned16(out) &&
                     (w_scale_count == 1 || aligned16(w_scale));
    const int threads = 256;
    if (vec) {
        const int64_t work = rows * (cols / 8);
        const int grid = static_cast<int>(std::min<int64_t>((work + threads - 1) / threads, dev.num_sms * 16));
        ctu::deq::dequant_vec8_kernel<<<grid, threads, 0, s>>>(acc, acc_stride, a_scale, w_scale,
                                                                static_cast<int>(w_scale_count),
                                                                static_cast<__nv_bfloat16 *>(out), rows, cols);
    } else {
        const int64_t work = rows * cols;
        const int grid = static_cast<int>(std::min<int64_t>((work + threads - 1) / threads, dev.num_sms * 16));
        ctu::deq::dequant_scalar_kernel<<<grid, threads, 0, s>>>(acc, acc_stride, a_scale, w_scale,
                                                                  static_cast<int>(w_scale_count),
                                                                  static_cast<__nv_bfloat16 *>(out), rows, cols);
    }
    CTU_CUDA(cudaGetLastError());
    return CTU_OK;
}

int ctu_segmented_rms_adaln(const void *x, const void *weight, const void *scale, int64_t scale_stride,
                            const void *shift, int64_t shift_stride, const int32_t *segments, int64_t segment_count,
                            void *out, int64_t rows, int64_t hidden, int64_t param_rows, float epsilon, int dtype,
                            void *stream) {
    if (dtype < CTU_DTYPE_BF16 || dtype > CTU_DTYPE_FP32)
        return fail(CTU_ERR_INVALID_ARGUMENT, "norm input must be float16, bfloat16, or float32");
    if (rows <= 0 || hidden <= 0)
        return fail(CTU_ERR_INVALID_ARGUMENT, "segmented RMSNorm+AdaLN input dimensions must be positive");
    if (param_rows <= 0) return fail(CTU_ERR_INVALID_ARGUMENT, "scale must be [modulation_rows, hidden]");
    if (segment_count <= 0) return fail(CTU_ERR_INVALID_ARGUMENT, "segments must contain at least one row");
    if (rows > INT32_MAX || hidden > INT32_MAX || param_rows > INT32_MAX || segment_count > INT32_MAX ||
        scale_stride < 0 || shift_stride < 0 || scale_stride > INT32_MAX || shift_stride > INT32_MAX)
        return fail(CTU_ERR_INVALID_ARGUMENT, "segmented RMSNorm+AdaLN dimensions exceed the CUDA kernel range");
    if (!(std::isfinite(epsilon) && epsilon > 0.0f))
        return fail(CTU_ERR_INVALID_ARGUMENT, "RMSNorm epsilon must be finite and positive");
    if (!x || !weight || !scale || !shift || !segments || !out) return fail(CTU_ERR_INVALID_ARGUMENT, "null tensor pointer");
    DeviceInfo dev;
    if (int rc = device_info(&dev)) return rc;
    ctu::norm::RmsArgs a{};
    a.x = x;
    a.weight = weight;
    a.scale = scale;
    a.shift = shift;
    a.segments = segments;
    a.out = out;
    a.scale_stride = scale_stride;
    a.shift_stride = shift_stride;
    a.rows = static_cast<int>(rows);
    a.hidden = static_cast<int>(hidden);
    a.param_rows = static_cast<int>(param_rows);
    a.segment_count = static_cast<int>(segment_count);
    a.epsilon = epsilon;
    CTU_CUDA(ctu::norm::launch_segmented_rms_adaln(a, dtype, static_cast<cudaStream_t>(stream)));
    return CTU_OK;
}

int ctu_layer_norm_adaln(const void *x, const void *scale, const void *shift, void *out, int64_t batch,
                         int64_t sequence, int64_t hidden, int64_t modulation_steps, float epsilon, int dtype,
                         void *stream) {
    if (dtype < CTU_DTYPE_BF16 || dtype > CTU_DTYPE_FP32)
        return fail(CTU_ERR_INVALID_ARGUMENT, "LayerNorm+AdaLN input must be float16, bfloat16, or float32");
    if (batch <= 0 || sequence <= 0 || hidden <= 0 || modulation_steps <= 0)
        return fail(CTU_ERR_INVALID_ARGUMENT, "LayerNorm+AdaLN dimensions must be positive");
    if (batch * sequence > INT32_MAX || sequence > INT32_MAX || hidden > INT32_MAX || modulation_steps > INT32_MAX)
        return fail(CTU_ERR_INVALID_ARGUMENT, "LayerNorm+AdaLN dimensions exceed the CUDA kernel range");
    if (!(std::isfinite(epsilon) && epsilon > 0.0f))
        return fail(CTU_ERR_INVALID_ARGUMENT, "LayerNorm epsilon must be finite and positive");
    if (!x || !scale || !shift || !out) return fail(CTU_ERR_INVALID_ARGUMENT, "null tensor pointer");
    DeviceInfo dev;
    if (int rc = device_info(&dev)) return rc;
    ctu::norm::LnArgs a{};
    a.x = x;
    a.scale = scale;
    a.shift = shift;
    a.out = out;
    a.rows = batch * sequence;
    a.sequence = static_cast<int>(sequence);
    a.hidden = static_cast<int>(hidden);
    a.modulation_steps = static_cast<int>(modulation_steps);
    a.epsilon = epsilon;
    a.err = dev.err;
    CTU_CUDA(ctu::norm::launch_layer_norm_adaln(a, dtype, dev.num_sms, static_cast<cudaStream_t>(stream)));
    return CTU_OK;
}

}  // extern "C"
