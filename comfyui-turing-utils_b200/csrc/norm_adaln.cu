// Affine RMSNorm + segmented AdaLN, and LayerNorm + Wan AdaLN, for bf16 / fp16 / fp32
// rows (reference: kernel/csrc/turing/segmented_rms_adaln.cu:133-297).
//
// Both norms are HBM-streaming: one CTA of 256 threads per row reads the row from HBM
// once with 16-byte coalesced loads (vector path) and keeps it in registers for the
// output pass; the reference reads it twice.  The thread-to-column mapping and the
// reduction tree are the reference's, because they fix the fp32 rounding of the
// statistics and so the output bits:
//   * RMS: thread t accumulates fma(v, v, s) over 16-byte vectors t, t+256, ... in
//     order (or columns t, t+256, ... when the reference launch is not vectorized);
//   * LayerNorm: thread t runs Welford over columns t, t+256, ... with IEEE division;
//   * a shfl_down tree inside each warp, then the 8 warp partials combined in order.
// Every arithmetic step is written with round-to-nearest intrinsics so that the
// compiler cannot contract or reorder it differently from the reference's build.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "norm_adaln.cuh"
#include "norm_math.cuh"
#include "ptx.cuh"

namespace ctu {
namespace norm {

namespace {

constexpr int kWarps = kRowThreads / 32;

template <typename T>
struct Elem;
template <>
struct Elem<__nv_bfloat16> {
    static __device__ __forceinline__ float load(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 store(float v) { return __float2bfloat16_rn(v); }
};
template <>
struct Elem<__half> {
    static __device__ __forceinline__ float load(__half v) { return __half2float(v); }
    static __device__ __forceinline__ __half store(float v) { return __float2half_rn(v); }
};
template <>
struct Elem<float> {
    static __device__ __forceinline__ float load(float v) { return v; }
    static __device__ __forceinline__ float store(float v) { return v; }
};

template <typename T>
struct alignas(16) Vec {
    static constexpr int kWidth = 16 / static_cast<int>(sizeof(T));
    T v[kWidth];
};

// A 32-bit word of two 16-bit storage values as an f32x2 pair (low half first) and back
// (round to nearest even, per lane as __float2bfloat16_rn / __float2half_rn).
template <typename T>
struct Words;
template <>
struct Words<__nv_bfloat16> {
    static __device__ __forceinline__ f32x2 unpack(uint32_t w) {
        return pk2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
    }
    static __device__ __forceinline__ uint32_t pack(f32x2 v) {
        float lo, hi;
        unpk2(v, lo, hi);
        return pack_bf16x2(lo, hi);
    }
};
template <>
struct Words<__half> {
    static __device__ __forceinline__ f32x2 unpack(uint32_t w) {
        __half2 h;
        __builtin_memcpy(&h, &w, 4);
        const float2 f = __half22float2(h);
        return pk2(f.x, f.y);
    }
    static __device__ __forceinline__ uint32_t pack(f32x2 v) {
        float lo, hi;
        unpk2(v, lo, hi);
        const __half2 h = __floats2half2_rn(lo, hi);
        uint32_t w;
        __builtin_memcpy(&w, &h, 4);
        return w;
    }
};

// fma(v, v, sq) over the values of one 16-byte vector, in element order.
template <typename T>
__device__ __forceinline__ float sum_squares(const uint4 v, float sq) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        if constexpr (sizeof(T) == 4) {
            const float f = __uint_as_float(w[q]);
            sq = __fmaf_rn(f, f, sq);
        } else {
            float lo, hi;
            unpk2(Words<T>::unpack(w[q]), lo, hi);
            sq = __fmaf_rn(lo, lo, sq);
            sq = __fmaf_rn(hi, hi, sq);
        }
    }
    return sq;
}

// rms_output on the values of one 16-byte vector, two values per packed instruction.
template <typename T>
__device__ __forceinline__ uint4 rms_vector(const uint4 x, const uint4 w, const uint4 s, const uint4 h, f32x2 inv2) {
    const f32x2 one2 = pk2(1.0f, 1.0f);
    auto f = [&](f32x2 xv, f32x2 wv, f32x2 sv, f32x2 hv) {
        return ffma2(fmul2(fmul2(xv, inv2), wv), fadd2(one2, sv), hv);
    };
    if constexpr (sizeof(T) == 4) {
        auto p = [](uint32_t a, uint32_t b) { return pk2(__uint_as_float(a), __uint_as_float(b)); };
        float o0, o1, o2, o3;
        unpk2(f(p(x.x, x.y), p(w.x, w.y), p(s.x, s.y), p(h.x, h.y)), o0, o1);
        unpk2(f(p(x.z, x.w), p(w.z, w.w), p(s.z, s.w), p(h.z, h.w)), o2, o3);
        return make_uint4(__float_as_uint(o0), __float_as_uint(o1), __float_as_uint(o2), __float_as_uint(o3));
    } else {
        using Wd = Words<T>;
        return make_uint4(Wd::pack(f(Wd::unpack(x.x), Wd::unpack(w.x), Wd::unpack(s.x), Wd::unpack(h.x))),
                          Wd::pack(f(Wd::unpack(x.y), Wd::unpack(w.y), Wd::unpack(s.y), Wd::unpack(h.y))),
                          Wd::pack(f(Wd::unpack(x.z), Wd::unpack(w.z), Wd::unpack(s.z), Wd::unpack(h.z))),
                          Wd::pack(f(Wd::unpack(x.w), Wd::unpack(w.w), Wd::unpack(s.w), Wd::unpack(h.w))));
    }
}

template <typename T, bool kVec, int kCache>
__global__ void __launch_bounds__(kRowThreads) segmented_rms_adaln_kernel(const RmsArgs a) {
    using E = Elem<T>;
    constexpr int W = Vec<T>::kWidth;
    __shared__ float warp_sums[kWarps];
    __shared__ int modulation_row;

    const int row = static_cast<int>(blockIdx.x);
    const int tid = static_cast<int>(threadIdx.x);
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int64_t row_off = static_cast<int64_t>(row) * a.hidden;
    const T *x = static_cast<const T *>(a.x) + row_off;

    if (tid == 0) modulation_row = modulation_row_of(a.segments, a.segment_count, a.param_rows, row);

    float sq = 0.0f;
    uint4 cache[kCache];
    float scache[kCache];
    if constexpr (kVec) {
        const int nvec = a.hidden / W;
        const uint4 *xv = reinterpret_cast<const uint4 *>(x);
#pragma unroll
        for (int i = 0; i < kCache; ++i) {
            const int j = tid + i * kRowThreads;
            if (j < nvec) {
                cache[i] = xv[j];
                sq = sum_squares<T>(cache[i], sq);
            }
        }
        for (int j = tid + kCache * kRowThreads; j < nvec; j += kRowThreads) sq = sum_squares<T>(xv[j], sq);
    } else {
#pragma unroll
        for (int i = 0; i < kCache; ++i) {
            const int c = tid + i * kRowThreads;
            if (c < a.hidden) {
                const float v = E::load(x[c]);
                scache[i] = v;
                sq = __fmaf_rn(v, v, sq);
            }
        }
        for (int c = tid + kCache * kRowThreads; c < a.hidden; c += kRowThreads) {
            const float v = E::load(x[c]);
            sq = __fmaf_rn(v, v, sq);
        }
    }

#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sq = __fadd_rn(sq, __shfl_down_sync(0xffffffffu, sq, off));
    if (lane == 0) warp_sums[warp] = sq;
    __syncthreads();
    float total = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) total = __fadd_rn(total, warp_sums[w]);
    const float inv = inverse_rms(total, a.hidden, a.epsilon);

    const int mod = modulation_row;
    const T *weight = static_cast<const T *>(a.weight);
    const T *scale = static_cast<const T *>(a.scale) + static_cast<int64_t>(mod) * a.scale_stride;
    const T *shift = static_cast<const T *>(a.shift) + static_cast<int64_t>(mod) * a.shift_stride;
    T *out = static_cast<T *>(a.out) + row_off;

    if constexpr (kVec) {
        const int nvec = a.hidden / W;
        const uint4 *wv = reinterpret_cast<const uint4 *>(weight);
        const uint4 *sv = reinterpret_cast<const uint4 *>(scale);
        const uint4 *hv = reinterpret_cast<const uint4 *>(shift);
        const f32x2 inv2 = pk2(inv, inv);
        auto emit = [&](int j, const uint4 xin) {
            const uint4 o = rms_vector<T>(xin, __ldg(wv + j), __ldg(sv + j), __ldg(hv + j), inv2);
            if (a.vector_store) {
                reinterpret_cast<uint4 *>(out)[j] = o;
            } else {
                const uint32_t ow[4] = {o.x, o.y, o.z, o.w};
                uint16_t *o16 = reinterpret_cast<uint16_t *>(out + static_cast<int64_t>(j) * W);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    o16[2 * q] = static_cast<uint16_t>(ow[q]);
                    o16[2 * q + 1] = static_cast<uint16_t>(ow[q] >> 16);
                }
            }
        };
#pragma unroll
        for (int i = 0; i < kCache; ++i) {
            const int j = tid + i * kRowThreads;
            if (j < nvec) emit(j, cache[i]);
        }
        const uint4 *xv = reinterpret_cast<const uint4 *>(x);
        for (int j = tid + kCache * kRowThreads; j < nvec; j += kRowThreads) emit(j, xv[j]);
    } else {
        auto emit = [&](int c, float v) {
            out[c] = E::store(rms_output(v, inv, E::load(weight[c]), E::load(scale[c]), E::load(shift[c])));
        };
#pragma unroll
        for (int i = 0; i < kCache; ++i) {
            const int c = tid + i * kRowThreads;
            if (c < a.hidden) emit(c, scache[i]);
        }
        for (int c = tid + kCache * kRowThreads; c < a.hidden; c += kRowThreads) emit(c, E::load(x[c]));
    }
}

// One LayerNorm output: round(round((x - mean) * inv) * round(1 + s) + h), each round to
// the storage type (segmented_rms_adaln.cu:290-296).
template <typename T>
__device__ __forceinline__ float ln_output(float x, float mean, float inv, float s, float h) {
    using E = Elem<T>;
    const float normalized = E::load(E::store(__fmul_rn(__fsub_rn(x, mean), inv)));
    const float multiplier = E::load(E::store(__fadd_rn(1.0f, s)));
    return __fmaf_rn(normalized, multiplier, h);
}

// ln_output on the values of one 16-byte vector, stored in the storage type.
template <typename T>
__device__ __forceinline__ uint4 ln_vector(const uint4 x, const uint4 s, const uint4 h, float mean, float inv) {
    using E = Elem<T>;
    if constexpr (sizeof(T) == 4) {
        auto f = [&](uint32_t xv, uint32_t sv, uint32_t hv) {
            return __float_as_uint(ln_output<T>(__uint_as_float(xv), mean, inv, __uint_as_float(sv), __uint_as_float(hv)));
        };
        return make_uint4(f(x.x, s.x, h.x), f(x.y, s.y, h.y), f(x.z, s.z, h.z), f(x.w, s.w, h.w));
    } else {
        using Wd = Words<T>;
        auto f = [&](uint32_t xw, uint32_t sw, uint32_t hw) {
            float x0, x1, s0, s1, h0, h1;
            unpk2(Wd::unpack(xw), x0, x1);
            unpk2(Wd::unpack(sw), s0, s1);
            unpk2(Wd::unpack(hw), h0, h1);
            return Wd::pack(pk2(ln_output<T>(x0, mean, inv, s0, h0), ln_output<T>(x1, mean, inv, s1, h1)));
        };
        (void)sizeof(E);
        return make_uint4(f(x.x, s.x, h.x), f(x.y, s.y, h.y), f(x.z, s.z, h.z), f(x.w, s.w, h.w));
    }
}

struct Welford {
    float mean;
    float m2;
    int count;
};

__device__ __noinline__ float ieee_div(float a, float b) { return __fdiv_rn(a, b); }

// a / count with IEEE round-to-nearest, for a positive integer count: the correction
// step of Markstein's division with rcp = RN(1 / count) -- q0 = a * rcp,
// r = fma(-q0, count, a) (exact), q = fma(r, rcp, q0) -- which equals the IEEE quotient
// for every count <= kMaxMarksteinCount and every a with 2^-96 <= |a| <= FLT_MAX (checked
// over every significand by tests/native/division_check.c); the IEEE division otherwise.
constexpr int kMaxMarksteinCount = 16384;

__device__ __forceinline__ float div_by_count(float a, float count, float rcp, bool count_ok) {
    const float mag = fabsf(a);
    if (count_ok && mag >= 0x1p-96f && mag <= 3.40282347e38f) {
        const float q0 = __fmul_rn(a, rcp);
        return __fmaf_rn(__fmaf_rn(-q0, count, a), rcp, q0);
    }
    return ieee_div(a, count);
}

// welford_combine, segmented_rms_adaln.cu:89-105 (same operation order).
__device__ __forceinline__ Welford combine(Welford l, const Welford r) {
    if (r.count == 0) return l;
    if (l.count == 0) return r;
    const int count = l.count + r.count;
    const float c = static_cast<float>(count);
    const float lc = static_cast<float>(l.count);
    const float rc = static_cast<float>(r.count);
    const bool ok = count <= kMaxMarksteinCount;
    const float rcp = ok ? __frcp_rn(c) : 0.0f;
    const float delta = __fsub_rn(r.mean, l.mean);
    l.mean = __fadd_rn(l.mean, div_by_count(__fmul_rn(delta, rc), c, rcp, ok));
    l.m2 = __fadd_rn(l.m2, __fadd_rn(r.m2, div_by_count(__fmul_rn(__fmul_rn(__fmul_rn(delta, delta), lc), rc), c,
                                                        rcp, ok)));
    l.count = count;
    return l;
}

// Welford step of the register-cached pass, where the count is the compile-time `count`
// (every earlier cached column of the thread was pushed) and `rcp` = RN(1 / count) is a
// compile-time constant; the division is div_by_count's.
__device__ __forceinline__ void welford_push_fixed(Welford &s, float v, float count, float rcp) {
    ++s.count;
    const float delta = __fsub_rn(v, s.mean);
    s.mean = __fadd_rn(s.mean, div_by_count(delta, count, rcp, true));
    s.m2 = __fmaf_rn(delta, __fsub_rn(v, s.mean), s.m2);
}

__device__ __forceinline__ void welford_push(Welford &s, float v) {
    ++s.count;
    const float delta = __fsub_rn(v, s.mean);
    s.mean = __fadd_rn(s.mean, __fdiv_rn(delta, static_cast<float>(s.count)));
    s.m2 = __fmaf_rn(delta, __fsub_rn(v, s.mean), s.m2);
}

// Modulation row offset of token row `row` (segmented_rms_adaln.cu:248-257).
__device__ __forceinline__ int64_t ln_modulation_offset(const LnArgs &a, int64_t row) {
    const int64_t batch = row / a.sequence;
    const int token = static_cast<int>(row - batch * a.sequence);
    int mtoken = 0;
    if (a.modulation_steps > 1) {
        const int repeats = a.sequence / a.modulation_steps;
        const int group = repeats * a.modulation_steps == a.sequence ? repeats : repeats + 1;
        mtoken = min(token / max(group, 1), a.modulation_steps - 1);
    }
    return (batch * a.modulation_steps + mtoken) * a.hidden;
}

// Mean and 1/std of the row held in `row_s`, in the reference's order: Welford per
// thread over columns t, t+256, ... (the first kSteps steps with the compile-time
// reciprocal of the count), the shfl_down Welford tree, the in-order combine of the
// 8 warps by warp 0.  Every thread of the CTA must call it.
template <typename T, int kSteps, typename Load>
__device__ __forceinline__ void ln_statistics(Load load, int hidden, float epsilon, float *warp_mean,
                                              float *warp_m2, int *warp_count, float &mean, float &inv) {
    using E = Elem<T>;
    const int tid = static_cast<int>(threadIdx.x);
    const int lane = tid & 31;
    const int warp = tid >> 5;
    Welford st{0.0f, 0.0f, 0};
#pragma unroll
    for (int i = 0; i < kSteps; ++i) {
        const int c = tid + i * kRowThreads;
        if (c < hidden) welford_push_fixed(st, E::load(load(c)), static_cast<float>(i + 1), 1.0f / static_cast<float>(i + 1));
    }
    for (int c = tid + kSteps * kRowThreads; c < hidden; c += kRowThreads) welford_push(st, E::load(load(c)));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const Welford other{__shfl_down_sync(0xffffffffu, st.mean, off), __shfl_down_sync(0xffffffffu, st.m2, off),
                            __shfl_down_sync(0xffffffffu, st.count, off)};
        st = combine(st, other);
    }
    if (lane == 0) {
        warp_mean[warp] = st.mean;
        warp_m2[warp] = st.m2;
        warp_count[warp] = st.count;
    }
    __syncthreads();
    if (warp == 0) {
        st = Welford{0.0f, 0.0f, 0};
#pragma unroll
        for (int w = 0; w < kWarps; ++w) st = combine(st, Welford{warp_mean[w], warp_m2[w], warp_count[w]});
        __syncwarp();
        if (lane == 0) {
            warp_mean[0] = st.mean;
            warp_m2[0] = rsqrtf(__fadd_rn(__fdiv_rn(st.m2, static_cast<float>(st.count)), epsilon));
        }
    }
    __syncthreads();
    mean = warp_mean[0];
    inv = warp_m2[0];
}

// Rows of at most kLnSmemBytes: the row is staged in shared memory with 16-byte loads
// (all of them in flight at once), the strided Welford pass reads it from there, and the
// output pass reads it back as 16-byte vectors.
template <typename T, int kSteps>
__global__ void __launch_bounds__(kRowThreads) layer_norm_adaln_kernel(const LnArgs a) {
    using E = Elem<T>;
    extern __shared__ uint4 row_v[];
    __shared__ float warp_mean[kWarps];
    __shared__ float warp_m2[kWarps];
    __shared__ int warp_count[kWarps];
    const T *row_s = reinterpret_cast<const T *>(row_v);

    const int64_t row = blockIdx.x;
    const int tid = static_cast<int>(threadIdx.x);
    const T *x = static_cast<const T *>(a.x) + row * a.hidden;
    constexpr int W = Vec<T>::kWidth;
    if (a.vector_in) {
        const uint4 *xv = reinterpret_cast<const uint4 *>(x);
        for (int j = tid; j < a.hidden / W; j += kRowThreads) row_v[j] = xv[j];
    } else {
        T *rw = reinterpret_cast<T *>(row_v);
        for (int c = tid; c < a.hidden; c += kRowThreads) rw[c] = x[c];
    }
    __syncthreads();
    float mean, inv;
    ln_statistics<T, kSteps>([&](int c) { return row_s[c]; }, a.hidden, a.epsilon, warp_mean, warp_m2, warp_count,
                             mean, inv);

    const int64_t mod_off = ln_modulation_offset(a, row);
    const T *scale = static_cast<const T *>(a.scale) + mod_off;
    const T *shift = static_cast<const T *>(a.shift) + mod_off;
    T *out = static_cast<T *>(a.out) + row * a.hidden;
    if (a.vector_out) {
        const uint4 *sv = reinterpret_cast<const uint4 *>(scale);
        const uint4 *hv = reinterpret_cast<const uint4 *>(shift);
        uint4 *ov = reinterpret_cast<uint4 *>(out);
        for (int j = tid; j < a.hidden / W; j += kRowThreads) ov[j] = ln_vector<T>(row_v[j], __ldg(sv + j), __ldg(hv + j), mean, inv);
    } else {
        for (int c = tid; c < a.hidden; c += kRowThreads)
            out[c] = E::store(ln_output<T>(E::load(row_s[c]), mean, inv, E::load(scale[c]), E::load(shift[c])));
    }
}

// Rows larger than kLnSmemBytes: the same computation reading the row from global memory
// in both passes.
template <typename T>
__global__ void __launch_bounds__(kRowThreads) layer_norm_adaln_wide_kernel(const LnArgs a) {
    using E = Elem<T>;
    __shared__ float warp_mean[kWarps];
    __shared__ float warp_m2[kWarps];
    __shared__ int warp_count[kWarps];
    const int64_t row = blockIdx.x;
    const T *x = static_cast<const T *>(a.x) + row * a.hidden;
    float mean, inv;
    ln_statistics<T, 8>([&](int c) { return x[c]; }, a.hidden, a.epsilon, warp_mean, warp_m2, warp_count, mean,
                        inv);
    const int64_t mod_off = ln_modulation_offset(a, row);
    const T *scale = static_cast<const T *>(a.scale) + mod_off;
    const T *shift = static_cast<const T *>(a.shift) + mod_off;
    T *out = static_cast<T *>(a.out) + row * a.hidden;
    for (int c = static_cast<int>(threadIdx.x); c < a.hidden; c += kRowThreads)
        out[c] = E::store(ln_output<T>(E::load(x[c]), mean, inv, E::load(scale[c]), E::load(shift[c])));
}

template <typename T, bool kVec>
cudaError_t launch_rms_t(const RmsArgs &a, cudaStream_t stream) {
    const int per_thread = kVec ? (a.hidden / Vec<T>::kWidth + kRowThreads - 1) / kRowThreads
                                : (a.hidden + kRowThreads - 1) / kRowThreads;
    const dim3 grid(static_cast<unsigned>(a.rows));
    if (per_thread <= 1) {
        segmented_rms_adaln_kernel<T, kVec, 1><<<grid, kRowThreads, 0, stream>>>(a);
    } else if (per_thread <= 2) {
        segmented_rms_adaln_kernel<T, kVec, 2><<<grid, kRowThreads, 0, stream>>>(a);
    } else if (per_thread <= 4) {
        segmented_rms_adaln_kernel<T, kVec, 4><<<grid, kRowThreads, 0, stream>>>(a);
    } else {
        segmented_rms_adaln_kernel<T, kVec, kRmsCacheVectors><<<grid, kRowThreads, 0, stream>>>(a);
    }
    return cudaGetLastError();
}

template <typename T>
cudaError_t launch_ln_t(const LnArgs &a, cudaStream_t stream) {
    const int per_thread = (a.hidden + kRowThreads - 1) / kRowThreads;
    const size_t bytes = (static_cast<size_t>(a.hidden) * sizeof(T) + 15) & ~size_t(15);
    const dim3 grid(static_cast<unsigned>(a.rows));
    if (bytes > kLnSmemBytes) {
        layer_norm_adaln_wide_kernel<T><<<grid, kRowThreads, 0, stream>>>(a);
    } else if (per_thread <= 8) {
        layer_norm_adaln_kernel<T, 8><<<grid, kRowThreads, bytes, stream>>>(a);
    } else if (per_thread <= 16) {
        layer_norm_adaln_kernel<T, 16><<<grid, kRowThreads, bytes, stream>>>(a);
    } else if (per_thread <= 32) {
        layer_norm_adaln_kernel<T, 32><<<grid, kRowThreads, bytes, stream>>>(a);
    } else {
        layer_norm_adaln_kernel<T, kLnSteps><<<grid, kRowThreads, bytes, stream>>>(a);
    }
    return cudaGetLastError();
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

bool rms_vectorized(const RmsArgs &a, int type) {
    const int width = type == kNormFp32 ? 4 : 8;
    return a.hidden % width == 0 && a.scale_stride % width == 0 && a.shift_stride % width == 0 && aligned16(a.x) &&
           aligned16(a.weight) && aligned16(a.scale) && aligned16(a.shift);
}

cudaError_t launch_segmented_rms_adaln(const RmsArgs &args, int type, cudaStream_t stream) {
    RmsArgs a = args;
    const bool vec = rms_vectorized(a, type);
    a.vector_store = aligned16(a.out) ? 1 : 0;
    switch (type) {
        case kNormBf16:
            return vec ? launch_rms_t<__nv_bfloat16, true>(a, stream) : launch_rms_t<__nv_bfloat16, false>(a, stream);
        case kNormFp16:
            return vec ? launch_rms_t<__half, true>(a, stream) : launch_rms_t<__half, false>(a, stream);
        case kNormFp32:
            return vec ? launch_rms_t<float, true>(a, stream) : launch_rms_t<float, false>(a, stream);
        default:
            return cudaErrorInvalidValue;
    }
}

cudaError_t launch_layer_norm_adaln(const LnArgs &args, int type, cudaStream_t stream) {
    LnArgs a = args;
    const int width = type == kNormFp32 ? 4 : 8;
    a.vector_in = a.hidden % width == 0 && aligned16(a.x);
    a.vector_out = a.hidden % width == 0 && aligned16(a.scale) && aligned16(a.shift) && aligned16(a.out);
    switch (type) {
        case kNormBf16:
            return launch_ln_t<__nv_bfloat16>(a, stream);
        case kNormFp16:
            return launch_ln_t<__half>(a, stream);
        case kNormFp32:
            return launch_ln_t<float>(a, stream);
        default:
            return cudaErrorInvalidValue;
    }
}

}  // namespace norm
}  // namespace ctu
