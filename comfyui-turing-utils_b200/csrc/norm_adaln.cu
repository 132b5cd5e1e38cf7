// Affine RMSNorm + segmented AdaLN, and LayerNorm + Wan AdaLN, for bf16 / fp16 / fp32
// rows (reference: kernel/csrc/turing/segmented_rms_adaln.cu:133-297).
//
// Both norms are HBM-streaming and read each row from HBM once (the reference reads it
// twice): RMS with one CTA of 256 threads per row that keeps its 16-byte vectors in
// registers for the output pass; LayerNorm with persistent 256-thread CTAs that bring
// each row into shared memory by a bulk copy issued one row ahead.  The thread-to-column
// mapping and the reduction tree are the reference's, because they fix the fp32
// rounding of the statistics and so the output bits:
//   * RMS: thread t accumulates fma(v, v, s) over 16-byte vectors t, t+256, ... in
//     order (or columns t, t+256, ... when the reference launch is not vectorized);
//   * LayerNorm: thread t runs Welford over columns t, t+256, ..., every quotient equal
//     to the reference's IEEE division by the count;
//   * a shfl_down tree inside each warp, then the 8 warp partials combined in order.
// Every arithmetic step is written with round-to-nearest intrinsics so that the
// compiler cannot contract or reorder it differently from the reference's build.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <map>
#include <mutex>
#include <tuple>

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
        // ln_output on two values per packed instruction; each rounding to the storage
        // type is the pack of the pair (round to nearest even per lane).
        using Wd = Words<T>;
        const f32x2 mean2 = pk2(mean, mean);
        const f32x2 inv2 = pk2(inv, inv);
        const f32x2 one2 = pk2(1.0f, 1.0f);
        auto f = [&](uint32_t xw, uint32_t sw, uint32_t hw) {
            const f32x2 normalized = Wd::unpack(Wd::pack(fmul2(fsub2(Wd::unpack(xw), mean2), inv2)));
            const f32x2 multiplier = Wd::unpack(Wd::pack(fadd2(one2, Wd::unpack(sw))));
            return Wd::pack(ffma2(normalized, multiplier, Wd::unpack(hw)));
        };
        (void)sizeof(E);
        return make_uint4(f(x.x, s.x, h.x), f(x.y, s.y, h.y), f(x.z, s.z, h.z), f(x.w, s.w, h.w));
    }
}

// store(1 + s) for the values of one 16-byte vector (the multiplier of ln_output).
template <typename T>
__device__ __forceinline__ uint4 ln_multiplier(const uint4 s) {
    if constexpr (sizeof(T) == 4) {
        auto f = [](uint32_t v) { return __float_as_uint(__fadd_rn(1.0f, __uint_as_float(v))); };
        return make_uint4(f(s.x), f(s.y), f(s.z), f(s.w));
    } else {
        using Wd = Words<T>;
        const f32x2 one2 = pk2(1.0f, 1.0f);
        auto f = [&](uint32_t w) { return Wd::pack(fadd2(one2, Wd::unpack(w))); };
        return make_uint4(f(s.x), f(s.y), f(s.z), f(s.w));
    }
}

// ln_vector with the multiplier already rounded to the storage type (m = store(1 + s)).
template <typename T>
__device__ __forceinline__ uint4 ln_vector_mult(const uint4 x, const uint4 m, const uint4 h, float mean, float inv) {
    using E = Elem<T>;
    if constexpr (sizeof(T) == 4) {
        auto f = [&](uint32_t xv, uint32_t mv, uint32_t hv) {
            const float normalized = E::load(E::store(__fmul_rn(__fsub_rn(__uint_as_float(xv), mean), inv)));
            return __float_as_uint(__fmaf_rn(normalized, __uint_as_float(mv), __uint_as_float(hv)));
        };
        return make_uint4(f(x.x, m.x, h.x), f(x.y, m.y, h.y), f(x.z, m.z, h.z), f(x.w, m.w, h.w));
    } else {
        using Wd = Words<T>;
        const f32x2 mean2 = pk2(mean, mean);
        const f32x2 inv2 = pk2(inv, inv);
        auto f = [&](uint32_t xw, uint32_t mw, uint32_t hw) {
            const f32x2 normalized = Wd::unpack(Wd::pack(fmul2(fsub2(Wd::unpack(xw), mean2), inv2)));
            return Wd::pack(ffma2(normalized, Wd::unpack(mw), Wd::unpack(hw)));
        };
        return make_uint4(f(x.x, m.x, h.x), f(x.y, m.y, h.y), f(x.z, m.z, h.z), f(x.w, m.w, h.w));
    }
}

struct Welford {
    float mean;
    float m2;
    int count;
};

// Welford step with IEEE division by the new count (segmented_rms_adaln.cu:74-78).
__device__ __forceinline__ void welford_push(Welford &s, float v) {
    ++s.count;
    const float delta = __fsub_rn(v, s.mean);
    s.mean = __fadd_rn(s.mean, __fdiv_rn(delta, static_cast<float>(s.count)));
    s.m2 = __fmaf_rn(delta, __fsub_rn(v, s.mean), s.m2);
}

// welford_combine, segmented_rms_adaln.cu:86-100 (same operation order, IEEE division).
__device__ __forceinline__ Welford combine_ieee(Welford l, const Welford r) {
    if (r.count == 0) return l;
    if (l.count == 0) return r;
    const int count = l.count + r.count;
    const float c = static_cast<float>(count);
    const float delta = __fsub_rn(r.mean, l.mean);
    l.mean = __fadd_rn(l.mean, __fdiv_rn(__fmul_rn(delta, static_cast<float>(r.count)), c));
    l.m2 = __fadd_rn(l.m2, __fadd_rn(r.m2, __fdiv_rn(__fmul_rn(__fmul_rn(__fmul_rn(delta, delta),
                                                                        static_cast<float>(l.count)),
                                                               static_cast<float>(r.count)),
                                                      c)));
    l.count = count;
    return l;
}

// a / c for a positive integer c by the correction step of Markstein's division with
// rcp = RN(1 / c): q0 = a * rcp, r = fma(-q0, c, a) (exact), q = fma(r, rcp, q0).  It
// equals the IEEE quotient for every c <= kMaxMarksteinCount and every a with
// 2^-96 <= |a| <= FLT_MAX (checked over every significand by
// tests/native/division_check.c), and is NaN for a NaN a as the IEEE one is.  For a == 0
// it returns +0 where IEEE gives the sign of a; that cannot change any sum below, because
// no running mean or m2 is ever -0 (they start at +0, and a round-to-nearest sum is -0
// only when both terms are), so x + (+-0) == x.
constexpr int kMaxMarksteinCount = 16384;

__device__ __forceinline__ float markstein_div(float a, float c, float rcp) {
    const float q0 = __fmul_rn(a, rcp);
    return __fmaf_rn(__fmaf_rn(-q0, c, a), rcp, q0);
}

// False when a Welford step's quotient markstein_div(delta, ...) may differ from the IEEE
// one in a way that can reach the output: 0 < |delta| < 2^-96.  An infinite delta (an
// infinite input, or an overflowing difference of finite ones) gives NaN here and +-inf
// in the reference, but either way that thread's m2 becomes NaN or -inf for good (the
// step's fma(delta, v - mean, m2) meets inf - inf or inf * -inf), no later combine can
// turn that into a finite or positive value, and rsqrtf of the row's variance is NaN on
// both paths, so every output of the row is NaN on both.
__device__ __forceinline__ bool markstein_safe(float a) {
    const float mag = fabsf(a);
    return !(mag < 0x1p-96f && mag != 0.0f);
}

// Reciprocal of the count of Welford step I (the count is I + 1), a compile-time constant.
template <int I>
struct StepRcp {
    static constexpr float value = 1.0f / static_cast<float>(I + 1);
};

// Welford step I of one thread (column tid + I * 256), count and reciprocal constants.
template <int I, typename T, typename Load>
__device__ __forceinline__ void welford_step(Welford &st, Load load, int tid, bool &exact) {
    const float v = Elem<T>::load(load(tid + I * kRowThreads));
    const float delta = __fsub_rn(v, st.mean);
    exact = exact && markstein_safe(delta);
    st.mean = __fadd_rn(st.mean, markstein_div(delta, static_cast<float>(I + 1), StepRcp<I>::value));
    st.m2 = __fmaf_rn(delta, __fsub_rn(v, st.mean), st.m2);
}

// Welford steps I..N-1 of one thread (columns tid + I * 256, ...).  Steps that every
// thread takes run unguarded; the first one that not every thread takes is the last and
// is guarded per thread (the tests on I are uniform).  `exact` is cleared when a step's
// quotient may differ from the IEEE one; the caller then redoes the chain.
template <int I, int N, typename T, typename Load>
__device__ __forceinline__ void welford_steps(Welford &st, Load load, int hidden, int tid, bool &exact) {
    if constexpr (I < N) {
        if ((I + 1) * kRowThreads <= hidden) {
            welford_step<I, T>(st, load, tid, exact);
            welford_steps<I + 1, N, T>(st, load, hidden, tid, exact);
        } else if (tid + I * kRowThreads < hidden) {
            welford_step<I, T>(st, load, tid, exact);
        }
    }
}

// The counts of one combine are fixed by the row length alone, so each CTA works them
// out once: (left count, right count, total, RN(1 / total)) as floats (rcp 0 when the
// total is 0 or above kMaxMarksteinCount).
__device__ __forceinline__ float4 combine_plan(int lc, int rc) {
    const int c = lc + rc;
    const float rcp = (c > 0 && c <= kMaxMarksteinCount) ? __frcp_rn(static_cast<float>(c)) : 0.0f;
    return make_float4(static_cast<float>(lc), static_cast<float>(rc), static_cast<float>(c), rcp);
}

// welford_combine on (mean, m2) for two positive counts with a total of at most
// kMaxMarksteinCount, taken from `plan`.  Returns false when a quotient may differ from
// the IEEE one (the caller redoes the reduction with IEEE division).  Both quotients are
// exact when delta == 0 or 2^-96 <= |a2| <= FLT_MAX, a2 = delta^2 * lc * rc: then
// a1 = delta * rc is in that range too (with lc * rc <= 2^28, a2 >= 2^-96 needs
// |delta| >= 2^-62, and |delta| >= 1 gives |a1| <= |a2|).  A NaN stays NaN on both paths.
__device__ __forceinline__ bool combine_fast(float &mean, float &m2, float rmean, float rm2, const float4 plan) {
    const float delta = __fsub_rn(rmean, mean);
    const float a1 = __fmul_rn(delta, plan.y);
    const float a2 = __fmul_rn(__fmul_rn(__fmul_rn(delta, delta), plan.x), plan.y);
    mean = __fadd_rn(mean, markstein_div(a1, plan.z, plan.w));
    m2 = __fadd_rn(m2, __fadd_rn(rm2, markstein_div(a2, plan.z, plan.w)));
    const float mag = fabsf(a2);
    return delta == 0.0f || !(mag < 0x1p-96f || mag > 3.40282347e38f);
}

// combine_fast where either count may be 0 (rows shorter than 256 columns): a right
// count of 0 keeps the left state and a left count of 0 takes the right one, as
// welford_combine's early returns do.
__device__ __forceinline__ bool combine_general(float &mean, float &m2, float rmean, float rm2, const float4 plan) {
    float nmean = mean, nm2 = m2;
    const bool ok = combine_fast(nmean, nm2, rmean, rm2, plan);
    const bool keep = plan.y == 0.0f;
    const bool take = plan.x == 0.0f;
    mean = keep ? mean : (take ? rmean : nmean);
    m2 = keep ? m2 : (take ? rm2 : nm2);
    return keep || take || ok;
}

constexpr int kTreeLevels = 5;  // shfl_down offsets 16, 8, 4, 2, 1
enum TreeMode : int { kTreeFast = 0, kTreeGeneral = 1, kTreeIeee = 2 };
constexpr int kPlanKinds = 3;  // warps whose lanes hold base + 1, base, or both column counts
constexpr size_t kTreePlanBytes = static_cast<size_t>(kPlanKinds) * kTreeLevels * 32 * sizeof(float4);

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

// LayerNorm + AdaLN over rows blockIdx.x, blockIdx.x + gridDim.x, ... (persistent CTAs of
// 256 threads).  Statistics in the reference's order: Welford per thread over columns t,
// t+256, ..., the shfl_down Welford tree in each warp, then warp 0 combines the 8 warp
// partials in order; every division by a count is the Markstein step with the count's
// reciprocal worked out in advance, and a row whose operands leave markstein_safe's
// range is redone with IEEE division.
// kStaged: the row (at most kLnSmemBytes) is copied into one of two shared-memory
// buffers -- a bulk copy issued one row ahead when rows are 16-byte aligned, plain loads
// otherwise -- and both passes read it from there.  Otherwise both passes read HBM.
template <typename T, bool kStaged>
__global__ void __launch_bounds__(kRowThreads) layer_norm_adaln_kernel(const LnArgs a) {
    using E = Elem<T>;
    constexpr int W = Vec<T>::kWidth;
    extern __shared__ float4 ln_smem[];
    float4 *tree_plan = ln_smem;  // [warp kind][level][lane]
    uint8_t *bufs = reinterpret_cast<uint8_t *>(ln_smem + kPlanKinds * kTreeLevels * 32);
    __shared__ float4 warp_plan[kWarps];
    __shared__ int warp_count[kWarps];
    __shared__ float warp_mean[kWarps];
    __shared__ float warp_m2[kWarps];
    __shared__ float row_mean;
    __shared__ float row_inv;
    __shared__ long long row_mod;
    __shared__ __align__(8) uint64_t full[2];

    const int tid = static_cast<int>(threadIdx.x);
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int hidden = a.hidden;
    const uint32_t row_bytes = static_cast<uint32_t>(hidden) * static_cast<uint32_t>(sizeof(T));
    const uint32_t buf_bytes = (row_bytes + 15u) & ~15u;
    const bool bulk = kStaged && a.vector_in;

    // Counts of every combine of this CTA's rows.  Thread t holds base + (t < rem)
    // columns, so a warp's lanes hold base + 1 columns (kind 0), base (kind 1), or base + 1
    // below lane rem % 32 (kind 2, the one warp that straddles rem); warp k < 3 works out
    // the tree counts of kind k.
    const int base = hidden / kRowThreads;
    const int rem = hidden % kRowThreads;
    const int kind = 32 * (warp + 1) <= rem ? 0 : (32 * warp >= rem ? 1 : 2);
    if (warp < kPlanKinds) {
        const int high_lanes = warp == 0 ? 32 : (warp == 1 ? 0 : rem % 32);
        int count = base + (lane < high_lanes ? 1 : 0);
#pragma unroll
        for (int k = 0; k < kTreeLevels; ++k) {
            const int off = 16 >> k;
            const int right = __shfl_down_sync(0xffffffffu, count, off);
            const int rc = lane + off < 32 ? right : 0;  // lanes past the warp end are discarded
            tree_plan[(warp * kTreeLevels + k) * 32 + lane] = combine_plan(count, rc);
            count += rc;
        }
    }
    if (lane == 0) warp_count[warp] = 32 * base + min(max(rem - 32 * warp, 0), 32);
    const float4 *my_plan = tree_plan + kind * kTreeLevels * 32 + lane;
    if (tid == 0 && bulk) {
        mbar_init(&full[0], 1);
        mbar_init(&full[1], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        int total = 0;
        for (int w = 0; w < kWarps; ++w) {
            warp_plan[w] = combine_plan(total, warp_count[w]);
            total += warp_count[w];
        }
        if (bulk && static_cast<int64_t>(blockIdx.x) < a.rows) {
            mbar_arrive_expect_tx(&full[0], row_bytes);
            bulk_load(bufs, static_cast<const T *>(a.x) + static_cast<int64_t>(blockIdx.x) * hidden, row_bytes,
                      &full[0]);
        }
    }
    __syncthreads();
    // Which combines take the Markstein path: every tree count and total is at most
    // kMaxMarksteinCount (warp 0 holds the most columns), and (fast) every count is
    // positive.  Warp 0's partial always has a count, so the in-order combine of the
    // warps starts from it (welford_combine with an empty left state returns the right).
    const int tree_mode = warp_count[0] > kMaxMarksteinCount ? kTreeIeee
                          : hidden >= kRowThreads            ? kTreeFast
                                                             : kTreeGeneral;
    const int final_mode = hidden > kMaxMarksteinCount      ? kTreeIeee
                           : hidden > (kWarps - 1) * 32      ? kTreeFast
                                                             : kTreeGeneral;

    int64_t mult_off = -1;  // modulation offset whose multiplier row is in shared memory
    int it = 0;
    for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x, ++it) {
        const T *x = static_cast<const T *>(a.x) + row * hidden;
        const int b = it & 1;
        const T *row_s = reinterpret_cast<const T *>(bufs + b * buf_bytes);
        bool ok = true;
        if constexpr (kStaged) {
            if (bulk) {
                ok = mbar_wait(&full[b], static_cast<uint32_t>(it >> 1) & 1u, nullptr, a.err, kErrTimeoutFull);
            } else {
                // Buffer b was last read two rows ago, before the previous row's barriers.
                T *rw = reinterpret_cast<T *>(bufs + b * buf_bytes);
                for (int c = tid; c < hidden; c += kRowThreads) rw[c] = x[c];
                __syncthreads();
            }
        }
        auto load = [&](int c) -> T {
            if constexpr (kStaged) {
                return row_s[c];
            } else {
                return x[c];
            }
        };

        // Per-thread Welford chain.
        Welford st{0.0f, 0.0f, 0};
        bool exact = true;
        welford_steps<0, kLnSteps, T>(st, load, hidden, tid, exact);
        st.count = hidden > tid ? min(kLnSteps, (hidden - 1 - tid) / kRowThreads + 1) : 0;
        if (!exact) {
            st = Welford{0.0f, 0.0f, 0};
#pragma unroll 1
            for (int c = tid; c < min(hidden, kLnSteps * kRowThreads); c += kRowThreads)
                welford_push(st, E::load(load(c)));
        }
#pragma unroll 1
        for (int c = tid + kLnSteps * kRowThreads; c < hidden; c += kRowThreads) welford_push(st, E::load(load(c)));

        // Warp tree.  Lanes whose partner lies past the warp end read their own state
        // (delta 0); their results, like those of every lane >= off, are discarded.
        {
            const float mean0 = st.mean, m20 = st.m2;
            bool good = tree_mode != kTreeIeee;
            if (tree_mode == kTreeFast) {
#pragma unroll
                for (int k = 0; k < kTreeLevels; ++k) {
                    const float rmean = __shfl_down_sync(0xffffffffu, st.mean, 16 >> k);
                    const float rm2 = __shfl_down_sync(0xffffffffu, st.m2, 16 >> k);
                    good = combine_fast(st.mean, st.m2, rmean, rm2, my_plan[k * 32]) && good;
                }
            } else if (tree_mode == kTreeGeneral) {
#pragma unroll
                for (int k = 0; k < kTreeLevels; ++k) {
                    const float rmean = __shfl_down_sync(0xffffffffu, st.mean, 16 >> k);
                    const float rm2 = __shfl_down_sync(0xffffffffu, st.m2, 16 >> k);
                    good = combine_general(st.mean, st.m2, rmean, rm2, my_plan[k * 32]) && good;
                }
            }
            if (!__all_sync(0xffffffffu, good)) {
                Welford w{mean0, m20, hidden > tid ? (hidden - 1 - tid) / kRowThreads + 1 : 0};
#pragma unroll 1
                for (int off = 16; off > 0; off >>= 1) {
                    const Welford other{__shfl_down_sync(0xffffffffu, w.mean, off),
                                        __shfl_down_sync(0xffffffffu, w.m2, off),
                                        __shfl_down_sync(0xffffffffu, w.count, off)};
                    w = combine_ieee(w, other);
                }
                st.mean = w.mean;
                st.m2 = w.m2;
            }
        }
        if (lane == 0) {
            warp_mean[warp] = st.mean;
            warp_m2[warp] = st.m2;
        }
        if (__syncthreads_or(!ok)) {
            // A row copy did not arrive in time: wait (bounded) for it, then stop.
            if (tid == 0 && bulk) (void)mbar_wait(&full[b], static_cast<uint32_t>(it >> 1) & 1u, nullptr, a.err,
                                                  kErrTimeoutDrain);
            return;
        }
        if (tid == 0 && bulk && row + gridDim.x < a.rows) {
            // Prefetch the CTA's next row into the other buffer, last read one row ago.
            const int nb = b ^ 1;
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(&full[nb], row_bytes);
            bulk_load(bufs + nb * buf_bytes, x + static_cast<int64_t>(gridDim.x) * hidden, row_bytes, &full[nb]);
        }
        if (warp == 0) {
            float mean = warp_mean[0], m2 = warp_m2[0];
            bool good = final_mode != kTreeIeee;
            if (final_mode == kTreeFast) {
#pragma unroll
                for (int w = 1; w < kWarps; ++w)
                    good = combine_fast(mean, m2, warp_mean[w], warp_m2[w], warp_plan[w]) && good;
            } else if (final_mode == kTreeGeneral) {
#pragma unroll
                for (int w = 1; w < kWarps; ++w)
                    good = combine_general(mean, m2, warp_mean[w], warp_m2[w], warp_plan[w]) && good;
            }
            if (!good) {
                Welford s{0.0f, 0.0f, 0};
#pragma unroll 1
                for (int w = 0; w < kWarps; ++w) s = combine_ieee(s, Welford{warp_mean[w], warp_m2[w], warp_count[w]});
                mean = s.mean;
                m2 = s.m2;
            }
            if (lane == 0) {
                row_mean = mean;
                row_inv = rsqrtf(__fadd_rn(__fdiv_rn(m2, static_cast<float>(hidden)), a.epsilon));
                row_mod = ln_modulation_offset(a, row);
            }
        }
        __syncthreads();
        const float mean = row_mean;
        const float inv = row_inv;
        const int64_t mod_off = row_mod;

        const T *scale = static_cast<const T *>(a.scale) + mod_off;
        const T *shift = static_cast<const T *>(a.shift) + mod_off;
        T *out = static_cast<T *>(a.out) + row * hidden;
        if (kStaged && a.vector_out) {
            // store(1 + scale) of the row's modulation row, kept in shared memory while
            // consecutive rows of the CTA share it (mod_off is uniform across the CTA).
            uint4 *mult = reinterpret_cast<uint4 *>(bufs + 2 * buf_bytes);
            const uint4 *sv = reinterpret_cast<const uint4 *>(scale);
            if (mod_off != mult_off) {
                for (int j = tid; j < hidden / W; j += kRowThreads) mult[j] = ln_multiplier<T>(__ldg(sv + j));
                __syncthreads();
                mult_off = mod_off;
            }
            const uint4 *xv = reinterpret_cast<const uint4 *>(row_s);
            const uint4 *hv = reinterpret_cast<const uint4 *>(shift);
            uint4 *ov = reinterpret_cast<uint4 *>(out);
            for (int j = tid; j < hidden / W; j += kRowThreads)
                ov[j] = ln_vector_mult<T>(xv[j], mult[j], __ldg(hv + j), mean, inv);
        } else if (a.vector_out && (kStaged || a.vector_in)) {
            const uint4 *xv = kStaged ? reinterpret_cast<const uint4 *>(row_s) : reinterpret_cast<const uint4 *>(x);
            const uint4 *sv = reinterpret_cast<const uint4 *>(scale);
            const uint4 *hv = reinterpret_cast<const uint4 *>(shift);
            uint4 *ov = reinterpret_cast<uint4 *>(out);
            for (int j = tid; j < hidden / W; j += kRowThreads)
                ov[j] = ln_vector<T>(xv[j], __ldg(sv + j), __ldg(hv + j), mean, inv);
        } else {
            for (int c = tid; c < hidden; c += kRowThreads)
                out[c] = E::store(ln_output<T>(E::load(load(c)), mean, inv, E::load(scale[c]), E::load(shift[c])));
        }
    }
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

// CTAs per SM of one LayerNorm kernel at one shared-memory size, per device.  Filled on
// first use, so the first call of a shape should come before any stream capture.
std::mutex g_ln_mutex;
std::map<std::tuple<const void *, int, size_t>, int> g_ln_occupancy;

cudaError_t ln_ctas_per_sm(const void *kernel, size_t smem, int *per_sm) {
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return e;
    const auto key = std::make_tuple(kernel, device, smem);
    {
        std::lock_guard<std::mutex> lock(g_ln_mutex);
        auto it = g_ln_occupancy.find(key);
        if (it != g_ln_occupancy.end()) {
            *per_sm = it->second;
            return cudaSuccess;
        }
    }
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kTreePlanBytes + 3 * kLnSmemBytes));
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, kernel, kRowThreads, smem);
    if (e != cudaSuccess) return e;
    if (*per_sm < 1) return cudaErrorInvalidConfiguration;
    std::lock_guard<std::mutex> lock(g_ln_mutex);
    g_ln_occupancy[key] = *per_sm;
    return cudaSuccess;
}

template <typename T>
cudaError_t launch_ln_t(const LnArgs &a, int num_sms, cudaStream_t stream) {
    const size_t row_bytes = (static_cast<size_t>(a.hidden) * sizeof(T) + 15) & ~size_t(15);
    const bool staged = row_bytes <= static_cast<size_t>(kLnSmemBytes);
    const void *kernel = staged ? reinterpret_cast<const void *>(layer_norm_adaln_kernel<T, true>)
                                : reinterpret_cast<const void *>(layer_norm_adaln_kernel<T, false>);
    const size_t smem = kTreePlanBytes + (staged ? 3 * row_bytes : 0);  // two row buffers + the multiplier row
    int per_sm = 0;
    cudaError_t e = ln_ctas_per_sm(kernel, smem, &per_sm);
    if (e != cudaSuccess) return e;
    const dim3 grid(static_cast<unsigned>(std::min<int64_t>(a.rows, static_cast<int64_t>(num_sms) * per_sm)));
    if (staged) {
        layer_norm_adaln_kernel<T, true><<<grid, kRowThreads, smem, stream>>>(a);
    } else {
        layer_norm_adaln_kernel<T, false><<<grid, kRowThreads, smem, stream>>>(a);
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

cudaError_t launch_layer_norm_adaln(const LnArgs &args, int type, int num_sms, cudaStream_t stream) {
    LnArgs a = args;
    const int width = type == kNormFp32 ? 4 : 8;
    a.vector_in = a.hidden % width == 0 && aligned16(a.x);
    a.vector_out = a.hidden % width == 0 && aligned16(a.scale) && aligned16(a.shift) && aligned16(a.out);
    switch (type) {
        case kNormBf16:
            return launch_ln_t<__nv_bfloat16>(a, num_sms, stream);
        case kNormFp16:
            return launch_ln_t<__half>(a, num_sms, stream);
        case kNormFp32:
            return launch_ln_t<float>(a, num_sms, stream);
        default:
            return cudaErrorInvalidValue;
    }
}

}  // namespace norm
}  // namespace ctu
