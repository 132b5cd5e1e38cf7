// sm_100a PTX wrappers shared by the ConvRot kernels: mbarriers with bounded
// waits, bulk (TMA) copies, tensor-map tile loads, tcgen05 (TMEM alloc, MMA,
// commit, loads) and packed f32x2 arithmetic.  Every wait in this library is
// bounded: on timeout it records an error code in the device error word and
// reports failure instead of spinning forever.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

namespace ctu {

// ---------------------------------------------------------------------------
// Device error word.  Kernels OR a code into *err; the host reads and clears it
// (ctu_get_device_error).  Codes are bit flags so several sites can report.
enum DeviceError : uint32_t {
    kErrNone = 0,
    kErrTimeoutFull = 1u << 0,      // consumer waited too long for a TMA tile
    kErrTimeoutEmpty = 1u << 1,     // producer waited too long for a free stage
    kErrTimeoutAccum = 1u << 2,     // epilogue waited too long for an accumulator
    kErrTimeoutAccumFree = 1u << 3, // MMA waited too long for the epilogue
    kErrTimeoutDrain = 1u << 4,     // teardown waited too long for copies in flight
    kErrTmemAlloc = 1u << 5,        // TMEM allocation returned an unusable address
    kErrInjected = 1u << 6,         // test hook: a wait on a barrier nobody arrives on
    kErrTimeoutRows = 1u << 7,      // fused linear: GEMM waited too long for quantized rows
};

// Wait limit in nanoseconds of %globaltimer.  Far above any legitimate wait in
// these kernels (a whole launch takes milliseconds).
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar_addr), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity.  `abort_flag` (shared
// memory) lets one timed-out role stop the others quickly; `err` is the global
// error word.  Returns false on timeout or abort.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                          uint32_t *err, uint32_t code, uint64_t limit_ns = kWaitLimitNs) {
    const uint32_t addr = smem_u32(bar);
    if (mbar_try_wait(addr, parity)) return true;
    const uint64_t start = globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(addr, parity)) return true;
        if ((i & 31u) == 0u) {
            if (abort_flag != nullptr && *abort_flag) return false;
            if (globaltimer() - start > limit_ns) {
                if (abort_flag != nullptr) *abort_flag = 1;
                atomicOr(err, code);
                return false;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Bulk copies (TMA, untiled) and proxy fences
__device__ __forceinline__ void bulk_load(void *smem_dst, const void *gmem_src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void bulk_store(void *gmem_dst, const void *smem_src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gmem_dst),
                 "r"(smem_u32(smem_src)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

__device__ __forceinline__ void bulk_wait_read_all() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Orders this thread's generic-proxy view of global memory with its async-proxy
// (TMA) accesses: after acquiring data that other SMs wrote with ordinary stores, a
// tensor-map load issued behind this fence reads those values.
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Cross-CTA progress counters in global memory (gpu scope)
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_gpu_add(uint32_t *p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait until *counter >= target, with acquire semantics on success.  Sleeps
// briefly between polls so the waiting warp leaves the issue slots to the others.
__device__ __forceinline__ bool counter_wait(const uint32_t *counter, uint32_t target, volatile int *abort_flag,
                                             uint32_t *err, uint32_t code, uint64_t limit_ns = kWaitLimitNs) {
    if (ld_acquire_gpu(counter) >= target) return true;
    const uint64_t start = globaltimer();
    for (uint32_t i = 1;; ++i) {
        __nanosleep(100);
        if (ld_acquire_gpu(counter) >= target) return true;
        if ((i & 15u) == 0u) {
            if (abort_flag != nullptr && *abort_flag) return false;
            if (globaltimer() - start > limit_ns) {
                if (abort_flag != nullptr) *abort_flag = 1;
                atomicOr(err, code);
                return false;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Tensor-map tile loads (2D, no multicast)
__device__ __forceinline__ void tma_load_2d(void *smem_dst, const void *tmap, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(smem_dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void *tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 (5th-generation tensor cores, TMEM accumulators)
__device__ __forceinline__ void tmem_alloc(uint32_t *smem_result, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, int8 x int8 -> int32.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

// Packed pair of 32-bit TMEM columns (2i in the low half, 2i + 1 in the high half).
typedef unsigned long long u32x2;

// 32 lanes x 32 consecutive 32-bit columns, waited for and returned as 16 packed pairs.
__device__ __forceinline__ void tmem_ld_32x32b_x32_pairs(uint32_t taddr, u32x2 (&r)[16]) {
    asm volatile(
        "{\n\t.reg .b32 t0,t1,t2,t3,t4,t5,t6,t7,t8,t9,t10,t11,t12,t13,t14,t15,t16,t17,t18,t19,t20,t21,t22,t23,t24,t25,t26,t27,t28,t29,t30,t31;\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {t0,t1,t2,t3,t4,t5,t6,t7,t8,t9,t10,t11,t12,t13,t14,t15,t16,t17,t18,t19,t20,t21,t22,t23,t24,t25,t26,t27,t28,t29,t30,t31}, [%16];\n\t"
        "tcgen05.wait::ld.sync.aligned;\n\t"
        "mov.b64 %0, {t0, t1};\n\t"
        "mov.b64 %1, {t2, t3};\n\t"
        "mov.b64 %2, {t4, t5};\n\t"
        "mov.b64 %3, {t6, t7};\n\t"
        "mov.b64 %4, {t8, t9};\n\t"
        "mov.b64 %5, {t10, t11};\n\t"
        "mov.b64 %6, {t12, t13};\n\t"
        "mov.b64 %7, {t14, t15};\n\t"
        "mov.b64 %8, {t16, t17};\n\t"
        "mov.b64 %9, {t18, t19};\n\t"
        "mov.b64 %10, {t20, t21};\n\t"
        "mov.b64 %11, {t22, t23};\n\t"
        "mov.b64 %12, {t24, t25};\n\t"
        "mov.b64 %13, {t26, t27};\n\t"
        "mov.b64 %14, {t28, t29};\n\t"
        "mov.b64 %15, {t30, t31};\n\t"
        "}"
        : "=l"(r[0]), "=l"(r[1]), "=l"(r[2]), "=l"(r[3]), "=l"(r[4]), "=l"(r[5]), "=l"(r[6]), "=l"(r[7]), "=l"(r[8]), "=l"(r[9]), "=l"(r[10]), "=l"(r[11]), "=l"(r[12]), "=l"(r[13]), "=l"(r[14]), "=l"(r[15])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }


// Shared-memory matrix descriptor for a K-major operand tile stored with the
// 128-byte swizzle: rows of 128 bytes, 8-row core groups 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);  // start address  [0,14)
    d |= static_cast<uint64_t>(1) << 16;                       // leading byte offset (unused for SW128 K-major)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;               // stride byte offset [32,46)
    d |= static_cast<uint64_t>(1) << 46;                       // descriptor version for sm_100
    d |= static_cast<uint64_t>(2) << 61;                       // layout: 128-byte swizzle
    return d;
}

// Instruction descriptor: kind::i8, s8 x s8 -> s32, saturating, K-major A and B.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
    return (1u << 3)                                  // saturate
           | (2u << 4)                                // D format: s32
           | (1u << 7)                                // A: signed 8-bit
           | (1u << 10)                               // B: signed 8-bit
           | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
           | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

// ---------------------------------------------------------------------------
// Packed fp32 pairs (Blackwell FADD2/FMUL2): two IEEE round-to-nearest results.
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
    float2 r;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %5};\n\t"
        "sub.rn.f32x2 rd, ra, rb;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(r.x), "=f"(r.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return r;
}

// Packed fp32 pairs held in one 64-bit register (low half = first value).  Keeping
// pairs in 64-bit containers end to end lets every FADD2/FMUL2/FFMA2 take its
// operands without re-pairing moves.
typedef unsigned long long f32x2;

__device__ __forceinline__ f32x2 pk2(float lo, float hi) {
    f32x2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void unpk2(f32x2 v, float &lo, float &hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ f32x2 fadd2(f32x2 a, f32x2 b) {
    f32x2 d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ f32x2 fsub2(f32x2 a, f32x2 b) {
    f32x2 d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ f32x2 fmul2(f32x2 a, f32x2 b) {
    f32x2 d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ f32x2 ffma2(f32x2 a, f32x2 b, f32x2 c) {
    f32x2 d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

// max(a, |b|, |c|) with fmaxf semantics (a NaN operand is ignored).
__device__ __forceinline__ float max_abs3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(fabsf(b)), "f"(fabsf(c)));
    return r;
}

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// Two fp32 -> packed bf16x2 (round to nearest even); `lo` lands in bits [0,16).
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

}  // namespace ctu

namespace ctu {

// ---------------------------------------------------------------------------
// Thread-block clusters of two CTAs sharing one tcgen05 MMA (cta_group::2).
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Address of the same shared variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t smem_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on an mbarrier of another CTA of the cluster (shared::cluster address).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar_addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar_addr), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait with cluster-scope acquire (for barriers that receive arrivals or
// transaction bytes from the peer CTA).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                                  uint32_t *err, uint32_t code) {
    const uint32_t addr = smem_u32(bar);
    if (mbar_try_wait_cluster(addr, parity)) return true;
    const uint64_t start = globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait_cluster(addr, parity)) return true;
        if ((i & 31u) == 0u) {
            if (abort_flag != nullptr && *abort_flag) return false;
            if (globaltimer() - start > kWaitLimitNs) {
                if (abort_flag != nullptr) *abort_flag = 1;
                atomicOr(err, code);
                return false;
            }
        }
    }
}

// 2D tile load into this CTA's shared memory whose completion (transaction bytes)
// is signalled on an mbarrier of the pair's leader CTA.  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void *smem_dst, const void *tmap, int x, int y,
                                                 uint32_t leader_bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
        "%3}], [%4];" ::"r"(smem_u32(smem_dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(leader_bar)
        : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t *smem_result, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Pair MMA (issued by the leader): A rows and B columns come half from each CTA's
// shared memory at the same offsets; each CTA's TMEM receives its 128 rows.
__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on the barrier at this offset in both CTAs of the pair once the leader's
// previously issued tcgen05 operations complete.
__device__ __forceinline__ void mma_commit_pair_both(uint64_t *bar) {
    const uint16_t mask = 0x3;
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(mask)
        : "memory");
}

// Arrive on the leader's own barrier only.
__device__ __forceinline__ void mma_commit_pair_local(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

}  // namespace ctu
