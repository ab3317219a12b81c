// Device helpers shared by the add+RMSNorm and SiLU-and-mul kernels (sm_100a).
//
// bf16 is handled as raw 16-bit words: widening to fp32 is an exact shift, narrowing is the
// hardware round-to-nearest-even convert (cvt.rn.bf16x2.f32), the same rounding torch applies in
// Tensor.to(torch.bfloat16).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace ipl {

constexpr int kWarpSize = 32;

// Fault bits stored in the per-device fault word (see ipl_device_fault_flags).
constexpr uint32_t kFaultFullBarrierTimeout = 1u << 0;   // a consumer never saw its stage fill
constexpr uint32_t kFaultEmptyBarrierTimeout = 1u << 1;  // the producer never saw a stage drain
constexpr uint32_t kFaultCopyDrainTimeout = 1u << 2;     // a copy the producer issued never landed

// Bounded waits give up after this long (nanoseconds of %globaltimer). A stage fills within
// microseconds on a healthy GPU; the bound only exists so that a lost copy ends the kernel
// with a recorded fault instead of a hang. Test builds shorten it (IPL_WAIT_LIMIT_NS) so that a
// test can make a wait run out quickly.
#ifndef IPL_WAIT_LIMIT_NS
#define IPL_WAIT_LIMIT_NS 2000000000ull
#endif
constexpr uint64_t kWaitLimitNs = IPL_WAIT_LIMIT_NS;

// Per-device fault word (read by ipl_device_fault_flags). Defined here: the library is a single
// translation unit (ipl_b200.cu includes every kernel header).
__device__ uint32_t g_fault_word = 0;

__device__ __forceinline__ float bf16_lo(uint32_t packed) { return __uint_as_float(packed << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t packed) { return __uint_as_float(packed & 0xffff0000u); }
__device__ __forceinline__ float bf16_bits_to_float(uint16_t bits) {
    return __uint_as_float(static_cast<uint32_t>(bits) << 16);
}

// Two floats -> bf16x2 word (lo in bits 0..15), round to nearest even.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t packed;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(packed) : "f"(hi), "f"(lo));
    return packed;
}
// fp32 -> fp8 e4m3 (OCP E4M3FN: bias 7, max 448, no infinities), round to nearest even,
// saturating to +-448; NaN -> 0x7F.
__device__ __forceinline__ uint8_t float_to_e4m3(float value) {
    uint16_t packed;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(packed) : "f"(0.0f), "f"(value));
    return static_cast<uint8_t>(packed & 0xffu);
}
__device__ __forceinline__ uint16_t float_to_bf16_bits(float value) {
    return static_cast<uint16_t>(pack_bf16x2(value, 0.0f) & 0xffffu);
}

// ---- packed fp32 pairs (sm_100 f32x2 arithmetic: one instruction for two IEEE fp32 ops) ------

using F32x2 = unsigned long long;  // .b64 register pair: low half = first float

__device__ __forceinline__ F32x2 f32x2_make(float lo, float hi) {
    F32x2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f32x2_split(F32x2 v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ F32x2 f32x2_add(F32x2 a, F32x2 b) {
    F32x2 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ F32x2 f32x2_mul(F32x2 a, F32x2 b) {
    F32x2 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ F32x2 f32x2_fma(F32x2 a, F32x2 b, F32x2 c) {
    F32x2 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
// bf16x2 word -> fp32 pair (exact).
__device__ __forceinline__ F32x2 bf16x2_widen(uint32_t packed) {
    return f32x2_make(__uint_as_float(packed << 16), __uint_as_float(packed & 0xffff0000u));
}
// fp32 pair -> two e4m3 bytes (low element in the low byte), saturating, round to nearest even.
__device__ __forceinline__ uint32_t f32x2_to_e4m3x2(F32x2 v) {
    float lo, hi;
    f32x2_split(v, lo, hi);
    uint16_t packed;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(packed) : "f"(hi), "f"(lo));
    return packed;
}

// fp32 pair -> bf16x2 word, round to nearest even.
__device__ __forceinline__ uint32_t f32x2_to_bf16x2(F32x2 v) {
    float lo, hi;
    f32x2_split(v, lo, hi);
    return pack_bf16x2(lo, hi);
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---- global memory vectors -------------------------------------------------------------------

struct alignas(16) U32x4 {
    uint32_t v[4];
};
struct alignas(32) U32x8 {
    uint32_t v[8];
};

// Streaming read-only loads: the data is used once, so keep it out of L1.
__device__ __forceinline__ U32x4 ld_stream_v4(const void* p) {
    U32x4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.v[0]), "=r"(r.v[1]), "=r"(r.v[2]), "=r"(r.v[3])
                 : "l"(p));
    return r;
}
__device__ __forceinline__ U32x8 ld_stream_v8(const void* p) {
    U32x8 r;
    asm volatile("ld.global.nc.L1::no_allocate.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r.v[0]), "=r"(r.v[1]), "=r"(r.v[2]), "=r"(r.v[3]), "=r"(r.v[4]),
                   "=r"(r.v[5]), "=r"(r.v[6]), "=r"(r.v[7])
                 : "l"(p));
    return r;
}
// Coherent 16-byte load that does not allocate in L1 (the data may be rewritten by this kernel).
__device__ __forceinline__ U32x4 ld_v4(const void* p) {
    U32x4 r;
    asm volatile("ld.global.L1::no_allocate.v4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.v[0]), "=r"(r.v[1]), "=r"(r.v[2]), "=r"(r.v[3])
                 : "l"(p));
    return r;
}
// Coherent 32-byte load (256-bit, sm_100), not allocating in L1; p 32-byte aligned.
__device__ __forceinline__ U32x8 ld_v8(const void* p) {
    U32x8 r;
    asm volatile("ld.global.L1::no_allocate.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r.v[0]), "=r"(r.v[1]), "=r"(r.v[2]), "=r"(r.v[3]), "=r"(r.v[4]), "=r"(r.v[5]),
                   "=r"(r.v[6]), "=r"(r.v[7])
                 : "l"(p));
    return r;
}
// Read-only 4-byte load, ordered after the volatile loads issued before it in program order.
__device__ __forceinline__ float ld_nc_f32(const float* p) {
    float r;
    asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(r) : "l"(p));
    return r;
}
// Read-only 16-byte load that may stay in L1 (data every CTA on the SM reads, e.g. gamma).
__device__ __forceinline__ U32x4 ld_shared_ro_v4(const void* p) {
    U32x4 r;
    asm volatile("ld.global.nc.v4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.v[0]), "=r"(r.v[1]), "=r"(r.v[2]), "=r"(r.v[3])
                 : "l"(p));
    return r;
}
__device__ __forceinline__ void st_v2(void* p, uint32_t a, uint32_t b) {
    asm volatile("st.global.v2.b32 [%0], {%1,%2};" ::"l"(p), "r"(a), "r"(b) : "memory");
}
__device__ __forceinline__ void st_v4(void* p, const U32x4& r) {
    asm volatile("st.global.v4.b32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(r.v[0]), "r"(r.v[1]),
                 "r"(r.v[2]), "r"(r.v[3])
                 : "memory");
}
__device__ __forceinline__ void st_v8(void* p, const U32x8& r) {
    asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(r.v[0]),
                 "r"(r.v[1]), "r"(r.v[2]), "r"(r.v[3]), "r"(r.v[4]), "r"(r.v[5]), "r"(r.v[6]),
                 "r"(r.v[7])
                 : "memory");
}

// ---- shared memory ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ U32x4 lds_v4(uint32_t addr) {
    U32x4 r;
    asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.v[0]), "=r"(r.v[1]), "=r"(r.v[2]), "=r"(r.v[3])
                 : "r"(addr));
    return r;
}
__device__ __forceinline__ void sts_pairs(uint32_t addr, F32x2 a, F32x2 b) {
    asm volatile("st.shared.v2.b64 [%0], {%1, %2};" ::"r"(addr), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void lds_pairs(uint32_t addr, F32x2& a, F32x2& b) {
    asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "r"(addr) : "memory");
}
__device__ __forceinline__ float lds_f32(uint32_t addr) {
    float r;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(r) : "r"(addr));
    return r;
}
__device__ __forceinline__ uint16_t lds_u16(uint32_t addr) {
    uint16_t r;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(r) : "r"(addr));
    return r;
}

// ---- mbarrier + bulk async copy (TMA, non-tensor form) ----------------------------------------

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
// Tests the phase; if it is not complete the thread is suspended (it issues nothing) until the
// phase completes or about kWaitSliceNs pass, so waiting warps leave the issue slots to working
// ones.
constexpr uint32_t kWaitSliceNs = 100000;
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity), "r"(kWaitSliceNs)
        : "memory");
    return done != 0;
}

// Waits for the phase with the given parity to complete. Returns false (after recording
// `fault_bit` in the device fault word) if it has not completed within kWaitLimitNs, or as soon
// as *abort becomes nonzero (another warp of the CTA gave up).
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  volatile int* abort, uint32_t fault_bit) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = global_timer_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (global_timer_ns() - start > kWaitLimitNs) {
            atomicOr(&g_fault_word, fault_bit);
            *abort = 1;
            return false;
        }
    }
}

// Waits for the phase with the given parity to complete, bounded by kWaitLimitNs only (not by
// the abort flag): used to let copies already issued land before their CTA exits. Records
// `fault_bit` and returns false when the limit passes.
__device__ __forceinline__ bool mbar_wait_timed(uint32_t bar, uint32_t parity, uint32_t fault_bit) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = global_timer_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - start > kWaitLimitNs) {
            atomicOr(&g_fault_word, fault_bit);
            return false;
        }
    }
}

// Spins (with the same bound) until the shared counter reaches `target`.
__device__ __forceinline__ bool spin_until_at_least(const int* counter, int target, volatile int* abort,
                                                    uint32_t fault_bit) {
    const volatile int* c = counter;
    if (*c >= target) return true;
    const uint64_t start = global_timer_ns();
    for (uint32_t spin = 1;; ++spin) {
        if (*c >= target) return true;
        if ((spin & 63u) == 0) {
            if (*abort) return false;
            if (global_timer_ns() - start > kWaitLimitNs) {
                atomicOr(&g_fault_word, fault_bit);
                *abort = 1;
                return false;
            }
        }
        __nanosleep(32);
    }
}

// Asynchronous 16-byte copy global -> shared memory of this CTA (cp.async, allocating in L1, so
// the SM's other CTAs reading the same source hit L1); completion by cp_async_wait_all. dst and
// src 16-byte aligned. The copied bytes occupy no registers while in flight.
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
// Waits until every cp.async this thread issued has landed (visible to this thread; a barrier
// after it makes them visible to the CTA).
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Bulk copy global -> shared (this CTA), completion counted on `bar` in bytes.
// dst, src 16-byte aligned; bytes a multiple of 16. The L2 policy hint marks the source lines
// evict-first: every byte is read exactly once.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(policy)
        : "memory");
}
// Bulk prefetch of [src, src + bytes) into L2 (src 16-byte aligned, bytes a multiple of 16). A
// hint only: nothing is copied anywhere a later write could leave stale, since L2 is where every
// SM's loads and stores meet.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
// The same for any 2-byte aligned range: the 16-byte aligned span that covers [p, p + bytes)
// (every byte of which shares a 16-byte block with a byte of the range, so it is mapped).
__device__ __forceinline__ void prefetch_span_l2(const void* p, uint32_t bytes) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uintptr_t base = a & ~static_cast<uintptr_t>(15);
    const uint32_t span = (static_cast<uint32_t>(a - base) + bytes + 15u) & ~15u;
    bulk_prefetch_l2(reinterpret_cast<const void*>(base), span);
}
// Prefetch of the 128-byte line holding p into L2 (a hint, like bulk_prefetch_l2).
__device__ __forceinline__ void prefetch_l2(const void* p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p) : "memory");
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

// ---- named barriers + programmatic dependent launch ----------------------------------------

__device__ __forceinline__ void named_barrier_sync(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Wait until the grid this launch depends on (the previous kernel in the stream, when launched
// with programmatic stream serialisation) has completed and its writes are visible. A no-op
// for a normal launch.
__device__ __forceinline__ void grid_dependency_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
// Allow the next kernel in the stream to begin launching (its own dependency wait still orders
// its reads after this grid's completion).
__device__ __forceinline__ void grid_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- thread-block clusters and distributed shared memory -----------------------------------

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t rank;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
    return rank;
}
__device__ __forceinline__ uint32_t cluster_nctarank() {
    uint32_t n;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(n));
    return n;
}
// The cluster barrier is a hardware barrier over every thread of every CTA of the cluster, whose
// CTAs the GPU schedules together: it completes once all of them have arrived, with no spin of
// ours. Each thread must reach every arrive and wait (`.aligned`: whole warps, converged).
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The shared::cluster address of CTA `rank`'s copy of the variable at this CTA's `addr`.
__device__ __forceinline__ uint32_t map_shared_to_rank(uint32_t addr, uint32_t rank) {
    uint32_t mapped;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(mapped) : "r"(addr), "r"(rank));
    return mapped;
}
__device__ __forceinline__ void st_shared_cluster_f32(uint32_t addr, float value) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(value) : "memory");
}

__device__ __forceinline__ float warp_sum(float value) {
#pragma unroll
    for (int offset = kWarpSize / 2; offset > 0; offset >>= 1) {
        value += __shfl_xor_sync(0xffffffffu, value, offset);
    }
    return value;
}

}  // namespace ipl
