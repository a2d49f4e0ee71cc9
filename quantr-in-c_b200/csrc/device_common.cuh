// device_common.cuh -- sm_100a device helpers shared by the GEMV kernels:
// programmatic dependent launch, mbarriers with bounded waits, bulk copies,
// unaligned shared-memory word loads, and the x86-exact int8 rounding.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "kernels.cuh"

namespace qr {

constexpr unsigned long long kWaitNs = 250000000ull;  // bounded waits: 250 ms

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// Named barrier `id` (1..15) over `n` threads, a multiple of 32: only the
// warps that reach it take part (barrier 0 is __syncthreads).
__device__ __forceinline__ void bar_sync_n(int id, int n)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__device__ __forceinline__ uint32_t sptr(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long gtimer()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sptr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sptr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sptr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(sptr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait that may suspend the thread for up to `ns` nanoseconds while the
// phase is incomplete (it resumes as soon as the phase completes).
__device__ __forceinline__ bool mbar_try_wait_for(uint64_t* bar, uint32_t parity, uint32_t ns)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(sptr(bar)), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}

// Waits for the barrier phase with parity `parity`.  Gives up after kWaitNs
// (recording DEV_ERR_WAIT_TIMEOUT in *err when given) or as soon as *abort
// becomes non-zero (another role of the CTA gave up).  Never spins unboundedly.
// suspend_ns > 0 lets each poll suspend the thread that long (fewer polls,
// fewer issue slots taken from the warps that have work).
// The polling loop is out of line: every wait site's fast path (the phase is
// already complete) stays a single instruction in the caller's hot code.
static __device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, int* err, volatile int* abort,
                                            unsigned suspend_ns)
{
    const unsigned long long t0 = gtimer();
    while (!(suspend_ns ? mbar_try_wait_for(bar, parity, suspend_ns) : mbar_try_wait(bar, parity))) {
        if (abort && *abort) return false;
        if (gtimer() - t0 > kWaitNs) {
            if (err) atomicExch(err, DEV_ERR_WAIT_TIMEOUT);
            if (abort) *abort = 1;
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err,
                                                  volatile int* abort = nullptr, unsigned suspend_ns = 0)
{
    if (mbar_try_wait(bar, parity)) return true;
    return mbar_wait_slow(bar, parity, err, abort, suspend_ns);
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            sptr(dst)),
        "l"(src), "r"(bytes), "r"(sptr(bar))
        : "memory");
}

// Explicit shared-memory accesses by 32-bit shared-window address (always
// LDS/STS, never generic loads).
__device__ __forceinline__ uint4 lds128(uint32_t a)
{
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a)
{
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a)
{
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ float ldsf(uint32_t a)
{
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ void stsf(uint32_t a, float v)
{
    asm volatile("st.shared.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}
// 32-bit word at an arbitrary shared byte address (two aligned loads).
__device__ __forceinline__ uint32_t lds32_u(uint32_t a)
{
    const uint32_t b = a & ~3u;
    return __funnelshift_r(lds32(b), lds32(b + 4), (a & 3) * 8);
}
// N words from an arbitrary shared byte address.
template <int N>
__device__ __forceinline__ void lds_words_u(uint32_t a, uint32_t* out)
{
    uint32_t r[N + 1];
    const uint32_t b = a & ~3u, sh = (a & 3) * 8;
#pragma unroll
    for (int k = 0; k <= N; ++k) r[k] = lds32(b + 4 * k);
#pragma unroll
    for (int k = 0; k < N; ++k) out[k] = __funnelshift_r(r[k], r[k + 1], sh);
}

// 32-bit word starting at an arbitrary shared-memory byte offset `off`.
__device__ __forceinline__ uint32_t ld_u32(const uint32_t* s32, uint32_t off)
{
    const uint32_t a = s32[off >> 2], b = s32[(off >> 2) + 1];
    return __funnelshift_r(a, b, (off & 3) * 8);
}

// N consecutive 32-bit words starting at an arbitrary byte offset.
template <int N>
__device__ __forceinline__ void ld_words(const uint32_t* s32, uint32_t off, uint32_t* out)
{
    uint32_t r[N + 1];
    const uint32_t base = off >> 2, sh = (off & 3) * 8;
#pragma unroll
    for (int k = 0; k <= N; ++k) r[k] = s32[base + k];
#pragma unroll
    for (int k = 0; k < N; ++k) out[k] = __funnelshift_r(r[k], r[k + 1], sh);
}

// (int8_t)lrintf(v) as the x86-64 reference computes it: lrintf converts to a
// 64-bit long (cvtss2si), and a NaN or |v| >= 2^63 yields the "integer
// indefinite" 0x8000000000000000, whose low byte is 0.  CUDA's conversions
// saturate instead, so out-of-range values are mapped explicitly.  (Reached
// when a denormal block scale makes 1/d overflow to infinity.)
__device__ __forceinline__ int8_t lrintf_to_i8(float v)
{
    return fabsf(v) < 9.2233720368547758e18f ? (int8_t)__float2ll_rn(v) : (int8_t)0;
}

// 16-byte cp.async (global -> shared, bypassing L1) and its group fences.
// The copies of a thread are complete and visible to it after cp_wait<N>()
// leaves at most N of its newest groups pending; other threads see them after
// a barrier.
__device__ __forceinline__ void cp16(uint32_t dst, const void* src)
{
    asm volatile("cp.async.cg.shared.global.L2::128B [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait()
{
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// dp4a with unsigned bytes in `a` and signed bytes in `b`.
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c)
{
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Spreads bits 0,2,4,6 of a byte to bit 4 of byte lanes 0..3.  Collisions of
// the multiply only carry into bits 11, 17 and 23, which the mask drops.
__device__ __forceinline__ uint32_t spread_even_bits_to_b4(uint32_t hb)
{
    return ((hb & 0x55u) * 0x410410u) & 0x10101010u;
}

} // namespace qr
