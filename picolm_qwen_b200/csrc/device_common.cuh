// device_common.cuh -- shared device helpers for the sm_100a attention kernels.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

#include "picoattn.h"

namespace picoattn {

// ---------------------------------------------------------------------------
// fp16 storage format of the reference's KV cache.
// ---------------------------------------------------------------------------

// fp32 -> fp16 bits with the reference's rounding (cpp/quant.hpp:102-135): the
// magnitude is rounded half-up (half an ulp added, then truncated), f32
// subnormals flush to a signed zero, NaN keeps a quiet payload bit.  This is
// not the hardware's round-to-nearest-even, so it is written as integer code.
// Adding half an ulp to the rebiased exponent|fraction word lets the carry move
// into the exponent, which covers the reference's mantissa-overflow branch and
// its overflow to inf.
__device__ __forceinline__ uint16_t f32_to_f16_ref(float f) {
    const uint32_t u = __float_as_uint(f);
    const uint32_t sgn = (u >> 16) & 0x8000u;
    const uint32_t be = (u >> 23) & 0xFFu;
    const uint32_t frac = u & 0x7FFFFFu;
    if (be == 0u) return (uint16_t)sgn;
    if (be == 0xFFu) return (uint16_t)(sgn | 0x7C00u | (frac ? 0x200u : 0u));
    const int e = (int)be - 112;
    if (e >= 31) return (uint16_t)(sgn | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sgn;
        const uint32_t sig = frac | 0x800000u;
        const uint32_t sh = (uint32_t)(14 - e);
        return (uint16_t)(sgn | ((sig + (1u << (sh - 1))) >> sh));
    }
    const uint32_t word = (((uint32_t)e << 23) | frac) + 0x1000u;
    return (uint16_t)(sgn | (word >> 13));
}

// Two values through f32_to_f16_ref, packed (first in the low half).  Magnitudes
// in [2^-14, 2^16) -- fp32 exponent fields 113..142, the reference's normal
// branch -- take the straight-line form of that branch: the word minus the
// exponent rebias plus half an ulp, shifted (a carry out of 2^16 - 16 still
// gives inf, as there); anything else goes through the full function.
__device__ __forceinline__ uint32_t f32x2_to_f16_ref(float a, float b) {
    const uint32_t ua = __float_as_uint(a), ub = __float_as_uint(b);
    const uint32_t ma = ua & 0x7FFFFFFFu, mb = ub & 0x7FFFFFFFu;
    if (ma - 0x38800000u < 0x0F000000u && mb - 0x38800000u < 0x0F000000u) {
        const uint32_t ha = ((ma - 0x37FFF000u) >> 13) | ((ua >> 16) & 0x8000u);
        const uint32_t hb = ((mb - 0x37FFF000u) >> 13) | ((ub >> 16) & 0x8000u);
        return ha | (hb << 16);
    }
    return (uint32_t)f32_to_f16_ref(a) | ((uint32_t)f32_to_f16_ref(b) << 16);
}

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialisation may start as soon as every CTA of the kernel before it in the
// stream has called pdl_trigger() (or exited); pdl_wait() returns when that
// kernel has completed and its memory is visible, and is a no-op without such a
// dependency.  Every decode kernel calls pdl_wait() in every CTA before it
// exits, so a kernel completes only after all the kernels before it, and it
// calls pdl_wait() before touching anything those kernels may still use.  A
// kernel launched without the attribute (any library or user kernel) starts
// only after its predecessor completed, so chains begin and end cleanly.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Named barrier `id` (1..15) over `count` threads (a multiple of 32): sync
// waits for the count; arrive adds this warp without waiting.  Shared-memory
// writes made before either are visible to the threads after the sync.
__device__ __forceinline__ void named_bar_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void named_bar_arrive(int id, int count) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Orders this thread's earlier generic-proxy global writes before later
// async-proxy (TMA) accesses that another thread issues after synchronising.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait for the phase with the given parity to complete.  A legitimate
// wait here lasts microseconds; after ~2 s the wait gives up, sets
// PICOATTN_DEV_TIMEOUT in the sticky status word and returns false so that the
// kernel finishes instead of hanging the device.  Once that bit is set (by any
// CTA of any kernel sharing the workspace) every other wait gives up at its
// next check, so a broken pipeline costs one timeout, not one per wait.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int* status) {
    const uint32_t a = smem_u32(bar);
    uint64_t t0 = 0;
    for (uint32_t it = 0;; ++it) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
        if ((it & 1023u) == 0u) {
            if (*reinterpret_cast<volatile unsigned int*>(status) & PICOATTN_DEV_TIMEOUT) return false;
            const uint64_t now = global_timer_ns();
            if (it == 0u) t0 = now;
            else if (now - t0 > 2000000000ull) {
                atomicOr(status, PICOATTN_DEV_TIMEOUT);
                return false;
            }
        }
    }
}

// Non-blocking probe: has the phase with the given parity completed?  A thread
// that issues tcgen05.mma stalls for the latency of any load it makes, and the
// tensor pipe idles meanwhile (~180 cycles for a try_wait, ~100 for this probe),
// so such a thread probes all the phases it needs at once and falls back to
// mbar_wait only when one is not complete yet.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// One-dimensional bulk copy global -> shared (TMA engine), completion counted
// in bytes on `bar`.  dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Bulk prefetch of `bytes` of global memory into L2 (TMA engine, no completion
// to wait for: a hint).  src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Per-thread asynchronous copies global -> shared through the load path (not
// the TMA engine): 16 bytes (L2 only) or 8 bytes, grouped per thread by
// commit_group; wait_group<N> returns when at most N of this thread's groups
// are still in flight.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// D = A(16x16 f16, row) * B(16x8 f16, col) + D, fp32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic: one instruction for two lanes'
// worth of adds), low half = first element.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}

}  // namespace picoattn
