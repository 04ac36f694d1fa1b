// Device helpers for sm_100a: bulk-copy (TMA engine) + mbarrier pipeline, programmatic
// dependent launch, bounded waits, system-scope flag operations for NVLink peers.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define NCM_FULL 0xffffffffu

// Error word bits written by kernels (read back by the host after synchronising).
#define NCM_DEVERR_MBAR_TIMEOUT 0x1
#define NCM_DEVERR_PEER_TIMEOUT 0x2
#define NCM_DEVERR_BAD_ARG 0x4
#define NCM_DEVERR_CTX_FULL 0x8   // a decode step started at or past the context limit

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
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

// Bounded wait on an mbarrier phase.  Returns false (and the caller flags an error)
// if the phase has not completed within `limit_ns` of global time.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
    uint32_t addr = smem_u32(bar);
    uint32_t done = 0;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(done) : "r"(addr), "r"(parity) : "memory");
    if (done) return true;
    uint64_t t0 = global_timer_ns();
    while (true) {
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
            : "=r"(done) : "r"(addr), "r"(parity) : "memory");
        if (done) return true;
        if (global_timer_ns() - t0 > limit_ns) return false;
    }
}

// CTA-scope flags in shared memory: release store / acquire load, and a bounded wait for
// a flag to reach a value (false after limit_ns).
__device__ __forceinline__ uint32_t ld_acquire_cta(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_cta(uint32_t* p, uint32_t v) {
    asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}
__device__ __forceinline__ bool flag_wait_geq(const uint32_t* p, uint32_t v, uint64_t limit_ns) {
    if (ld_acquire_cta(p) >= v) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 1;; ++i) {
        if (ld_acquire_cta(p) >= v) return true;
        if ((i & 1023) == 0 && global_timer_ns() - t0 > limit_ns) return false;
    }
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// Untiled bulk copy global -> this CTA's shared memory, completion signalled on `bar`.
// Both addresses 16-byte aligned, bytes a multiple of 16 (checked by the host).
// Plain load: no cluster multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

// Programmatic dependent launch (PDL).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// System-scope release store / acquire load for cross-GPU flags.
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys(unsigned* p, unsigned v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
// Spins (no sleep: the waiting CTA has nothing else to do) until *p >= v; false once
// limit_ns has passed, the clock being read every 256 polls.
__device__ __forceinline__ bool wait_flag_sys(const unsigned* p, unsigned v, uint64_t limit_ns);
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ bool wait_flag_sys(const unsigned* p, unsigned v, uint64_t limit_ns) {
    if (ld_acquire_sys(p) >= v) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 1;; ++i) {
        if (ld_acquire_sys(p) >= v) return true;
        if ((i & 255u) == 0 && global_timer_ns() - t0 > limit_ns) return false;
    }
}

__device__ __forceinline__ void set_dev_error(int* err, int bits) {
    if (err) atomicOr(err, bits);
}

// Exact f16 -> f32 (q8.rs:3626-3642 fast_f16_to_f32 is exact too); hardware cvt.
__device__ __forceinline__ float f16_bits_to_f32(uint32_t bits) {
    float f;
    unsigned short h = (unsigned short)(bits & 0xffff);
    asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h));
    return f;
}
