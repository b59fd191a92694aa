// Shared device helpers for the sm_100a kernels: inline PTX wrappers for byte
// permutes, 16x8-bit dot products, mbarriers and bulk (TMA) copies, plus the
// bounded-wait policy every spin loop here follows.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#ifndef GP_DEVINL
#define GP_DEVINL __device__ __forceinline__
#endif

// Every device-side wait gives up after this many polls and records an error
// in the kernel's status word instead of hanging the GPU.
#ifndef GP_SPIN_LIMIT
#define GP_SPIN_LIMIT (1u << 22)
#endif

__host__ __device__ __forceinline__ int64_t gp_min64(int64_t a, int64_t b) { return a < b ? a : b; }

enum gp_dev_status : uint32_t {
    GP_DEV_OK = 0,
    GP_DEV_TIMEOUT_FULL = 1,     // consumer gave up waiting for a stage to land
    GP_DEV_TIMEOUT_EMPTY = 2,    // producer gave up waiting for a stage to drain
    GP_DEV_BAD_EXPERT = 4,       // an expert id outside [0, E)
    GP_DEV_BAD_SHAPE = 8,
    GP_DEV_FP16_RANGE = 16,      // a token value or an h value past the fp16 range (tensor-core path)
};

GP_DEVINL uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

// acc + a.lo16*b.byte0 + a.hi16*b.byte1  (signed 16-bit x signed 8-bit)
GP_DEVINL int dp2a_lo(uint32_t a, uint32_t b, int acc) {
    int r;
    asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(acc));
    return r;
}
// acc + a.lo16*b.byte2 + a.hi16*b.byte3
GP_DEVINL int dp2a_hi(uint32_t a, uint32_t b, int acc) {
    int r;
    asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(acc));
    return r;
}

GP_DEVINL uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

GP_DEVINL uint32_t lds32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
GP_DEVINL uint2 lds64(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}
GP_DEVINL uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
GP_DEVINL float ldsf(uint32_t addr) { return __uint_as_float(lds32(addr)); }
GP_DEVINL uint32_t lds16(uint32_t addr) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
    return v;
}

// ---- mbarrier ---------------------------------------------------------------
GP_DEVINL void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
GP_DEVINL void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
GP_DEVINL void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
GP_DEVINL void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
GP_DEVINL void mbar_arrive_cnt(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
GP_DEVINL bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: returns false (and leaves the barrier alone) after `limit`
// polls (GP_SPIN_LIMIT unless the kernel takes its limit at run time).
GP_DEVINL bool mbar_wait(uint32_t bar, uint32_t parity, uint32_t limit = GP_SPIN_LIMIT) {
    for (uint32_t i = 0; i < limit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// Bounded wait for a phase expected to take long: sleeps between polls so the
// waiting warp leaves the issue slots to the others.
GP_DEVINL bool mbar_wait_sleepy(uint32_t bar, uint32_t parity, uint32_t limit = GP_SPIN_LIMIT) {
    for (uint32_t i = 0; i < limit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        __nanosleep(256);
    }
    return false;
}

// 1-D bulk copy global -> shared (TMA engine), completion counted in bytes on bar.
// dst, src 16-byte aligned; bytes a multiple of 16.  No cluster multicast.
GP_DEVINL void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

GP_DEVINL void named_bar_sync(uint32_t id, uint32_t nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

GP_DEVINL float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---- grid-scope ordering (counters between CTAs) ----------------------------
GP_DEVINL void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
// Orders this thread's earlier generic-proxy accesses (an acquire of data that
// other CTAs wrote) before its later bulk-copy (async-proxy) reads of it.
GP_DEVINL void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
GP_DEVINL void red_release_add(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Returns the old value; releases this thread's (and, through a preceding
// warp/CTA barrier, its peers') writes and acquires those of earlier adders.
GP_DEVINL unsigned atom_add_acq_rel(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
GP_DEVINL unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Bounded wait for *p >= target (a counter other CTAs raise); false on timeout.
GP_DEVINL bool wait_geq(const unsigned* p, unsigned target) {
    for (uint32_t i = 0; i < GP_SPIN_LIMIT; ++i) {
        if (ld_acquire(p) >= target) return true;
        __nanosleep(32);
    }
    return false;
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue early / wait for the previous kernel's results.
GP_DEVINL void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
GP_DEVINL void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
