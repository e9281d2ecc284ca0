// Device-side helpers: shared-memory addressing, mbarriers, 1-D bulk copies
// (TMA into this CTA only), warp MMA, and int8 -> f16 unpacking.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace yf {

// Bounds of an mbarrier wait: it gives up after the call's limit of global time (the pool's
// wait_limit_us option, 1 s by default) or kMaxWaitIters tries, whichever comes first (a
// try_wait may itself suspend for a hardware-defined interval, so the iteration bound alone
// could stretch to minutes).
constexpr uint32_t kMaxWaitIters = 1u << 20;

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before later async-proxy
// (bulk copy) accesses of the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Programmatic dependent launch.  A kernel launched with programmatic stream serialization may
// start while the previous kernel of its stream still runs; pdl_wait blocks until that kernel
// has completed and its memory is visible (a no-op for a kernel launched without the attribute),
// so the decode kernels call it before their first global-memory access.  pdl_trigger lets the
// next kernel's CTAs launch early (a KV write before the attention that reads it).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the given phase parity; false if it gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1; i < kMaxWaitIters; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 7u) == 0 && globaltimer_ns() - t0 > limit_ns) return false;
    }
    return false;
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
// Both addresses 16-byte aligned, bytes a multiple of 16.  This CTA is the only destination.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    uint64_t g;
    asm volatile("cvta.to.global.u64 %0, %1;" : "=l"(g) : "l"(src));
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(g), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ uint4 lds128(const void* p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(smem_u32(p)));
    return v;
}

__device__ __forceinline__ uint2 lds64(const void* p) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(smem_u32(p)));
    return v;
}

__device__ __forceinline__ uint32_t lds32(const void* p) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)));
    return v;
}

// D(16x8 f32) += A(16x16 f16, row) * B(16x8 f16, col).
__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Pool bytes -> exact f16 pairs.  The pool stores a Q8_0 value x in [-128, 127] as the excess-128
// byte x + 128; placed as the low mantissa byte of the f16 0x6400 (= 1024) it gives exactly
// 1024 + x + 128, and subtracting 1152 leaves x.
__device__ __forceinline__ uint8_t excess128(int8_t x) { return (uint8_t)((uint8_t)x ^ 0x80u); }
__device__ __forceinline__ uint32_t h2_sub_1152(uint32_t v) {
    uint32_t r;
    const uint32_t k = 0x64806480u;  // (1152, 1152) in f16
    asm("sub.f16x2 %0, %1, %2;" : "=r"(r) : "r"(v), "r"(k));
    return r;
}
// bytes 0,1 of a pool word -> f16x2 (lo = byte 0)
__device__ __forceinline__ uint32_t s8lo_to_h2(uint32_t wb) {
    return h2_sub_1152(__byte_perm(wb, 0x64646464u, 0x4140));
}
// bytes 2,3 of a pool word -> f16x2 (lo = byte 2)
__device__ __forceinline__ uint32_t s8hi_to_h2(uint32_t wb) {
    return h2_sub_1152(__byte_perm(wb, 0x64646464u, 0x4342));
}

__device__ __forceinline__ uint32_t h2mul(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

// {lo, hi} floats -> f16x2 with lo in the low half (round to nearest even).
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// ---- thread-block clusters: barrier and distributed shared memory ---------------------------

// Every thread of every CTA of the cluster arrives and waits (release / acquire ordering).
__device__ __forceinline__ void cluster_barrier() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Shared-memory address (shared::cluster window) of this CTA's location `p` in CTA `rank`.
__device__ __forceinline__ uint32_t dsmem_addr(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}

__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

__device__ __forceinline__ float4 ld_dsmem_f32x4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}

}  // namespace yf
