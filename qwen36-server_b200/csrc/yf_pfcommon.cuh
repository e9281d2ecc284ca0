// Pieces shared by the tcgen05 prefill kernels (yf_prefill_tc.cu at D=128, yf_prefill_tc256.cu
// at D=256): key visibility, the row max and exponentials of 64 S values, and the bounded
// mbarrier waits with their diagnostic tags.
#pragma once

#include "yf_device.cuh"
#include "yf_internal.h"
#include "yf_tc.cuh"

namespace yf {

// Key k (0..127) of the current key tile is visible: causal limit and page validity.
__device__ __forceinline__ bool key_ok(int k, int lim, uint32_t pm) { return k < lim && ((pm >> (k >> 4)) & 1u); }

// Max of 64 S values (raw dot products); masked keys do not count.
template <bool kMasked>
__device__ __forceinline__ float row_max64(const float (&v)[64], int k0, int lim, uint32_t pm) {
    float a = -INFINITY, b = -INFINITY;
#pragma unroll
    for (int c = 0; c < 64; c += 4) {
        float x0 = v[c], x1 = v[c + 1], x2 = v[c + 2], x3 = v[c + 3];
        if (kMasked) {
            x0 = key_ok(k0 + c, lim, pm) ? x0 : -INFINITY;
            x1 = key_ok(k0 + c + 1, lim, pm) ? x1 : -INFINITY;
            x2 = key_ok(k0 + c + 2, lim, pm) ? x2 : -INFINITY;
            x3 = key_ok(k0 + c + 3, lim, pm) ? x3 : -INFINITY;
        }
        a = max3f(a, x0, x1);
        b = max3f(b, x2, x3);
    }
    return fmaxf(a, b);
}

// p = 2^(s * scale_log2 - m) for 64 keys, stored as 32 f16x2 TMEM columns; returns sum(p).
template <bool kMasked>
__device__ __forceinline__ float exp_store64(const float (&v)[64], int k0, int lim, uint32_t pm, float sl2,
                                             float nm, uint32_t taddr) {
    uint32_t pk[32];
    float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < 32; ++c) {
        float2 x = ffma2(make_float2(v[2 * c], v[2 * c + 1]), sl2, nm);
        if (kMasked) {
            x.x = key_ok(k0 + 2 * c, lim, pm) ? x.x : -INFINITY;
            x.y = key_ok(k0 + 2 * c + 1, lim, pm) ? x.y : -INFINITY;
        }
        const float2 e = make_float2(fast_exp2(x.x), fast_exp2(x.y));
        if (c & 1)
            acc1 = fadd2(acc1, e);
        else
            acc0 = fadd2(acc0, e);
        pk[c] = pack_h2(e.x, e.y);
    }
    tmem_st32(taddr, pk);
    const float2 s = fadd2(acc0, acc1);
    return s.x + s.y;
}

// Diagnostic tag of a wait that gave up: role (1 control, 2 dequant, 3 softmax) in bits 14-15,
// barrier in bits 10-13, the awaited completion (low 10 bits) in bits 0-9.
enum : uint32_t { kBarRawFull, kBarRawFree, kBarKFull, kBarVFull, kBarKFree, kBarVFree, kBarSFull, kBarPFull,
                  kBarODone, kBarDrain, kBarIdle };
__host__ __device__ constexpr uint32_t wait_tag(uint32_t role, uint32_t bar, int use) {
    return (role << 14) | (bar << 10) | ((uint32_t)use & 1023u);
}

// Raises the CTA's abort flag and, for the first wait of the launch that gives up, records
// its tag in bits 16-31 of the status word next to YF_DEV_TIMEOUT.
__device__ __forceinline__ void give_up(volatile int* abort, uint32_t* status, uint32_t tag) {
    *abort = 1;
    const uint32_t old = atomicOr(status, YF_DEV_TIMEOUT);
    if (!(old & YF_DEV_TIMEOUT)) atomicOr(status, tag << 16);
}

// Bounded wait for the use-th completion (0-based) of `bar` (limit_ns of global time).
// A wait that gives up raises the CTA's abort flag, after which every role skips its
// remaining waits and drains quickly.
__device__ __forceinline__ bool wait_phase(uint64_t* bar, int use, volatile int* abort, uint32_t* status,
                                           uint64_t limit_ns, uint32_t tag) {
    if (*abort) return false;
    if (mbar_try_wait(bar, (uint32_t)use & 1u)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, (uint32_t)use & 1u)) return true;
        if ((i & 7u) == 0) {
            if (*abort) return false;
            if (globaltimer_ns() - t0 > limit_ns) break;
        }
    }
    give_up(abort, status, tag);
    return false;
}


}  // namespace yf
