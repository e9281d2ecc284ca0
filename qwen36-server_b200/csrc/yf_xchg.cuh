// Device side of the partial exchange over NVLink peer memory, shared by the stand-alone push /
// combine kernels (yf_exchange.cu) and the cluster decode kernel with the exchange fused in
// (yf_decode.cu).
//
// Exchange area of every rank (its own HBM, mapped by the others through CUDA IPC):
//   [2 buffers][world slots][slot_floats] f32 | meta: [world] u32 flags | u32 epoch | u32 status
//   | [kXMaxSlices] u32 slice steps | [2 buffers][world slots][slot_floats] u64 words
// Push / combine: step s = epoch + 1 writes buffer s & 1; rank r's partial goes into slot r of
// that buffer in every area, and then r stores s into flag r of every area (release, system
// scope).  A rank combines once every flag of its own area has reached s (acquire).
// Fused into the decode kernel: every value travels as one 64-bit word (float bits | step << 32)
// into the word buffers, so a reader polls the words themselves until they carry its step --
// no fence and no flag (the low-latency protocol of collective libraries, restated here).  Each
// output slice of the decode keeps its own step count (slice steps), as the same CTA role stores
// and merges that slice every call.
#pragma once

#include <cuda_fp16.h>

#include "yf_device.cuh"
#include "yf_internal.h"

namespace yf {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t* xmeta(uint8_t* area, size_t flags_off) {
    return reinterpret_cast<uint32_t*>(area + flags_off);
}

__device__ __forceinline__ float* xslot(unsigned long long area, uint32_t step, int world, long long slot_floats,
                                        int r) {
    return reinterpret_cast<float*>(area) + ((long long)(step & 1u) * world + r) * slot_floats;
}

// Raises this rank's flag of `step` in every area (after the caller's system-scope fence).
__device__ __forceinline__ void xraise(const unsigned long long* peers, int world, int rank, size_t flags_off,
                                       uint32_t step) {
    for (int k = 0; k < world; ++k)
        st_release_sys(reinterpret_cast<uint32_t*>(peers[k] + flags_off) + rank, step);
}

// 64-bit words: the value's bits low, the step high.  An aligned 8-byte access is single-copy
// atomic, so a reader never sees a value of one step with the step of another.
__device__ __forceinline__ unsigned long long ll_word(float v, uint32_t step) {
    return ((unsigned long long)step << 32) | __float_as_uint(v);
}
__device__ __forceinline__ void st_ll2(unsigned long long* p, unsigned long long a, unsigned long long b) {
    asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void st_ll1(unsigned long long* p, unsigned long long a) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(a) : "memory");
}
__device__ __forceinline__ ulonglong2 ld_ll2(const unsigned long long* p) {
    ulonglong2 v;
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long ld_ll1(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// Polls one word until it carries `step`; false once wait_ns have passed since t0.
__device__ __forceinline__ bool ll_wait1(const unsigned long long* p, uint32_t step, uint64_t t0, uint64_t wait_ns,
                                         float& a) {
    for (uint32_t it = 0;; ++it) {
        const unsigned long long v = ld_ll1(p);
        if ((uint32_t)(v >> 32) == step) {
            a = __uint_as_float((uint32_t)v);
            return true;
        }
        if ((it & 15u) == 15u && globaltimer_ns() - t0 > wait_ns) return false;
    }
}
// Polls two adjacent words (16-byte aligned) until both carry `step`.
__device__ __forceinline__ bool ll_wait2(const unsigned long long* p, uint32_t step, uint64_t t0, uint64_t wait_ns,
                                         float& a, float& b) {
    for (uint32_t it = 0;; ++it) {
        const ulonglong2 v = ld_ll2(p);
        if ((uint32_t)(v.x >> 32) == step && (uint32_t)(v.y >> 32) == step) {
            a = __uint_as_float((uint32_t)v.x);
            b = __uint_as_float((uint32_t)v.y);
            return true;
        }
        if ((it & 15u) == 15u && globaltimer_ns() - t0 > wait_ns) return false;
    }
}

// One thread: waits until every flag of the own area has reached `step`, giving up after wait_ns
// (then YF_DEV_TIMEOUT in the area's status word).  True when all arrived.
__device__ __forceinline__ bool xwait(uint32_t* meta, int world, uint32_t step, uint64_t wait_ns) {
    const uint64_t t0 = globaltimer_ns();
    for (int k = 0; k < world; ++k) {
        for (uint32_t it = 0;; ++it) {
            if ((int)(ld_acquire_sys(meta + k) - step) >= 0) break;
            if ((it & 31u) == 31u && globaltimer_ns() - t0 > wait_ns) {
                atomicOr(meta + world + 1, YF_DEV_TIMEOUT);
                return false;
            }
            __nanosleep(64);
        }
    }
    return true;
}

// Element e of the merged output (head group g, partial row r, float4 column c): head group g's
// parts are the slots of ranks s * n_hg + g (s < n_seq), O at offset 0 and natural-log lse at
// lse_off of each slot; row r = b * hq + j goes to output row b * Hq + g * hq + j.
// out = sum_s w_s o_s / sum_s w_s, w_s = e^(lse_s - max_s lse_s) (zeros without keys).
__device__ __forceinline__ void xmerge4(const uint8_t* area, uint32_t step, int world, long long slot_floats,
                                        long long lse_off, int n_hg, int n_seq, int rows, int hq, int Hq, int d4n,
                                        int e, __half* __restrict__ out) {
    const int g = e / (rows * d4n), r = (e / d4n) % rows, c = e % d4n;
    const unsigned long long base = reinterpret_cast<unsigned long long>(area);
    float M = -INFINITY;
    for (int s = 0; s < n_seq; ++s)
        M = fmaxf(M, __ldcg(xslot(base, step, world, slot_floats, s * n_hg + g) + lse_off + r));
    float L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (M != -INFINITY) {
        for (int s = 0; s < n_seq; ++s) {
            const float* sl = xslot(base, step, world, slot_floats, s * n_hg + g);
            const float lv = __ldcg(sl + lse_off + r);
            if (lv == -INFINITY) continue;
            const float w = fast_exp2((lv - M) * 1.4426950408889634f);
            L += w;
            const float4 v = __ldcg(reinterpret_cast<const float4*>(sl) + (size_t)r * d4n + c);
            acc.x = fmaf(w, v.x, acc.x);
            acc.y = fmaf(w, v.y, acc.y);
            acc.z = fmaf(w, v.z, acc.z);
            acc.w = fmaf(w, v.w, acc.w);
        }
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    const int b = r / hq, j = r % hq;
    uint2 pk;
    pk.x = pack_h2(acc.x * inv, acc.y * inv);
    pk.y = pack_h2(acc.z * inv, acc.w * inv);
    reinterpret_cast<uint2*>(out + ((size_t)b * Hq + (size_t)g * hq + j) * (size_t)(4 * d4n))[c] = pk;
}

}  // namespace yf
