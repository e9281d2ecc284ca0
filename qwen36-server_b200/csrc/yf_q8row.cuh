// One warp, one (token, kv head) row: f16 loads and the Q8_0 quantize-and-store into a pool tile.
// Shared by the KV writer (yf_kvwrite.cu) and the fused attention prep (yf_prep.cu).
//
// Lane l owns dims [l*E, l*E+E) with E = D/32; a Q8_0 group of G = D/NB dims is G/E lanes, whose
// |x| maximum is a butterfly of xor-shuffles.  GGML's Q8_0 rule, bit-exact with the oracle:
// d = amax/127 and 1/d are IEEE divisions, q = roundf(x * (1/d)), d stored as f16 (RNE), q stored
// as the excess-128 byte q + 128.
#pragma once
#include <cuda_fp16.h>

#include "yf_device.cuh"

namespace yf {

// The lane's E f16 values of a row starting at `src` (16-byte aligned for E = 8, 8-byte for 4).
template <int E>
__device__ __forceinline__ void load_f16_row(const __half* src, float (&x)[E]) {
    static_assert(E == 4 || E == 8, "4 or 8 dims per lane");
    if constexpr (E == 4) {
        const uint2 w = *reinterpret_cast<const uint2*>(src);
        const __half2 a = *reinterpret_cast<const __half2*>(&w.x);
        const __half2 c = *reinterpret_cast<const __half2*>(&w.y);
        x[0] = __low2float(a);
        x[1] = __high2float(a);
        x[2] = __low2float(c);
        x[3] = __high2float(c);
    } else {
        const uint4 w = *reinterpret_cast<const uint4*>(src);
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const __half2 a = *reinterpret_cast<const __half2*>(&ww[k]);
            x[2 * k] = __low2float(a);
            x[2 * k + 1] = __high2float(a);
        }
    }
}

// Quantizes the warp's row (lane values x) and stores it as token t (0..15) of the 16-token
// `tile`, K (kv = 0) or V (kv = 1) half, in the tile layout of yf_pool_tile_offset.
template <int D, int NB>
__device__ __forceinline__ void q8_store_row(uint8_t* tile, int t, int kv, int lane, const float (&x)[D / 32]) {
    constexpr int E = D / 32;
    constexpr int G = D / NB;
    constexpr int LPG = G / E;
    constexpr int KS_OFF = 16 * D;
    constexpr int V_OFF = 16 * D + 32 * NB;
    constexpr int VS_OFF = 32 * D + 32 * NB;
    const int d0 = lane * E;
    const int grp = d0 / G;
    float amax = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) amax = fmaxf(amax, fabsf(x[e]));
#pragma unroll
    for (int off = 1; off < LPG; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
    int8_t qv[E];
#pragma unroll
    for (int e = 0; e < E; ++e) qv[e] = (int8_t)(int)roundf(__fmul_rn(x[e], id));

    if (kv == 0) {
        // dims d0..d0+E-1 are contiguous bytes of one K word
        const int b32 = d0 / 32, r = d0 % 32;
        uint8_t* dst = tile + b32 * 512 + ((t % 8) * 4 + r / 8) * 16 + (t / 8) * 8 + r % 8;
        if constexpr (E == 4) {
            uint32_t w = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) w |= (uint32_t)excess128(qv[e]) << (8 * e);
            *reinterpret_cast<uint32_t*>(dst) = w;
        } else {
            uint2 w = make_uint2(0, 0);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                w.x |= (uint32_t)excess128(qv[e]) << (8 * e);
                w.y |= (uint32_t)excess128(qv[4 + e]) << (8 * e);
            }
            *reinterpret_cast<uint2*>(dst) = w;
        }
        if (lane % LPG == 0) {
            const int off = KS_OFF + 2 * (((t % 8) * 2 + t / 8) * NB + grp);
            *reinterpret_cast<__half*>(tile + off) = __float2half_rn(d);
        }
    } else {
        const int tig = (t % 8) / 2, j = (t & 1) * 2 + t / 8;
#pragma unroll
        for (int e = 0; e < E; ++e) {
            const int dim = d0 + e, m = dim / 16, ii = dim % 16;
            tile[V_OFF + (m / 2) * 512 + ((ii % 8) * 4 + tig) * 16 + (m % 2) * 8 + (ii / 8) * 4 + j] =
                excess128(qv[e]);
        }
        if (lane % LPG == 0) {
            const int off = VS_OFF + 2 * ((tig * NB + grp) * 4 + j);
            *reinterpret_cast<__half*>(tile + off) = __float2half_rn(d);
        }
    }
}

}  // namespace yf
