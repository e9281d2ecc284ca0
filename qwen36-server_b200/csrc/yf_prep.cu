// Fused attention prep + Q8_0 KV append: replaces the engine's attn_prepare_decode (one kernel
// for the q/k RMSNorms with their own weights, partial RoPE of the first rope_dim dims, the
// gate half of the q projection split out, and V to f16;
// docs/research/2026-09-16-head-to-head-llamacpp-and-phase-profile.md:181-216) followed by
// kv_append_paged_f16 / launch_append_multi (docs/plans/2026-08-27-tiered-kv-cache.md:61-64):
// K leaves this kernel as Q8_0 pool bytes instead of an f16 tensor that a second launch reads.
//
// One warp per (new row, head slot); the first ceil(Hq/4) slots take four q heads each (norm, RoPE,
// q and gate out; the weights and cos/sin loaded once for the four), the next Hkv the kv heads (k: norm, RoPE, rounded to f16 as the unfused path stores it,
// then Q8_0 into the pool; v: Q8_0 into the pool).  Every float operation is an explicit IEEE
// round-to-nearest operation in a fixed order (no contraction, the sum of squares in lane order
// then an xor butterfly 16, 8, 4, 2, 1), so the oracle reproduces q, gate and the pool bytes
// exactly.  RoPE is the rotate-half (NeoX) form on dims [0, rope_dim) with the caller's cos/sin
// tables (the engine's rope cache): out[i] = x[i] c - x[i+h] s, out[i+h] = x[i+h] c + x[i] s,
// h = rope_dim/2, c/s = table[pos][i].
#include <cuda_fp16.h>

#include "yf_device.cuh"
#include "yf_internal.h"
#include "yf_q8row.cuh"

namespace yf {
namespace {

constexpr int kPrepWarps = 4;
constexpr int kPrepQHeads = 4;  // q heads per warp

struct PrepParams {
    uint8_t* layer_base;
    int n_pages;
    int H;
    long long phb;
    int Hq;
    const __half* qg;   // [T, Hq, 2D]: q then gate per head
    const __half* k;    // [T, H, D]
    const __half* v;    // [T, H, D]
    const float* wq;    // [D]
    const float* wk;    // [D]
    float eps;
    float w_offset;     // the norm multiplies by (w + w_offset)
    const float* cosb;  // [rope_rows][rope_dim / 2]
    const float* sinb;
    int rope_dim;
    int rope_rows;
    const int32_t* cu_rows;
    const int32_t* start_pos;
    const uint32_t* bt;
    int max_blocks;
    int max_rows;
    __half* q_out;      // [T, Hq, D]
    __half* gate_out;   // [T, Hq, D]
    uint32_t* status;
};

template <int E>
__device__ __forceinline__ void store_f16_row(__half* dst, const float (&x)[E]) {
    uint32_t w[E / 2];
#pragma unroll
    for (int k = 0; k < E / 2; ++k) w[k] = pack_h2(x[2 * k], x[2 * k + 1]);
    if constexpr (E == 4)
        *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
    else
        *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
}

// RMSNorm of the warp's row (lane values x, dims lane*E ..) times wf = (w + w_offset), then RoPE
// with the lane's cos/sin values c, s of the row's position.
template <int D>
__device__ __forceinline__ void norm_rope(const PrepParams& p, const float (&wf)[D / 32], const float (&c)[D / 32],
                                          const float (&s)[D / 32], int lane, float (&x)[D / 32]) {
    constexpr int E = D / 32;
    const int d0 = lane * E;
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) ss = __fadd_rn(ss, __fmul_rn(x[e], x[e]));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
    const float mean = __fmul_rn(ss, 1.0f / D);  // D is a power of two: exact
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = __fmul_rn(__fmul_rn(x[e], r), wf[e]);
    if (p.rope_dim == 0) return;
    const int half = p.rope_dim >> 1;
    float part[E];
#pragma unroll
    for (int e = 0; e < E; ++e) part[e] = __shfl_xor_sync(0xffffffffu, x[e], half / E);
    if (d0 >= p.rope_dim) return;
#pragma unroll
    for (int e = 0; e < E; ++e)
        x[e] = d0 < half ? __fsub_rn(__fmul_rn(x[e], c[e]), __fmul_rn(part[e], s[e]))
                         : __fadd_rn(__fmul_rn(x[e], c[e]), __fmul_rn(part[e], s[e]));
}

// The lane's norm weights (w + w_offset) and the position's cos/sin values, loaded once per warp.
template <int E>
__device__ __forceinline__ void load_row_consts(const PrepParams& p, const float* w, int pos, int lane,
                                                float (&wf)[E], float (&c)[E], float (&s)[E]) {
    const int d0 = lane * E;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        wf[e] = __fadd_rn(__ldg(w + d0 + e), p.w_offset);
        c[e] = 0.f;
        s[e] = 0.f;
    }
    if (p.rope_dim == 0 || d0 >= p.rope_dim) return;
    const int half = p.rope_dim >> 1, j0 = d0 % half;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        c[e] = __ldg(p.cosb + (size_t)pos * half + j0 + e);
        s[e] = __ldg(p.sinb + (size_t)pos * half + j0 + e);
    }
}

template <int D, int NB, int TPP>
__global__ void __launch_bounds__(kPrepWarps * 32) attn_prep_kernel(const PrepParams p) {
    pdl_trigger();  // the attention kernel that follows may be scheduled now (it waits for this one)
    constexpr int E = D / 32;
    constexpr int TB = 32 * D + 64 * NB;
    constexpr int P = TPP * 16;
    const int lane = threadIdx.x & 31;
    const int wi = blockIdx.x * kPrepWarps + (threadIdx.x >> 5);
    const int b = blockIdx.y;
    const int QW = (p.Hq + kPrepQHeads - 1) / kPrepQHeads;  // q-head warps per row
    const int S = QW + p.H;
    const int i = wi / S, slot = wi % S;
    const int r0 = p.cu_rows[b], n = p.cu_rows[b + 1] - r0;
    if (i == 0 && slot == 0 && lane == 0 && (n > p.max_rows || n < 0)) atomicOr(p.status, YF_DEV_BAD_ROWS);
    if (i >= n || i >= p.max_rows) return;
    const int row = r0 + i;
    const int pos = p.start_pos[b] + i;
    if (pos < 0 || (p.rope_dim > 0 && pos >= p.rope_rows)) {
        if (lane == 0) atomicOr(p.status, YF_DEV_BAD_POS);
        return;
    }
    const int d0 = lane * E;
    float x[E], wf[E], c[E], s[E];
    if (slot < QW) {
        // kPrepQHeads q heads of the row: the weights and cos/sin are loaded once for all of them
        load_row_consts<E>(p, p.wq, pos, lane, wf, c, s);
#pragma unroll
        for (int j = 0; j < kPrepQHeads; ++j) {
            const int h = slot * kPrepQHeads + j;
            if (h >= p.Hq) break;
            const __half* src = p.qg + ((size_t)row * p.Hq + h) * (2 * D);
            load_f16_row<E>(src + d0, x);
            norm_rope<D>(p, wf, c, s, lane, x);
            store_f16_row<E>(p.q_out + ((size_t)row * p.Hq + h) * D + d0, x);
            // the gate half, unchanged
            __half* go = p.gate_out + ((size_t)row * p.Hq + h) * D + d0;
            if constexpr (E == 4)
                *reinterpret_cast<uint2*>(go) = *reinterpret_cast<const uint2*>(src + D + d0);
            else
                *reinterpret_cast<uint4*>(go) = *reinterpret_cast<const uint4*>(src + D + d0);
        }
        return;
    }
    const int h = slot - QW;
    if (pos >= p.max_blocks * P) {
        if (lane == 0) atomicOr(p.status, YF_DEV_BAD_POS);
        return;
    }
    const uint32_t page = p.bt[(size_t)b * p.max_blocks + pos / P];
    if (page >= (uint32_t)p.n_pages) {
        if (lane == 0) atomicOr(p.status, YF_DEV_BAD_PAGE);
        return;
    }
    uint8_t* tile = p.layer_base + ((size_t)page * p.H + h) * p.phb + ((pos % P) / 16) * TB;
    const int t = pos % 16;
    load_row_consts<E>(p, p.wk, pos, lane, wf, c, s);
    load_f16_row<E>(p.k + ((size_t)row * p.H + h) * D + d0, x);
    norm_rope<D>(p, wf, c, s, lane, x);
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = __half2float(__float2half_rn(x[e]));  // K as the f16 tensor it replaces
    q8_store_row<D, NB>(tile, t, 0, lane, x);
    load_f16_row<E>(p.v + ((size_t)row * p.H + h) * D + d0, x);
    q8_store_row<D, NB>(tile, t, 1, lane, x);
}

template <int D, int NB, int TPP>
int launch_prep(const PrepParams& p, int batch, int max_rows, cudaStream_t s) {
    const long long warps = (long long)max_rows * ((p.Hq + kPrepQHeads - 1) / kPrepQHeads + p.H);
    const dim3 grid((unsigned)((warps + kPrepWarps - 1) / kPrepWarps), batch);
    attn_prep_kernel<D, NB, TPP><<<grid, kPrepWarps * 32, 0, s>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? YF_OK : cuda_fail(e, "attention prep launch");
}

}  // namespace
}  // namespace yf

using namespace yf;

extern "C" int yf_attn_prepare_append(yf_pool* pool, int32_t layer, int32_t n_q_heads, const void* qg, const void* k,
                                      const void* v, const float* q_norm_w, const float* k_norm_w, float eps,
                                      int32_t norm_weight_offset, const float* rope_cos, const float* rope_sin,
                                      int32_t rope_dim, int32_t rope_rows, const int32_t* cu_rows,
                                      const int32_t* start_pos, const uint32_t* block_table, int32_t max_blocks,
                                      int32_t batch, int32_t max_rows, void* q_out, void* gate_out, void* stream) {
    if (!pool) return fail(YF_E_INVALID, "pool is null");
    if (!pool->base) return fail(YF_E_INVALID, "host-only pool has no device memory");
    if (batch < 0 || max_rows < 0) return fail(YF_E_INVALID, "batch %d or max_rows %d < 0", batch, max_rows);
    if (batch == 0 || max_rows == 0) return YF_OK;
    if (batch > 65535) return fail(YF_E_UNSUPPORTED, "batch %d > 65535", batch);
    const yf_pool_desc& d = pool->desc;
    const int D = d.head_dim, E = D / 32;
    if (layer < 0 || layer >= d.n_layers) return fail(YF_E_RANGE, "layer %d out of range", layer);
    if (n_q_heads < d.n_kv_heads || n_q_heads % d.n_kv_heads)
        return fail(YF_E_INVALID, "n_q_heads %d is not a multiple of n_kv_heads %d", n_q_heads, d.n_kv_heads);
    if (max_blocks < 1) return fail(YF_E_INVALID, "max_blocks %d < 1", max_blocks);
    if (!qg || !k || !v || !q_norm_w || !k_norm_w || !cu_rows || !start_pos || !block_table || !q_out || !gate_out)
        return fail(YF_E_INVALID, "null device pointer");
    if (!aligned(qg, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(q_out, 16) || !aligned(gate_out, 16))
        return fail(YF_E_INVALID, "qg, k, v, q_out and gate_out must be 16-byte aligned");
    if (!(eps >= 0.f) || eps > 1.f) return fail(YF_E_INVALID, "eps must be in [0, 1]");
    if (norm_weight_offset != 0 && norm_weight_offset != 1)
        return fail(YF_E_INVALID, "norm_weight_offset must be 0 or 1");
    if (rope_dim != 0) {
        const int half = rope_dim / 2;
        if (rope_dim < 0 || rope_dim > D || rope_dim % (2 * E) || ((half / E) & (half / E - 1)))
            return fail(YF_E_UNSUPPORTED, "rope_dim %d: 0, or 2*%d*2^k up to head_dim %d", rope_dim, E, D);
        if (!rope_cos || !rope_sin || rope_rows < 1) return fail(YF_E_INVALID, "rope tables missing");
        if (!aligned(rope_cos, 16) || !aligned(rope_sin, 16))
            return fail(YF_E_INVALID, "rope tables must be 16-byte aligned");
    }
    if ((long long)max_rows * (n_q_heads + d.n_kv_heads) > 0x7fffffffLL)
        return fail(YF_E_UNSUPPORTED, "too many rows for one launch");
    PrepParams p;
    p.layer_base = pool->base + (size_t)layer * pool->layer_bytes;
    p.n_pages = d.n_pages;
    p.H = d.n_kv_heads;
    p.phb = (long long)pool->page_head_bytes;
    p.Hq = n_q_heads;
    p.qg = static_cast<const __half*>(qg);
    p.k = static_cast<const __half*>(k);
    p.v = static_cast<const __half*>(v);
    p.wq = q_norm_w;
    p.wk = k_norm_w;
    p.eps = eps;
    p.w_offset = (float)norm_weight_offset;
    p.cosb = rope_cos;
    p.sinb = rope_sin;
    p.rope_dim = rope_dim;
    p.rope_rows = rope_rows;
    p.cu_rows = cu_rows;
    p.start_pos = start_pos;
    p.bt = block_table;
    p.max_blocks = max_blocks;
    p.max_rows = max_rows;
    p.q_out = static_cast<__half*>(q_out);
    p.gate_out = static_cast<__half*>(gate_out);
    p.status = pool->d_status;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool row_scale = d.group_size == d.head_dim;
    const bool p16 = d.page_size == 16;
    if (D == 128) {
        if (row_scale) return p16 ? launch_prep<128, 1, 1>(p, batch, max_rows, s) : launch_prep<128, 1, 4>(p, batch, max_rows, s);
        return p16 ? launch_prep<128, 4, 1>(p, batch, max_rows, s) : launch_prep<128, 4, 4>(p, batch, max_rows, s);
    }
    if (row_scale) return p16 ? launch_prep<256, 1, 1>(p, batch, max_rows, s) : launch_prep<256, 1, 4>(p, batch, max_rows, s);
    return p16 ? launch_prep<256, 8, 1>(p, batch, max_rows, s) : launch_prep<256, 8, 4>(p, batch, max_rows, s);
}
