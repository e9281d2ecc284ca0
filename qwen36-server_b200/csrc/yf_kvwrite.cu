// Q8_0 quantize-and-scatter of new K/V rows into the paged pool.
//
// Replaces kv_append_paged_f16 (one row per slot, fork quantized.cu:6996) and
// launch_append_multi (T contiguous rows per slot, fork quantized.cu:7040),
// cited at docs/plans/2026-08-27-tiered-kv-cache.md:61-64 and
// docs/plans/2026-08-27-mtp-cuda-graphs.md:132-134.
//
// One warp per (row, kv head); the row's load, Q8_0 rounding and stores are
// yf_q8row.cuh's (one 8- or 16-byte f16 load per lane and tensor; K bytes land
// as one E-byte store per lane, V bytes and the scales as single stores into
// their permuted slots).
#include "yf_device.cuh"
#include "yf_internal.h"
#include "yf_q8row.cuh"

namespace yf {

constexpr int kWriteWarps = 4;

struct WriteParams {
    uint8_t* layer_base;
    int n_pages;
    int H;
    long long phb;
    const __half* k;
    const __half* v;
    const int32_t* pos;        // single: position of row b
    const int32_t* cu_rows;    // multi: rows of entry b
    const int32_t* start_pos;  // multi: position of the first row of entry b
    const uint32_t* bt;
    int max_blocks;
    int max_rows;              // multi: bound on rows per entry (1 for single)
    uint32_t* status;
};

template <int D, int NB, int TPP, bool MULTI>
__global__ void __launch_bounds__(kWriteWarps * 32) kv_write_kernel(const WriteParams p) {
    pdl_trigger();  // the attention kernel that follows may be scheduled now (it waits for this one)
    constexpr int E = D / 32;   // elements per lane
    constexpr int TB = 32 * D + 64 * NB;
    constexpr int P = TPP * 16;

    const int lane = threadIdx.x & 31;
    const int wi = blockIdx.x * kWriteWarps + (threadIdx.x >> 5);
    const int b = blockIdx.y;
    const int i = wi / p.H, h = wi % p.H;
    int row, pos;
    if (MULTI) {
        const int r0 = p.cu_rows[b], n = p.cu_rows[b + 1] - r0;
        if (i == 0 && h == 0 && lane == 0 && (n > p.max_rows || n < 0)) atomicOr(p.status, YF_DEV_BAD_ROWS);
        if (i >= n || i >= p.max_rows) return;
        row = r0 + i;
        pos = p.start_pos[b] + i;
    } else {
        if (i >= 1) return;
        row = b;
        pos = p.pos[b];
    }
    if (pos < 0 || pos >= p.max_blocks * P) {
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

#pragma unroll
    for (int kv = 0; kv < 2; ++kv) {
        float x[E];
        load_f16_row<E>((kv ? p.v : p.k) + ((size_t)row * p.H + h) * D + lane * E, x);
        q8_store_row<D, NB>(tile, t, kv, lane, x);
    }
}

// ---- multi-row writer: one CTA per (entry, 16-token tile, kv head) --------------------------
//
// Phase 1 loads the tile's K and V rows (16 tokens each) with coalesced 16-byte loads into a
// padded f16 copy in shared memory and takes each Q8_0 group's |x| maximum (exact in f16) over
// the group's lanes; one lane per group then forms d = amax/127 and 1/d (IEEE divisions) and
// puts d, as f16, into a copy of the tile's scale areas.  Phase 2 builds every 16-byte chunk of
// the pool tile from the staged rows -- a K chunk is 8 dims of tokens t and t+8, a V chunk is
// 4 dims x the 4 tokens that share a word -- rounds the values (roundf(x * (1/d)), the Q8_0
// rule of q8_store_row, bit-exact with it) and stores the chunk straight to the pool: each
// warp's stores cover 512 contiguous bytes.  A tile the entry's rows only partly cover keeps
// the bytes of its other tokens (their chunks are merged with the pool's current bytes).
constexpr int kTileThreads = 64;

template <int D>
constexpr int stage_pitch() { return 2 * D + 16; }  // bytes per staged row (16 B pad: spreads banks)

template <int D, int NB, int TPP>
__global__ void __launch_bounds__(kTileThreads) kv_write_tiles_kernel(const WriteParams p) {
    pdl_trigger();  // the attention kernel that follows may be scheduled now (it waits for this one)
    constexpr int TB = 32 * D + 64 * NB;
    constexpr int P = TPP * 16;
    constexpr int G = D / NB;
    constexpr int RP = stage_pitch<D>();
    constexpr int KS_OFF = 16 * D, V_OFF = 16 * D + 32 * NB, VS_OFF = 32 * D + 32 * NB;
    constexpr int CPR = D / 8;   // 16-byte chunks per input row
    constexpr int LPG = G / 8;   // lanes (chunks) per group in phase 1
    static_assert(LPG <= 32 && (32 % LPG) == 0, "a group's chunks lie in one warp");
    __shared__ __align__(16) uint8_t rows[2][16][RP];     // f16 K and V rows of the tile's tokens
    __shared__ __align__(16) float inv[2][16][NB];         // 1/d per (kv, token, group)
    __shared__ __align__(16) uint16_t scl[2][16 * NB];     // the tile's K and V scale areas (f16 bits)
    const int b = blockIdx.z, h = blockIdx.y;
    const int n_raw = p.cu_rows[b + 1] - p.cu_rows[b];
    if (blockIdx.x == 0 && h == 0 && threadIdx.x == 0 && (n_raw > p.max_rows || n_raw < 0))
        atomicOr(p.status, YF_DEV_BAD_ROWS);
    const int n = min(max(n_raw, 0), p.max_rows);
    if (n == 0) return;
    const int s = p.start_pos[b];
    const int cap = p.max_blocks * P;
    const int first = s >= 0 ? s / 16 : -((15 - s) / 16);  // floor(s / 16)
    const int T = first + (int)blockIdx.x;
    const int lo = max(s, 16 * T), hi = min(s + n, 16 * T + 16);
    if (lo >= hi) return;
    if (T < 0 || 16 * T >= cap) {  // positions outside the table: the rows are skipped
        if (threadIdx.x == 0 && h == 0) atomicOr(p.status, YF_DEV_BAD_POS);
        return;
    }
    const uint32_t page = p.bt[(size_t)b * p.max_blocks + (16 * T) / P];
    if (page >= (uint32_t)p.n_pages) {
        if (threadIdx.x == 0 && h == 0) atomicOr(p.status, YF_DEV_BAD_PAGE);
        return;
    }
    uint8_t* gtile = p.layer_base + ((size_t)page * p.H + h) * p.phb + ((16 * T) % P) / 16 * (size_t)TB;
    const int t_lo = lo - 16 * T, t_hi = hi - 16 * T;  // live tokens [t_lo, t_hi)
    const bool partial = t_lo > 0 || t_hi < 16;
    auto live = [&](int t) { return t >= t_lo && t < t_hi; };
    if (partial) {  // the scale areas start as the pool's; live tokens overwrite theirs
        for (int k = threadIdx.x; k < 2 * 16 * NB; k += kTileThreads)
            scl[k / (16 * NB)][k % (16 * NB)] =
                *reinterpret_cast<const uint16_t*>(gtile + (k < 16 * NB ? KS_OFF : VS_OFF) + 2 * (k % (16 * NB)));
        __syncthreads();
    }

    // ---- phase 1: rows into shared memory, group maxima, scales.  All of the thread's loads are
    // issued before the first is used.
    constexpr int ITER = 2 * 16 * CPR / kTileThreads;
    static_assert((2 * 16 * CPR) % kTileThreads == 0, "whole iterations");
    uint4 wv[ITER];
#pragma unroll
    for (int i = 0; i < ITER; ++i) {
        const int c = threadIdx.x + i * kTileThreads;
        const int kv = c / (16 * CPR), t = (c / CPR) % 16, q = c % CPR;
        wv[i] = make_uint4(0, 0, 0, 0);
        if (live(t)) {
            const __half* src = (kv ? p.v : p.k) + ((size_t)(p.cu_rows[b] + 16 * T + t - s) * p.H + h) * D;
            wv[i] = __ldcs(reinterpret_cast<const uint4*>(src) + q);
        }
    }
#pragma unroll
    for (int i = 0; i < ITER; ++i) {
        const int c = threadIdx.x + i * kTileThreads;
        const int kv = c / (16 * CPR), t = (c / CPR) % 16, q = c % CPR;
        const uint4 w = wv[i];
        *reinterpret_cast<uint4*>(&rows[kv][t][16 * q]) = w;
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
        __half2 m2 = __float2half2_rn(0.f);
#pragma unroll
        for (int k = 0; k < 4; ++k) m2 = __hmax2(m2, __habs2(*reinterpret_cast<const __half2*>(&ww[k])));
        float amax = fmaxf(__low2float(m2), __high2float(m2));
#pragma unroll
        for (int off = 1; off < LPG; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
        if (live(t) && q % LPG == 0) {
            const int grp = q / LPG;
            const float d = __fdiv_rn(amax, 127.0f);
            inv[kv][t][grp] = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
            const int tig = (t % 8) / 2, j = (t & 1) * 2 + t / 8;
            const int si = kv == 0 ? ((t % 8) * 2 + t / 8) * NB + grp : (tig * NB + grp) * 4 + j;
            scl[kv][si] = __half_as_ushort(__float2half_rn(d));
        }
    }
    __syncthreads();

    // roundf(y) for |y| < 2^23 as trunc(y + copysign(0.5 - 2^-25, y)) with a round-to-nearest
    // add: below .5 the sum stays under the next integer, from .5 up it reaches it (|y| <= 127
    // here); the same value as roundf, in three instructions
    auto q8 = [](float x, float id) -> uint32_t {
        const float y = __fmul_rn(x, id);
        const int q = __float2int_rz(__fadd_rn(y, copysignf(0.49999997f, y)));
        return (uint32_t)(q + 128) & 0xFFu;
    };
    // ---- phase 2a: K chunks (chunk kc = b32*32 + (t%8)*4 + r/8: dims 32*b32 + 8*(r/8) .. +7 of
    // tokens t%8 (bytes 0-7) and t%8 + 8 (bytes 8-15))
    for (int kc = threadIdx.x; kc < D * 16 / 16; kc += kTileThreads) {
        const int b32 = kc / 32, t0 = (kc % 32) / 4, q4 = kc % 4;
        const int d0 = 32 * b32 + 8 * q4, grp = d0 / G;
        uint32_t out[4];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int t = t0 + 8 * half;
            const uint4 w = *reinterpret_cast<const uint4*>(&rows[0][t][2 * d0]);
            const float id = inv[0][t][grp];
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
            uint32_t lo32 = 0, hi32 = 0;
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const __half2 a = *reinterpret_cast<const __half2*>(&ww[k]);
                const __half2 c2 = *reinterpret_cast<const __half2*>(&ww[k + 2]);
                lo32 |= (q8(__low2float(a), id) | (q8(__high2float(a), id) << 8)) << (16 * k);
                hi32 |= (q8(__low2float(c2), id) | (q8(__high2float(c2), id) << 8)) << (16 * k);
            }
            out[2 * half] = lo32;
            out[2 * half + 1] = hi32;
        }
        uint4* dst = reinterpret_cast<uint4*>(gtile + b32 * 512 + (t0 * 4 + q4) * 16);
        uint4 o = make_uint4(out[0], out[1], out[2], out[3]);
        if (partial) {
            const uint4 old = *dst;
            if (!live(t0)) { o.x = old.x; o.y = old.y; }
            if (!live(t0 + 8)) { o.z = old.z; o.w = old.w; }
        }
        *dst = o;
    }
    // ---- phase 2b: V chunks (chunk vc = M*32 + iim*4 + tig: word (m%2)*2 + ii/8 holds dim
    // 16*(2M + m%2) + iim + 8*(ii/8) of tokens 2tig, 2tig+8, 2tig+1, 2tig+9 in bytes 0..3)
    for (int vc = threadIdx.x; vc < D * 16 / 16; vc += kTileThreads) {
        const int M = vc / 32, iim = (vc % 32) / 4, tig = vc % 4;
        const int tok[4] = {2 * tig, 2 * tig + 8, 2 * tig + 1, 2 * tig + 9};
        const int grp = 32 * M / G;  // the chunk's dims lie in one 32-dim block, so in one group
        float id[4];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) id[jj] = inv[1][tok[jj]][grp];
        uint32_t out[4];
#pragma unroll
        for (int wd = 0; wd < 4; ++wd) {
            const int dim = 16 * (2 * M + wd / 2) + iim + 8 * (wd % 2);
            uint32_t word = 0;
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                const float x = __half2float(*reinterpret_cast<const __half*>(&rows[1][tok[jj]][2 * dim]));
                word |= q8(x, id[jj]) << (8 * jj);
            }
            out[wd] = word;
        }
        uint4* dst = reinterpret_cast<uint4*>(gtile + V_OFF + M * 512 + (iim * 4 + tig) * 16);
        uint4 o = make_uint4(out[0], out[1], out[2], out[3]);
        if (partial) {
            uint32_t keep = 0;  // bytes of tokens outside the chunk's live range
#pragma unroll
            for (int jj = 0; jj < 4; ++jj)
                if (!live(tok[jj])) keep |= 0xFFu << (8 * jj);
            const uint4 old = *dst;
            o.x = (o.x & ~keep) | (old.x & keep);
            o.y = (o.y & ~keep) | (old.y & keep);
            o.z = (o.z & ~keep) | (old.z & keep);
            o.w = (o.w & ~keep) | (old.w & keep);
        }
        *dst = o;
    }
    // ---- phase 2c: the two scale areas (16 * NB f16 each, 16-byte aligned)
    for (int k = threadIdx.x; k < 2 * 16 * NB * 2 / 16; k += kTileThreads) {
        const int kv = k / (16 * NB * 2 / 16), i = k % (16 * NB * 2 / 16);
        *reinterpret_cast<uint4*>(gtile + (kv ? VS_OFF : KS_OFF) + 16 * i) = reinterpret_cast<const uint4*>(scl[kv])[i];
    }
}

template <int D, int NB, int TPP>
static int launch_write_tiles(const WriteParams& p, int batch, int max_rows, cudaStream_t s) {
    const dim3 grid((unsigned)((max_rows + 15) / 16 + 1), p.H, batch);
    kv_write_tiles_kernel<D, NB, TPP><<<grid, kTileThreads, 0, s>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? YF_OK : cuda_fail(e, "kv tile write launch");
}

static int dispatch_write_tiles(const yf_pool* pool, const WriteParams& p, int batch, int rows, cudaStream_t s) {
    const yf_pool_desc& d = pool->desc;
    const bool row_scale = d.group_size == d.head_dim;
    const bool p16 = d.page_size == 16;
    if (d.head_dim == 128) {
        if (row_scale)
            return p16 ? launch_write_tiles<128, 1, 1>(p, batch, rows, s) : launch_write_tiles<128, 1, 4>(p, batch, rows, s);
        return p16 ? launch_write_tiles<128, 4, 1>(p, batch, rows, s) : launch_write_tiles<128, 4, 4>(p, batch, rows, s);
    }
    if (row_scale)
        return p16 ? launch_write_tiles<256, 1, 1>(p, batch, rows, s) : launch_write_tiles<256, 1, 4>(p, batch, rows, s);
    return p16 ? launch_write_tiles<256, 8, 1>(p, batch, rows, s) : launch_write_tiles<256, 8, 4>(p, batch, rows, s);
}

template <int D, int NB, int TPP, bool MULTI>
static int launch_write(const WriteParams& p, int batch, int rows_per_entry, cudaStream_t s) {
    const long long warps = (long long)rows_per_entry * p.H;
    const dim3 grid((unsigned)((warps + kWriteWarps - 1) / kWriteWarps), batch);
    kv_write_kernel<D, NB, TPP, MULTI><<<grid, kWriteWarps * 32, 0, s>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? YF_OK : cuda_fail(e, "kv write launch");
}

template <bool MULTI>
static int dispatch_write(const yf_pool* pool, const WriteParams& p, int batch, int rows, cudaStream_t s) {
    const yf_pool_desc& d = pool->desc;
    const bool row_scale = d.group_size == d.head_dim;
    const bool p16 = d.page_size == 16;
    if (d.head_dim == 128) {
        if (row_scale)
            return p16 ? launch_write<128, 1, 1, MULTI>(p, batch, rows, s) : launch_write<128, 1, 4, MULTI>(p, batch, rows, s);
        return p16 ? launch_write<128, 4, 1, MULTI>(p, batch, rows, s) : launch_write<128, 4, 4, MULTI>(p, batch, rows, s);
    }
    if (row_scale)
        return p16 ? launch_write<256, 1, 1, MULTI>(p, batch, rows, s) : launch_write<256, 1, 4, MULTI>(p, batch, rows, s);
    return p16 ? launch_write<256, 8, 1, MULTI>(p, batch, rows, s) : launch_write<256, 8, 4, MULTI>(p, batch, rows, s);
}

static int check_write(const yf_pool* pool, int32_t layer, const void* k, const void* v, const void* bt,
                       int32_t max_blocks, int32_t batch) {
    if (!pool) return fail(YF_E_INVALID, "pool is null");
    if (!pool->base) return fail(YF_E_INVALID, "host-only pool has no device memory");
    if (batch < 0) return fail(YF_E_INVALID, "batch %d < 0", batch);
    if (batch == 0) return YF_OK;
    if (batch > 65535) return fail(YF_E_UNSUPPORTED, "batch %d > 65535", batch);
    if (!k || !v || !bt) return fail(YF_E_INVALID, "null device pointer");
    if (!aligned(k, 16) || !aligned(v, 16)) return fail(YF_E_INVALID, "k and v must be 16-byte aligned");
    if (layer < 0 || layer >= pool->desc.n_layers) return fail(YF_E_RANGE, "layer %d out of range", layer);
    if (max_blocks < 1) return fail(YF_E_INVALID, "max_blocks %d < 1", max_blocks);
    return YF_OK;
}

static WriteParams make_params(const yf_pool* pool, int32_t layer, const void* k, const void* v,
                               const uint32_t* bt, int32_t max_blocks) {
    WriteParams p;
    p.layer_base = pool->base + (size_t)layer * pool->layer_bytes;
    p.n_pages = pool->desc.n_pages;
    p.H = pool->desc.n_kv_heads;
    p.phb = (long long)pool->page_head_bytes;
    p.k = static_cast<const __half*>(k);
    p.v = static_cast<const __half*>(v);
    p.pos = nullptr;
    p.cu_rows = nullptr;
    p.start_pos = nullptr;
    p.bt = bt;
    p.max_blocks = max_blocks;
    p.max_rows = 1;
    p.status = pool->d_status;
    return p;
}

}  // namespace yf

using namespace yf;

extern "C" int yf_kv_append_paged(yf_pool* pool, int32_t layer, const void* k, const void* v, const int32_t* pos,
                                  const uint32_t* bt, int32_t max_blocks, int32_t batch, void* stream) {
    const int rc = check_write(pool, layer, k, v, bt, max_blocks, batch);
    if (rc || batch == 0) return rc;
    if (!pos) return fail(YF_E_INVALID, "d_pos is null");
    WriteParams p = make_params(pool, layer, k, v, bt, max_blocks);
    p.pos = pos;
    return dispatch_write<false>(pool, p, batch, 1, static_cast<cudaStream_t>(stream));
}

extern "C" int yf_kv_append_paged_multi(yf_pool* pool, int32_t layer, const void* k, const void* v,
                                        const int32_t* cu_rows, const int32_t* start_pos, const uint32_t* bt,
                                        int32_t max_blocks, int32_t batch, int32_t max_rows, void* stream) {
    const int rc = check_write(pool, layer, k, v, bt, max_blocks, batch);
    if (rc || batch == 0) return rc;
    if (!cu_rows || !start_pos) return fail(YF_E_INVALID, "d_cu_rows / d_start_pos is null");
    if (max_rows < 0) return fail(YF_E_INVALID, "max_rows %d < 0", max_rows);
    if (max_rows == 0) return YF_OK;
    if ((long long)max_rows * pool->desc.n_kv_heads > (1LL << 30)) return fail(YF_E_UNSUPPORTED, "max_rows too large");
    WriteParams p = make_params(pool, layer, k, v, bt, max_blocks);
    p.cu_rows = cu_rows;
    p.start_pos = start_pos;
    p.max_rows = max_rows;
    // blocks of rows fill whole tiles: staged tile writer (rows of different entries must not share
    // a tile within one call); a few rows per entry: a warp per row
    if (max_rows >= 16 && pool->desc.n_kv_heads <= 65535)
        return dispatch_write_tiles(pool, p, batch, max_rows, static_cast<cudaStream_t>(stream));
    return dispatch_write<true>(pool, p, batch, max_rows, static_cast<cudaStream_t>(stream));
}
