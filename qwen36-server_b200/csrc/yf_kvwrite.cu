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

// ---- multi-row writer: whole tiles staged in shared memory -------------------------------
//
// One CTA of two warps per (entry, 16-token tile its rows touch, kv head) quantizes the tile's K
// and V rows into a shared-memory copy of the tile and then writes it out with 16-byte coalesced
// stores; a tile the entry's rows only partly cover is first loaded, so its other tokens keep
// their bytes.  Lane work: one Q8_0 group of one row.  A group of <= 32 dims is loaded once into
// registers as packed f16 (the |x| maximum is exact in f16), then the pair of IEEE divisions and
// the group's values; a row-scale group (G = D) takes an amax pass and a quantize pass over its
// row.  Same arithmetic as q8_store_row: bit-exact with it.
constexpr int kTileThreads = 64;

// Stores the 8 quantized values of dims d0..d0+7 (d0 % 8 == 0) of token t into the tile.
__device__ __forceinline__ void put8(uint8_t* tile, int D, int NB, int t, int kv, int d0, const uint8_t (&qb)[8]) {
    const int V_OFF = 16 * D + 32 * NB;
    if (kv == 0) {
        const int b32 = d0 / 32, r = d0 % 32;
        uint2 w;
        w.x = qb[0] | (qb[1] << 8) | (qb[2] << 16) | ((uint32_t)qb[3] << 24);
        w.y = qb[4] | (qb[5] << 8) | (qb[6] << 16) | ((uint32_t)qb[7] << 24);
        *reinterpret_cast<uint2*>(tile + b32 * 512 + ((t % 8) * 4 + r / 8) * 16 + (t / 8) * 8) = w;
    } else {
        const int tig = (t % 8) / 2, j = (t & 1) * 2 + t / 8;
        const int m = d0 / 16, hi8 = (d0 % 16) / 8;
        uint8_t* vb = tile + V_OFF + (m / 2) * 512 + tig * 16 + (m % 2) * 8 + hi8 * 4 + j;
#pragma unroll
        for (int e = 0; e < 8; ++e) vb[e * 64] = qb[e];
    }
}

__device__ __forceinline__ void quant8(const uint4 w, float id, uint8_t (&qb)[8]) {
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const __half2 a = *reinterpret_cast<const __half2*>(&ww[k]);
        qb[2 * k] = excess128((int8_t)(int)roundf(__fmul_rn(__low2float(a), id)));
        qb[2 * k + 1] = excess128((int8_t)(int)roundf(__fmul_rn(__high2float(a), id)));
    }
}

__device__ __forceinline__ void put_scale(uint8_t* tile, int D, int NB, int t, int kv, int grp, float d) {
    const int KS_OFF = 16 * D, VS_OFF = 32 * D + 32 * NB;
    const int tig = (t % 8) / 2, j = (t & 1) * 2 + t / 8;
    const int off = kv == 0 ? KS_OFF + 2 * (((t % 8) * 2 + t / 8) * NB + grp) : VS_OFF + 2 * ((tig * NB + grp) * 4 + j);
    *reinterpret_cast<__half*>(tile + off) = __float2half_rn(d);
}

template <int D, int NB, int TPP>
__global__ void __launch_bounds__(kTileThreads) kv_write_tiles_kernel(const WriteParams p) {
    constexpr int TB = 32 * D + 64 * NB;
    constexpr int P = TPP * 16;
    constexpr int G = D / NB;
    constexpr int RPJ = 32 / NB;        // rows per warp job (a lane = one group of one row)
    constexpr int JOBS = 32 / RPJ;      // (kv, token) rows of the tile = 32
    constexpr int JPW = (JOBS + 1) / 2; // jobs per warp
    __shared__ __align__(16) uint8_t stage[TB];
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
    uint4* gtile = reinterpret_cast<uint4*>(p.layer_base + ((size_t)page * p.H + h) * p.phb +
                                            ((16 * T) % P) / 16 * (size_t)TB);
    if (lo > 16 * T || hi < 16 * T + 16) {  // partly covered: keep the tile's other tokens
        for (int k = threadIdx.x; k < TB / 16; k += kTileThreads) reinterpret_cast<uint4*>(stage)[k] = gtile[k];
        __syncthreads();
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = lane % NB;
    if constexpr (G <= 32) {
        // every job's loads first (JPW x G/8 independent 16-byte loads per lane), then the math
        uint4 w[JPW][G / 8];
        bool live[JPW];
        int tt[JPW], kvv[JPW];
#pragma unroll
        for (int q = 0; q < JPW; ++q) {
            const int R = (warp * JPW + q) * RPJ + lane / NB;  // (kv, token) row of the tile
            kvv[q] = R / 16;
            tt[q] = R % 16;
            const int pos = 16 * T + tt[q];
            live[q] = warp * JPW + q < JOBS && pos >= lo && pos < hi;
            if (live[q]) {
                const uint4* src = reinterpret_cast<const uint4*>((kvv[q] ? p.v : p.k) +
                                                                  ((size_t)(p.cu_rows[b] + pos - s) * p.H + h) * D + grp * G);
#pragma unroll
                for (int c = 0; c < G / 8; ++c) w[q][c] = __ldcs(src + c);
            }
        }
#pragma unroll
        for (int q = 0; q < JPW; ++q) {
            if (!live[q]) continue;
            __half2 m2 = __float2half2_rn(0.f);
#pragma unroll
            for (int c = 0; c < G / 8; ++c) {
                const uint32_t ww[4] = {w[q][c].x, w[q][c].y, w[q][c].z, w[q][c].w};
#pragma unroll
                for (int k = 0; k < 4; ++k) m2 = __hmax2(m2, __habs2(*reinterpret_cast<const __half2*>(&ww[k])));
            }
            const float amax = fmaxf(__low2float(m2), __high2float(m2));
            const float d = __fdiv_rn(amax, 127.0f);
            const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
#pragma unroll
            for (int c = 0; c < G / 8; ++c) {
                uint8_t qb[8];
                quant8(w[q][c], id, qb);
                put8(stage, D, NB, tt[q], kvv[q], grp * G + 8 * c, qb);
            }
            put_scale(stage, D, NB, tt[q], kvv[q], grp, d);
        }
    } else {
        // row scale: lane = one (kv, token) row; an amax pass and a quantize pass over the row
        const int R = warp * 32 + lane;
        const int kv = R / 16, t = R % 16, pos = 16 * T + t;
        if (R < 32 && pos >= lo && pos < hi) {
            const uint4* src = reinterpret_cast<const uint4*>((kv ? p.v : p.k) +
                                                              ((size_t)(p.cu_rows[b] + pos - s) * p.H + h) * D);
            __half2 m2 = __float2half2_rn(0.f);
#pragma unroll 4
            for (int c = 0; c < D / 8; ++c) {
                const uint4 x = src[c];
                const uint32_t ww[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) m2 = __hmax2(m2, __habs2(*reinterpret_cast<const __half2*>(&ww[k])));
            }
            const float amax = fmaxf(__low2float(m2), __high2float(m2));
            const float d = __fdiv_rn(amax, 127.0f);
            const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
#pragma unroll 4
            for (int c = 0; c < D / 8; ++c) {
                uint8_t qb[8];
                quant8(src[c], id, qb);
                put8(stage, D, NB, t, kv, 8 * c, qb);
            }
            put_scale(stage, D, NB, t, kv, 0, d);
        }
    }
    __syncthreads();
    for (int k = threadIdx.x; k < TB / 16; k += kTileThreads) gtile[k] = reinterpret_cast<const uint4*>(stage)[k];
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
