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
    return dispatch_write<true>(pool, p, batch, max_rows, static_cast<cudaStream_t>(stream));
}
