// Pool lifetime, page allocator, snapshot export/restore, argument checks and
// the attention entry points of the C ABI (include/yfattn.h).
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>

#include "yf_internal.h"

namespace {
thread_local char g_err[512] = "";
}

namespace yf {

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(YF_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

namespace {
std::mutex g_launch_mu;  // guards every LaunchCache
}

int raise_smem_attr(const void* kern, int smem, int dev, LaunchCache& c) {
    std::lock_guard<std::mutex> lock(g_launch_mu);
    if (dev >= 0 && dev < 64 && c.smem_set[dev] >= smem) return YF_OK;
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic shared memory)");
    if (dev >= 0 && dev < 64) c.smem_set[dev] = smem;
    return YF_OK;
}

int occupancy(const void* kern, int threads, int smem, int dev, LaunchCache& c, int* out) {
    std::lock_guard<std::mutex> lock(g_launch_mu);
    if (dev >= 0 && dev < 64 && c.occ_smem[dev] == smem && c.occ_val[dev] > 0) {
        *out = c.occ_val[dev];
        return YF_OK;
    }
    int occ = 0;
    const cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, threads, smem);
    if (e != cudaSuccess) return cuda_fail(e, "occupancy query");
    if (dev >= 0 && dev < 64) {
        c.occ_smem[dev] = smem;
        c.occ_val[dev] = occ;
    }
    *out = occ;
    return YF_OK;
}

static int check_desc(const yf_pool_desc* d) {
    if (!d) return fail(YF_E_INVALID, "desc is null");
    if (d->n_layers < 1 || d->n_pages < 1 || d->n_kv_heads < 1)
        return fail(YF_E_INVALID, "n_layers, n_pages and n_kv_heads must be >= 1");
    if (d->head_dim != 128 && d->head_dim != 256)
        return fail(YF_E_UNSUPPORTED, "head_dim %d: built for 128 and 256", d->head_dim);
    if (d->page_size != 16 && d->page_size != 64)
        return fail(YF_E_UNSUPPORTED, "page_size %d: built for 16 and 64", d->page_size);
    if (d->group_size != 32 && d->group_size != d->head_dim)
        return fail(YF_E_UNSUPPORTED, "group_size %d: built for 32 and head_dim", d->group_size);
    return YF_OK;
}

static size_t tile_bytes_of(const yf_pool_desc* d) {
    return tile_geom(d->head_dim, d->head_dim / d->group_size).tile;
}

// Splits the tile range of every (entry, kv head, row group) into chunks so
// that the grid covers the SMs several times over; the last chunk of each
// unit is partial, so more, smaller chunks keep the tail short.
SplitPlan plan_split(const yf_pool* pool, int n_q_heads, int batch, int max_seqlen_q, int max_seqlen_k, bool tree) {
    SplitPlan p;
    const int H = pool->desc.n_kv_heads;
    const int G = n_q_heads / H;
    const int rows = G * (max_seqlen_q > 0 ? max_seqlen_q : 1);
    p.rows_per_cta = (rows <= 8 || pool->desc.head_dim > 128) ? 8 : 16;
    p.n_row_groups = (rows + p.rows_per_cta - 1) / p.rows_per_cta;
    const int tiles = (max_seqlen_k + kTileTokens - 1) / kTileTokens;
    const long long units = (long long)batch * H * p.n_row_groups;
    const long long target = (long long)pool->sm_count * 16;
    const yf_attn_options& o = pool->opts;
    int chunk;
    if (o.chunk_tiles > 0) {
        chunk = o.chunk_tiles;
    } else {
        long long c = (units * tiles + target - 1) / target;
        if (c < 8) c = 8;
        c = (c + 3) / 4 * 4;
        if (c > (1 << 20)) c = 1 << 20;
        chunk = (int)c;
    }
    if (tiles > 65535LL * chunk) chunk = (tiles + 65534) / 65535;  // grid z <= 65535
    p.chunk_tiles = chunk;
    p.max_chunks = tiles > 0 ? (tiles + chunk - 1) / chunk : 1;
    p.stages = o.copy_stages == 3 ? 3 : (pool->desc.head_dim == 128 ? 4 : 2);
    const bool in_kernel_merge = o.merge != YF_MERGE_SEPARATE;
    // the in-kernel merge of the chunked schedule keeps (chunks + 1) x rows floats of weights
    // in the CTA's stage area (4 warps x stages x tile bytes); the persistent schedule merges
    // its CTAs (at most kMaxGroupCounters / 2) in one cooperative pass
    {
        const int D = pool->desc.head_dim, NB = D / pool->desc.group_size;
        const long long area_floats = 4LL * p.stages * (32 * D + 64 * NB) / 4;
        p.fused_combine = in_kernel_merge && (long long)(p.max_chunks + 1) * p.rows_per_cta <= area_floats;
    }
    // Persistent schedule: one row group per entry (decode, small verify blocks), a batch whose
    // tile prefix fits in shared memory, and the merge counters available.
    p.persistent = !tree && o.schedule != YF_SCHED_CHUNKED && p.n_row_groups == 1 && batch <= kPersistentMaxBatch &&
                   units <= kMaxCombineUnits && in_kernel_merge;
    if (p.persistent) p.fused_combine = true;
    // A few long units of one entry (long-context decode, one rank's shard, a small decode): whole
    // clusters of kClusterCtas CTAs per unit, at least 16 tiles per CTA and about two CTAs per SM
    // in all (a third CTA per SM measured slower: more partials to merge, uneven CTAs per SM).
    // One entry only: its units (kv heads) have equal lengths, while clusters sized for the
    // longest of several entries leave the shorter ones' CTAs idle (a 4-slot share of
    // decode_batch: 52.0 us clustered, 42.3 us persistent).
    p.cluster = p.persistent && o.schedule == YF_SCHED_AUTO && p.rows_per_cta == 8 && batch == 1 &&
                units <= kClusterMaxUnits && tiles > 0;
    if (p.cluster) {
        p.persistent = false;
        // one wave of clusters: cluster placement is per GPC, so the device's cluster capacity,
        // not SMs x CTAs per SM, bounds the grid (a partial second wave doubles the time)
        const long long target = std::min((long long)pool->sm_count * 2, std::max<long long>(kClusterCtas, units * tiles / 16));
        const long long cap = cluster_capacity(pool, p.stages);
        const long long cpu = std::max<long long>(
            1, std::min<long long>(std::min(target / (units * kClusterCtas), cap / units), kClusterMaxParts));
        p.max_chunks = (int)cpu;                         // clusters per unit
        p.chunk_tiles = (int)((tiles + cpu - 1) / cpu);  // tiles per cluster
        const size_t row_bytes_c = p.rows_per_cta * (pool->desc.head_dim + 1) * sizeof(float);
        p.ws_bytes = cpu > 1 ? (size_t)units * cpu * row_bytes_c : 0;
        p.persistent_ctas = 0;
        return p;
    }
    const size_t row_bytes = p.rows_per_cta * (pool->desc.head_dim + 1) * sizeof(float);
    if (p.persistent) {
        // at least 16 tiles (4 per warp) per CTA, at most kMaxCtasPerSm CTAs per SM
        const long long by_work = (units * tiles + 15) / 16;
        long long ctas = (long long)pool->sm_count * kMaxCtasPerSm;
        if (by_work < ctas) ctas = by_work > 0 ? by_work : 1;
        // few long units: more than ~128 parts per unit only lengthens the merge once ~1.75 CTAs
        // per SM keep HBM busy (the 131072-key, 2-head decode: 42 us at 444 CTAs, 39 at 256)
        const long long by_units = std::max((long long)pool->sm_count * 7 / 4, units * 128);
        if (by_units < ctas) ctas = by_units;
        if (2 * ctas > kMaxGroupCounters) ctas = kMaxGroupCounters / 2;
        p.persistent_ctas = (int)ctas;
        p.ws_bytes = (size_t)p.persistent_ctas * 2 * row_bytes;  // two partial slots per CTA
    } else {
        p.persistent_ctas = 0;
        p.ws_bytes = p.max_chunks <= 1 ? 0 : (size_t)units * p.max_chunks * row_bytes;
    }
    return p;
}

}  // namespace yf

using namespace yf;

// One stream-ordered word store (the counter fault-injection hook).
__global__ void store_word_kernel(uint32_t* dst, uint32_t value) { *dst = value; }

extern "C" {

const char* yf_last_error(void) { return g_err; }
int yf_abi_version(void) { return YFATTN_ABI_VERSION; }

size_t yf_pool_page_head_bytes(const yf_pool_desc* d) {
    if (check_desc(d) != YF_OK) return 0;
    return (size_t)(d->page_size / kTileTokens) * tile_bytes_of(d);
}

size_t yf_pool_bytes(const yf_pool_desc* d) {
    const size_t phb = yf_pool_page_head_bytes(d);
    if (!phb) return 0;
    return (size_t)d->n_layers * d->n_pages * d->n_kv_heads * phb;
}

int64_t yf_pool_tile_offset(const yf_pool_desc* d, int is_v, int t, int dim) {
    if (check_desc(d) != YF_OK || t < 0 || t >= 16 || dim < 0 || dim >= d->head_dim) return -1;
    const TileGeom g = tile_geom(d->head_dim, d->head_dim / d->group_size);
    if (!is_v) {
        const int b = dim / 32, r = dim % 32;
        return (int64_t)b * 512 + ((t % 8) * 4 + r / 8) * 16 + (t / 8) * 8 + r % 8;
    }
    const int m = dim / 16, i = dim % 16;
    const int tig = (t % 8) / 2, j = (t & 1) * 2 + t / 8;
    return (int64_t)g.v_off + (m / 2) * 512 + ((i % 8) * 4 + tig) * 16 + (m % 2) * 8 + (i / 8) * 4 + j;
}

int64_t yf_pool_scale_offset(const yf_pool_desc* d, int is_v, int t, int group) {
    if (check_desc(d) != YF_OK || t < 0 || t >= 16) return -1;
    const int NB = d->head_dim / d->group_size;
    if (group < 0 || group >= NB) return -1;
    const TileGeom g = tile_geom(d->head_dim, NB);
    if (!is_v) return (int64_t)g.ks_off + 2 * (((t % 8) * 2 + t / 8) * NB + group);
    const int tig = (t % 8) / 2, j = (t & 1) * 2 + t / 8;
    return (int64_t)g.vs_off + 2 * ((tig * NB + group) * 4 + j);
}

int yf_pool_create(const yf_pool_desc* desc, yf_pool** out_pool) {
    if (!out_pool) return fail(YF_E_INVALID, "out_pool is null");
    *out_pool = nullptr;
    const int rc = check_desc(desc);
    if (rc) return rc;
    yf_pool* p = new (std::nothrow) yf_pool();
    if (!p) return fail(YF_E_NOMEM, "host allocation failed");
    p->desc = *desc;
    p->tile_bytes = tile_bytes_of(desc);
    p->page_head_bytes = yf_pool_page_head_bytes(desc);
    p->page_bytes = p->page_head_bytes * desc->n_kv_heads;
    p->layer_bytes = p->page_bytes * desc->n_pages;
    p->bytes = p->layer_bytes * desc->n_layers;
    p->refcount.assign(desc->n_pages, 0);
    p->free_stack.resize(desc->n_pages);
    for (int i = 0; i < desc->n_pages; ++i) p->free_stack[i] = desc->n_pages - 1 - i;  // pops 0,1,2,...
    init_record_ops(p);
    if (desc->device < 0) {  // host-only pool: the page allocator without device memory
        p->desc.device_mem = nullptr;
        *out_pool = p;
        return YF_OK;
    }
    cudaError_t e = cudaSetDevice(desc->device);
    if (e != cudaSuccess) {
        delete p;
        return cuda_fail(e, "cudaSetDevice");
    }
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, desc->device) == cudaSuccess && sms > 0)
        p->sm_count = sms;
    if (desc->device_mem) {
        if (!aligned(desc->device_mem, 256)) {
            delete p;
            return fail(YF_E_INVALID, "device_mem must be 256-byte aligned");
        }
        p->base = static_cast<uint8_t*>(desc->device_mem);
        p->owns_mem = false;
    } else {
        e = cudaMalloc(&p->base, p->bytes);
        if (e != cudaSuccess) {
            cudaGetLastError();
            delete p;
            return fail(YF_E_NOMEM, "cudaMalloc of %zu pool bytes: %s", p->bytes, cudaGetErrorString(e));
        }
        p->owns_mem = true;
    }
    e = cudaMalloc(&p->d_status, sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemset(p->d_status, 0, sizeof(uint32_t));
    const size_t n_counters = (size_t)kMaxCombineUnits + kMaxGroupCounters;
    if (e == cudaSuccess) e = cudaMalloc(&p->d_counters, sizeof(uint32_t) * n_counters);
    if (e == cudaSuccess) e = cudaMemset(p->d_counters, 0, sizeof(uint32_t) * n_counters);
    if (e == cudaSuccess) e = cudaMemset(p->base, 0, p->bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        if (p->owns_mem) cudaFree(p->base);
        if (p->d_status) cudaFree(p->d_status);
        if (p->d_counters) cudaFree(p->d_counters);
        delete p;
        return cuda_fail(e, "pool initialisation");
    }
    *out_pool = p;
    return YF_OK;
}

int yf_pool_destroy(yf_pool* pool) {
    if (!pool) return YF_OK;
    if (pool->base || pool->d_status) {
        cudaSetDevice(pool->desc.device);
        if (pool->owns_mem && pool->base) cudaFree(pool->base);
        if (pool->d_status) cudaFree(pool->d_status);
        if (pool->d_counters) cudaFree(pool->d_counters);
    }
    delete pool;
    return YF_OK;
}

int yf_pool_get_desc(const yf_pool* pool, yf_pool_desc* out) {
    if (!pool || !out) return fail(YF_E_INVALID, "null argument");
    *out = pool->desc;
    out->device_mem = pool->base;
    return YF_OK;
}

int yf_pool_layer_ptr(const yf_pool* pool, int32_t layer, void** out_ptr) {
    if (!pool || !out_ptr) return fail(YF_E_INVALID, "null argument");
    if (!pool->base) return fail(YF_E_INVALID, "host-only pool has no device memory");
    if (layer < 0 || layer >= pool->desc.n_layers) return fail(YF_E_RANGE, "layer %d out of range", layer);
    *out_ptr = pool->base + (size_t)layer * pool->layer_bytes;
    return YF_OK;
}

int yf_pool_alloc_pages(yf_pool* pool, int32_t n, int32_t* out) {
    if (!pool || n < 0 || (n > 0 && !out)) return fail(YF_E_INVALID, "bad alloc arguments");
    if ((size_t)n > pool->free_stack.size())
        return fail(YF_E_NOMEM, "requested %d pages, %zu free", n, pool->free_stack.size());
    for (int i = 0; i < n; ++i) {
        const int32_t pg = pool->free_stack.back();
        pool->free_stack.pop_back();
        pool->refcount[pg] = 1;
        out[i] = pg;
    }
    return YF_OK;
}

int yf_pool_retain_pages(yf_pool* pool, int32_t n, const int32_t* pages) {
    if (!pool || n < 0 || (n > 0 && !pages)) return fail(YF_E_INVALID, "bad retain arguments");
    for (int i = 0; i < n; ++i) {
        if (pages[i] < 0 || pages[i] >= pool->desc.n_pages) return fail(YF_E_RANGE, "page %d out of range", pages[i]);
        if (pool->refcount[pages[i]] <= 0) return fail(YF_E_STATE, "retain of free page %d", pages[i]);
    }
    for (int i = 0; i < n; ++i) pool->refcount[pages[i]] += 1;
    return YF_OK;
}

int yf_pool_free_pages(yf_pool* pool, int32_t n, const int32_t* pages) {
    if (!pool || n < 0 || (n > 0 && !pages)) return fail(YF_E_INVALID, "bad free arguments");
    // Validate the whole list first (counting repeats) so that a bad list changes nothing.
    std::vector<int32_t> drops;
    drops.reserve(n);
    for (int i = 0; i < n; ++i) {
        const int32_t pg = pages[i];
        if (pg < 0 || pg >= pool->desc.n_pages) return fail(YF_E_RANGE, "page %d out of range", pg);
        int seen = 0;
        for (int32_t x : drops) seen += (x == pg);
        if (pool->refcount[pg] - seen <= 0) return fail(YF_E_STATE, "free of free page %d", pg);
        drops.push_back(pg);
    }
    for (int32_t pg : drops)
        if (--pool->refcount[pg] == 0) pool->free_stack.push_back(pg);
    return YF_OK;
}

int yf_pool_free_count(const yf_pool* pool, int32_t* out_free) {
    if (!pool || !out_free) return fail(YF_E_INVALID, "null argument");
    *out_free = (int32_t)pool->free_stack.size();
    return YF_OK;
}

int yf_pool_refcount(const yf_pool* pool, int32_t page, int32_t* out) {
    if (!pool || !out) return fail(YF_E_INVALID, "null argument");
    if (page < 0 || page >= pool->desc.n_pages) return fail(YF_E_RANGE, "page %d out of range", page);
    *out = pool->refcount[page];
    return YF_OK;
}

int yf_pool_status(yf_pool* pool, uint32_t* out_bits, int clear) {
    if (!pool || !out_bits) return fail(YF_E_INVALID, "null argument");
    if (!pool->d_status) return fail(YF_E_INVALID, "host-only pool has no device status");
    cudaSetDevice(pool->desc.device);
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(out_bits, pool->d_status, sizeof(uint32_t), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && clear) e = cudaMemset(pool->d_status, 0, sizeof(uint32_t));
    // a merge wait that gave up left its unit's arrival counter mid-count (late parts may still
    // have arrived after the mergers left): start every counter from zero again
    if (e == cudaSuccess && clear && (*out_bits & YF_DEV_TIMEOUT))
        e = cudaMemset(pool->d_counters, 0, sizeof(uint32_t) * ((size_t)kMaxCombineUnits + kMaxGroupCounters));
    if (e == cudaSuccess && clear) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "status read");
    return YF_OK;
}

static int check_options(const yf_attn_options* o) {
    if (!o) return fail(YF_E_INVALID, "options are null");
    if (o->schedule != YF_SCHED_AUTO && o->schedule != YF_SCHED_CHUNKED && o->schedule != YF_SCHED_PERSISTENT)
        return fail(YF_E_INVALID, "schedule %d unknown", o->schedule);
    if (o->chunk_tiles < 0) return fail(YF_E_INVALID, "chunk_tiles %d < 0", o->chunk_tiles);
    if (o->copy_stages != 0 && o->copy_stages != 3)
        return fail(YF_E_INVALID, "copy_stages %d: 0 (default) or 3", o->copy_stages);
    if (o->merge != YF_MERGE_IN_KERNEL && o->merge != YF_MERGE_SEPARATE)
        return fail(YF_E_INVALID, "merge %d unknown", o->merge);
    if (o->prefill_kernel != YF_PREFILL_AUTO && o->prefill_kernel != YF_PREFILL_SPLITKV)
        return fail(YF_E_INVALID, "prefill_kernel %d unknown", o->prefill_kernel);
    if (o->wait_limit_us > 60u * 1000000u) return fail(YF_E_INVALID, "wait_limit_us above 60 s");
    if (o->launch != YF_LAUNCH_PLAIN && o->launch != YF_LAUNCH_COOPERATIVE)
        return fail(YF_E_INVALID, "launch %d unknown", o->launch);
    if (o->verify_kernel != YF_VERIFY_AUTO && o->verify_kernel != YF_VERIFY_TCGEN05)
        return fail(YF_E_INVALID, "verify_kernel %d unknown", o->verify_kernel);
    for (int32_t r : o->reserved)
        if (r) return fail(YF_E_INVALID, "reserved option fields must be zero");
    return YF_OK;
}

int yf_pool_set_options(yf_pool* pool, const yf_attn_options* opts) {
    if (!pool) return fail(YF_E_INVALID, "pool is null");
    const int rc = check_options(opts);
    if (rc) return rc;
    pool->opts = *opts;
    return YF_OK;
}

int yf_pool_get_options(const yf_pool* pool, yf_attn_options* out) {
    if (!pool || !out) return fail(YF_E_INVALID, "null argument");
    *out = pool->opts;
    return YF_OK;
}

int yf_pool_plant_counter(yf_pool* pool, int32_t index, uint32_t value, void* stream) {
    if (!pool) return fail(YF_E_INVALID, "pool is null");
    if (!pool->d_counters) return fail(YF_E_INVALID, "host-only pool has no device counters");
    if (index < 0 || index >= kMaxCombineUnits + kMaxGroupCounters)
        return fail(YF_E_RANGE, "counter %d out of range", index);
    cudaSetDevice(pool->desc.device);
    store_word_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(pool->d_counters + index, value);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? YF_OK : cuda_fail(e, "counter store");
}

// Page copies between the pool and a snapshot buffer: one cudaMemcpyAsync per
// run of consecutive page ids.
static int copy_pages(yf_pool* pool, int32_t layer, int32_t n, const int32_t* pages, uint8_t* ext,
                      bool to_pool, void* stream) {
    if (!pool || n < 0 || (n > 0 && (!pages || !ext))) return fail(YF_E_INVALID, "bad page-copy arguments");
    if (!pool->base) return fail(YF_E_INVALID, "host-only pool has no device memory");
    if (layer < 0 || layer >= pool->desc.n_layers) return fail(YF_E_RANGE, "layer %d out of range", layer);
    for (int i = 0; i < n; ++i)
        if (pages[i] < 0 || pages[i] >= pool->desc.n_pages) return fail(YF_E_RANGE, "page %d out of range", pages[i]);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint8_t* lb = pool->base + (size_t)layer * pool->layer_bytes;
    const size_t pb = pool->page_bytes;
    int i = 0;
    while (i < n) {
        int j = i + 1;
        while (j < n && pages[j] == pages[j - 1] + 1) ++j;
        uint8_t* dev = lb + (size_t)pages[i] * pb;
        uint8_t* ext_i = ext + (size_t)i * pb;
        const cudaError_t e = to_pool ? cudaMemcpyAsync(dev, ext_i, (size_t)(j - i) * pb, cudaMemcpyDefault, s)
                                      : cudaMemcpyAsync(ext_i, dev, (size_t)(j - i) * pb, cudaMemcpyDefault, s);
        if (e != cudaSuccess) return cuda_fail(e, "page copy");
        i = j;
    }
    return YF_OK;
}

int yf_pool_export_pages(yf_pool* pool, int32_t layer, int32_t n, const int32_t* pages, void* dst, void* stream) {
    return copy_pages(pool, layer, n, pages, static_cast<uint8_t*>(dst), false, stream);
}

int yf_pool_restore_pages(yf_pool* pool, int32_t layer, int32_t n, const int32_t* pages, const void* src,
                          void* stream) {
    return copy_pages(pool, layer, n, pages, static_cast<uint8_t*>(const_cast<void*>(src)), true, stream);
}

// ---- attention entry points ------------------------------------------------

static int check_attn(const yf_pool* pool, int32_t layer, const void* q, int32_t hq, const void* cu_k,
                      const void* bt, int32_t max_blocks, int32_t batch, int32_t max_q, int32_t max_k,
                      float scale, const void* out) {
    if (!pool) return fail(YF_E_INVALID, "pool is null");
    if (!pool->base) return fail(YF_E_INVALID, "host-only pool has no device memory");
    if (batch < 0) return fail(YF_E_INVALID, "batch %d < 0", batch);
    if (batch == 0) return YF_OK;
    if (!q || !cu_k || !bt || !out) return fail(YF_E_INVALID, "null device pointer");
    if (!aligned(q, 16) || !aligned(out, 16)) return fail(YF_E_INVALID, "q and out must be 16-byte aligned");
    if (layer < 0 || layer >= pool->desc.n_layers) return fail(YF_E_RANGE, "layer %d out of range", layer);
    const int H = pool->desc.n_kv_heads;
    if (hq < H || hq % H != 0) return fail(YF_E_INVALID, "n_q_heads %d is not a multiple of n_kv_heads %d", hq, H);
    if (max_blocks < 1) return fail(YF_E_INVALID, "max_blocks %d < 1", max_blocks);
    if (max_q < 1) return fail(YF_E_INVALID, "max_seqlen_q %d < 1", max_q);
    if (max_k < 0) return fail(YF_E_INVALID, "max_seqlen_k %d < 0", max_k);
    if ((long long)max_k > (long long)max_blocks * pool->desc.page_size)
        return fail(YF_E_RANGE, "max_seqlen_k %d exceeds max_blocks*page_size %lld", max_k,
                    (long long)max_blocks * pool->desc.page_size);
    if (!(scale == scale) || scale <= 0.0f || scale > 1e30f) return fail(YF_E_INVALID, "scale must be finite and > 0");
    if (batch > 65535) return fail(YF_E_UNSUPPORTED, "batch %d > 65535", batch);
    if ((long long)H * ((long long)(hq / H) * max_q + 7) / 8 > 65535)
        return fail(YF_E_UNSUPPORTED, "too many query rows per kv head for one launch");
    return YF_OK;
}

size_t yf_attn_workspace_size(const yf_pool* pool, int32_t hq, int32_t batch, int32_t max_q, int32_t max_k) {
    if (!pool || batch <= 0 || hq < pool->desc.n_kv_heads || hq % pool->desc.n_kv_heads) return 0;
    if (max_q > kMaxTreeRowsHost && (prefill_tc_applies(pool, hq, max_q) || prefill_tc256_applies(pool, hq, max_q)))
        return 0;
    // query blocks a causal or a tree verify can take: room for every schedule that may run
    size_t ws = plan_split(pool, hq, batch, max_q, max_k, false).ws_bytes;
    if (max_q <= 1 || max_q > kMaxTreeRowsHost) return ws;
    ws = std::max(ws, plan_split(pool, hq, batch, max_q, max_k, true).ws_bytes);
    if (verify_tc_applies(pool, hq, max_q, false) || verify_tc_applies(pool, hq, max_q, true))
        ws = std::max(ws, plan_verify(pool, hq, batch, max_q, max_k).ws_bytes);
    return ws;
}

static int run_attn(yf_pool* pool, int32_t layer, const void* q, int32_t hq, const uint32_t* cu_q,
                    const uint32_t* cu_k, const uint32_t* bt, int32_t max_blocks, int32_t batch, int32_t max_q,
                    int32_t max_k, float scale, void* out, void* ws, size_t ws_bytes, void* stream,
                    float* part_o = nullptr, float* part_lse = nullptr, const int32_t* trie = nullptr) {
    const int rc =
        check_attn(pool, layer, q, hq, cu_k, bt, max_blocks, batch, max_q, max_k, scale, part_o ? part_o : out);
    if (rc || batch == 0) return rc;
    if (part_o && (!part_lse || !aligned(part_lse, 4))) return fail(YF_E_INVALID, "lse output null or misaligned");
    const bool tc = !part_o && !trie && cu_q && prefill_tc_applies(pool, hq, max_q);
    const bool tc256 = !part_o && !trie && cu_q && prefill_tc256_applies(pool, hq, max_q);
    const bool vtc = !tc && !tc256 && !part_o && cu_q && verify_tc_applies(pool, hq, max_q, trie != nullptr);
    const SplitPlan plan = plan_split(pool, hq, batch, max_q, max_k, trie != nullptr);
    const VerifyPlan vplan = vtc ? plan_verify(pool, hq, batch, max_q, max_k) : VerifyPlan{};
    const size_t need = (tc || tc256) ? 0 : (vtc ? vplan.ws_bytes : plan.ws_bytes);
    if (need > 0 && (!ws || ws_bytes < need || !aligned(ws, 16)))
        return fail(YF_E_WORKSPACE, "workspace of %zu bytes (16-byte aligned) needed, %zu given", need,
                    ws ? ws_bytes : (size_t)0);
    AttnArgs a;
    a.pool = pool;
    a.layer = layer;
    a.q = static_cast<const __half*>(q);
    a.n_q_heads = hq;
    a.cu_q = cu_q;
    a.cu_k = cu_k;
    a.block_table = bt;
    a.max_blocks = max_blocks;
    a.batch = batch;
    a.max_seqlen_q = max_q;
    a.max_seqlen_k = max_k;
    a.scale = scale;
    a.out = static_cast<__half*>(out);
    a.workspace = ws;
    a.workspace_bytes = ws_bytes;
    a.stream = static_cast<cudaStream_t>(stream);
    a.part_o = part_o;
    a.part_lse = part_lse;
    a.trie = trie;
    if (tc) return launch_prefill_tc(a);
    if (tc256) return launch_prefill_tc256(a);
    if (vtc) return launch_verify_tc(a, vplan);
    return launch_splitkv(a, plan);
}

int yf_attn_decode(yf_pool* pool, int32_t layer, const void* q, int32_t hq, const uint32_t* cu_k,
                   const uint32_t* bt, int32_t max_blocks, int32_t batch, int32_t max_k, float scale, void* out,
                   void* ws, size_t ws_bytes, void* stream) {
    return run_attn(pool, layer, q, hq, nullptr, cu_k, bt, max_blocks, batch, 1, max_k, scale, out, ws, ws_bytes,
                    stream);
}

int yf_attn_decode_partial(yf_pool* pool, int32_t layer, const void* q, int32_t hq, const uint32_t* cu_k,
                           const uint32_t* bt, int32_t max_blocks, int32_t batch, int32_t max_k, float scale,
                           float* o_part, float* lse_part, void* ws, size_t ws_bytes, void* stream) {
    if (batch > 0 && !o_part) return fail(YF_E_INVALID, "partial O output is null");
    return run_attn(pool, layer, q, hq, nullptr, cu_k, bt, max_blocks, batch, 1, max_k, scale, nullptr, ws, ws_bytes,
                    stream, o_part, lse_part);
}

int yf_attn_prefill(yf_pool* pool, int32_t layer, const void* q, int32_t hq, const uint32_t* cu_q,
                    const uint32_t* cu_k, const uint32_t* bt, int32_t max_blocks, int32_t batch, int32_t max_q,
                    int32_t max_k, float scale, void* out, void* ws, size_t ws_bytes, void* stream) {
    if (batch > 0 && !cu_q) return fail(YF_E_INVALID, "cu_seqlens_q is null");
    return run_attn(pool, layer, q, hq, cu_q, cu_k, bt, max_blocks, batch, max_q, max_k, scale, out, ws, ws_bytes,
                    stream);
}

int yf_attn_verify_tree(yf_pool* pool, int32_t layer, const void* q, int32_t hq, const uint32_t* cu_q,
                        const uint32_t* cu_k, const uint32_t* bt, int32_t max_blocks, int32_t batch, int32_t max_q,
                        int32_t max_k, float scale, const int32_t* trie_ranges, void* out, void* ws,
                        size_t ws_bytes, void* stream) {
    if (batch > 0 && !cu_q) return fail(YF_E_INVALID, "cu_seqlens_q is null");
    if (batch > 0 && (!trie_ranges || !aligned(trie_ranges, 8)))
        return fail(YF_E_INVALID, "trie_ranges null or not 8-byte aligned");
    if (max_q > kMaxTreeRowsHost)
        return fail(YF_E_UNSUPPORTED, "tree verify of %d rows per entry (at most %d)", max_q, kMaxTreeRowsHost);
    return run_attn(pool, layer, q, hq, cu_q, cu_k, bt, max_blocks, batch, max_q, max_k, scale, out, ws, ws_bytes,
                    stream, nullptr, nullptr, batch > 0 ? trie_ranges : nullptr);
}

}  // extern "C"

namespace yf {

int decode_exchange(yf_pool* pool, int32_t layer, const void* q, int32_t hq, const uint32_t* cu_k, const uint32_t* bt,
                    int32_t max_blocks, int32_t batch, int32_t max_k, float scale, const XFuse& xf, void* ws,
                    size_t ws_bytes, void* stream, bool* fused) {
    *fused = false;
    const int rc = check_attn(pool, layer, q, hq, cu_k, bt, max_blocks, batch, 1, max_k, scale, xf.out);
    if (rc || batch == 0) return rc;
    const SplitPlan plan = plan_split(pool, hq, batch, 1, max_k, false);
    if (!plan.cluster || (long long)batch * pool->desc.n_kv_heads * kClusterCtas > kXMaxSlices ||
        xf.n_seq > kXMaxSeq)
        return YF_OK;
    if (plan.ws_bytes > 0 && (!ws || ws_bytes < plan.ws_bytes || !aligned(ws, 16)))
        return fail(YF_E_WORKSPACE, "workspace of %zu bytes (16-byte aligned) needed, %zu given", plan.ws_bytes,
                    ws ? ws_bytes : (size_t)0);
    AttnArgs a;
    a.pool = pool;
    a.layer = layer;
    a.q = static_cast<const __half*>(q);
    a.n_q_heads = hq;
    a.cu_q = nullptr;
    a.cu_k = cu_k;
    a.block_table = bt;
    a.max_blocks = max_blocks;
    a.batch = batch;
    a.max_seqlen_q = 1;
    a.max_seqlen_k = max_k;
    a.scale = scale;
    a.out = nullptr;
    a.workspace = ws;
    a.workspace_bytes = ws_bytes;
    a.stream = static_cast<cudaStream_t>(stream);
    a.xf = &xf;
    *fused = true;
    return launch_splitkv(a, plan);
}

}  // namespace yf

