// Snapshot wire records of pool pages, framed and checksummed on the GPU.
//
// The prefix cache's on-disk page format (docs/plans/2026-08-27-tiered-kv-cache.md:143-145,237-251):
// append-only records [u64 chain_hash][u32 page_index][u32 payload_len][u32 crc32c][payload],
// little-endian, packed, with a CRC-32C per page against media corruption.  Here a record's
// payload is one pool page in every layer (layer 0 first), and the records are built and checked
// where the pages live: the export kernel copies each page into its record and computes the CRC
// in the same pass, the import kernel checks the CRC and restores only intact records, so the
// host moves one contiguous, already framed buffer in either direction.
//
// CRC-32C: the Castagnoli polynomial, reflected (0x82F63B78), register preset and final xor
// 0xFFFFFFFF.  A record's payload moves through shared memory in blocks of <= 32 KB (coalesced
// loads and stores); each thread runs the byte-table (slicing-by-4) update over a contiguous run
// of the staged words from a zero register, and the runs and then the blocks are joined with the
// linearity of the CRC register: R(0, A||B) = R(0, A) * x^(8|B|) ^ R(0, B) mod P, the product
// taken in the reflected representation (x^0 in bit 31), as zlib's crc32_combine does.
#include <cuda_runtime.h>

#include <algorithm>

#include "yf_device.cuh"
#include "yf_internal.h"

namespace yf {
namespace {

constexpr uint32_t kCrcPoly = 0x82F63B78u;
constexpr int kRecThreads = 256;
constexpr int kRecHeader = 20;

// a * b mod P (reflected; bit 31 = x^0), 32 fixed steps.
__host__ __device__ __forceinline__ uint32_t gf2_mulmod(uint32_t a, uint32_t b) {
    uint32_t p = 0;
#pragma unroll 4
    for (int i = 0; i < 32; ++i) {
        if (a & (0x80000000u >> i)) p ^= b;
        b = (b & 1u) ? (b >> 1) ^ kCrcPoly : b >> 1;
    }
    return p;
}

// x^(8n) mod P (n < 2^29), by squaring.
__host__ uint32_t x8n_mod(unsigned long long n) {
    uint32_t x2k = 0x40000000u;  // x^(2^k), from x^1
    uint32_t p = 0x80000000u;    // x^0
    for (n <<= 3; n; n >>= 1) {
        if (n & 1ull) p = gf2_mulmod(x2k, p);
        x2k = gf2_mulmod(x2k, x2k);
    }
    return p;
}

// The CTA's slicing-by-4 tables in shared memory (T[0] is the byte table).
__device__ void build_tables(uint32_t (*T)[256]) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
        uint32_t c = (uint32_t)i;
        for (int b = 0; b < 8; ++b) c = (c & 1u) ? (c >> 1) ^ kCrcPoly : c >> 1;
        T[0][i] = c;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
        uint32_t c = T[0][i];
        for (int k = 1; k < 4; ++k) {
            c = (c >> 8) ^ T[0][c & 0xffu];
            T[k][i] = c;
        }
    }
    __syncthreads();
}

__device__ __forceinline__ uint32_t crc_word(uint32_t c, uint32_t w, const uint32_t (*T)[256]) {
    c ^= w;
    return T[3][c & 0xffu] ^ T[2][(c >> 8) & 0xffu] ^ T[1][(c >> 16) & 0xffu] ^ T[0][c >> 24];
}

struct RecParams {
    uint8_t* base;         // pool base (layer 0)
    size_t layer_bytes;
    size_t page_bytes;
    int n_layers;
    int n_pages;
    const int32_t* pages;
    const unsigned long long* hashes;
    const uint32_t* page_index;
    uint8_t* records;      // export: out; import: in
    const uint8_t* records_in;
    uint32_t* ok;
    size_t rec_bytes;
    uint32_t* status;
    int blk_words;         // words of one staged block (a page is 2^j blocks)
    int blks_per_page;
    // x^(8 * bytes of the block after thread t's words) mod P, x^(8 * block bytes) mod P, and the
    // preset's term 0xFFFFFFFF * x^(8 * payload) mod P
    uint32_t shift[kRecThreads];
    uint32_t blk_shift;
    uint32_t preset;
};

constexpr int kBlkMaxBytes = 32768;

// Thread t's words of a staged block: [w0, w1), contiguous, in thread order.
__device__ __forceinline__ void words_of(int n, int& w0, int& w1) {
    w0 = (int)((long long)threadIdx.x * n / kRecThreads);
    w1 = (int)((long long)(threadIdx.x + 1) * n / kRecThreads);
}

// The block's CRC register from a zero preset (the staged words), joined across the threads.
__device__ uint32_t block_crc(const uint32_t* blk, int n, uint32_t shift, const uint32_t (*T)[256], uint32_t* red) {
    int w0, w1;
    words_of(n, w0, w1);
    uint32_t c = 0;
    for (int w = w0; w < w1; ++w) c = crc_word(c, blk[w], T);
    uint32_t v = w1 > w0 ? gf2_mulmod(shift, c) : 0u;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v ^= __shfl_xor_sync(0xffffffffu, v, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    uint32_t r = 0;
    for (int k = 0; k < kRecThreads / 32; ++k) r ^= red[k];
    __syncthreads();  // red and the staged block are reused by the next block
    return r;
}

// One CTA per record: the page's blocks (every layer) are staged through shared memory with
// coalesced loads and stores, and each thread checksums a contiguous run of the staged words.
__global__ void __launch_bounds__(kRecThreads) export_records_kernel(const RecParams p) {
    __shared__ uint32_t T[4][256];
    __shared__ uint32_t red[kRecThreads / 32];
    __shared__ __align__(16) uint32_t blk[kBlkMaxBytes / 4];
    build_tables(T);
    const int r = blockIdx.x;
    const int page = p.pages[r];
    uint8_t* rec = p.records + (size_t)r * p.rec_bytes;
    const size_t payload = (size_t)p.n_layers * p.page_bytes;
    if (page < 0 || page >= p.n_pages) {
        // a header that every import rejects (length 0), so that a reused staging buffer never
        // passes an older record off as this one
        if (threadIdx.x == 0) {
            atomicOr(p.status, YF_DEV_BAD_PAGE);
            uint32_t* h = reinterpret_cast<uint32_t*>(rec);
            for (int k = 0; k < 5; ++k) h[k] = 0u;
        }
        return;
    }
    const int nw = p.blk_words;
    uint32_t* dst = reinterpret_cast<uint32_t*>(rec + kRecHeader);
    uint32_t acc = 0;  // the payload's CRC register from a zero preset, over the blocks so far
    for (int l = 0; l < p.n_layers; ++l) {
        const uint8_t* pg = p.base + (size_t)l * p.layer_bytes + (size_t)page * p.page_bytes;
        for (int bi = 0; bi < p.blks_per_page; ++bi) {
            const uint4* g = reinterpret_cast<const uint4*>(pg + (size_t)bi * nw * 4);
            for (int k = threadIdx.x; k < nw / 4; k += kRecThreads) reinterpret_cast<uint4*>(blk)[k] = __ldcs(g + k);
            __syncthreads();
            uint32_t* d = dst + ((size_t)l * p.blks_per_page + bi) * nw;
            for (int k = threadIdx.x; k < nw; k += kRecThreads) d[k] = blk[k];
            const uint32_t b = block_crc(blk, nw, p.shift[threadIdx.x], T, red);
            acc = gf2_mulmod(p.blk_shift, acc) ^ b;
        }
    }
    if (threadIdx.x == 0) {
        uint32_t* h = reinterpret_cast<uint32_t*>(rec);
        const unsigned long long hash = p.hashes ? p.hashes[r] : 0ull;
        h[0] = (uint32_t)hash;
        h[1] = (uint32_t)(hash >> 32);
        h[2] = p.page_index ? p.page_index[r] : (uint32_t)page;
        h[3] = (uint32_t)payload;
        h[4] = p.preset ^ acc ^ 0xFFFFFFFFu;
    }
}

__global__ void __launch_bounds__(kRecThreads) import_records_kernel(const RecParams p) {
    __shared__ uint32_t T[4][256];
    __shared__ uint32_t red[kRecThreads / 32];
    __shared__ __align__(16) uint32_t blk[kBlkMaxBytes / 4];
    __shared__ int s_good;
    build_tables(T);
    const int r = blockIdx.x;
    const int page = p.pages[r];
    const uint8_t* rec = p.records_in + (size_t)r * p.rec_bytes;
    const size_t payload = (size_t)p.n_layers * p.page_bytes;
    const uint32_t* h = reinterpret_cast<const uint32_t*>(rec);
    const uint32_t* src = reinterpret_cast<const uint32_t*>(rec + kRecHeader);
    const int nw = p.blk_words;
    const int n_blk = p.n_layers * p.blks_per_page;
    uint32_t acc = 0;
    for (int bi = 0; bi < n_blk; ++bi) {
        const uint32_t* s = src + (size_t)bi * nw;
        for (int k = threadIdx.x; k < nw; k += kRecThreads) blk[k] = __ldcg(s + k);
        __syncthreads();
        const uint32_t b = block_crc(blk, nw, p.shift[threadIdx.x], T, red);
        acc = gf2_mulmod(p.blk_shift, acc) ^ b;
    }
    if (threadIdx.x == 0) {
        const bool page_ok = page >= 0 && page < p.n_pages;
        if (!page_ok) atomicOr(p.status, YF_DEV_BAD_PAGE);
        s_good = page_ok && h[3] == (uint32_t)payload && h[4] == (p.preset ^ acc ^ 0xFFFFFFFFu);
        p.ok[r] = s_good ? 1u : 0u;
    }
    __syncthreads();
    if (!s_good) return;
    // second pass: the intact payload into the page, 4-byte loads (the record is only 4-byte
    // aligned) and 16-byte stores
    for (int l = 0; l < p.n_layers; ++l) {
        uint4* pg = reinterpret_cast<uint4*>(p.base + (size_t)l * p.layer_bytes + (size_t)page * p.page_bytes);
        const uint32_t* s = src + (size_t)l * (p.page_bytes / 4);
        for (size_t k = threadIdx.x; k < p.page_bytes / 16; k += kRecThreads)
            pg[k] = make_uint4(__ldcg(s + 4 * k), __ldcg(s + 4 * k + 1), __ldcg(s + 4 * k + 2), __ldcg(s + 4 * k + 3));
    }
}

int launch_records(yf_pool* pool, int32_t n, const int32_t* pages, const unsigned long long* hashes,
                   const uint32_t* page_index, void* records, uint32_t* ok, bool do_export, void* stream) {
    if (!pool) return fail(YF_E_INVALID, "pool is null");
    if (!pool->base) return fail(YF_E_INVALID, "host-only pool has no device memory");
    if (n < 0) return fail(YF_E_INVALID, "n %d < 0", n);
    if (n == 0) return YF_OK;
    if (!pages || !records || (!do_export && !ok)) return fail(YF_E_INVALID, "null device pointer");
    if (!aligned(records, 4)) return fail(YF_E_INVALID, "records must be 4-byte aligned");
    if (n > 0x7fffffff / 2) return fail(YF_E_UNSUPPORTED, "too many records");
    RecParams p;
    p.base = pool->base;
    p.layer_bytes = pool->layer_bytes;
    p.page_bytes = pool->page_bytes;
    p.n_layers = pool->desc.n_layers;
    p.n_pages = pool->desc.n_pages;
    p.pages = pages;
    p.hashes = hashes;
    p.page_index = page_index;
    p.records = static_cast<uint8_t*>(records);
    p.records_in = static_cast<const uint8_t*>(records);
    p.ok = ok;
    p.rec_bytes = kRecHeader + (size_t)pool->desc.n_layers * pool->page_bytes;
    p.status = pool->d_status;
    const size_t payload = p.rec_bytes - kRecHeader;
    if (payload >= (1ull << 29)) return fail(YF_E_UNSUPPORTED, "record payload of %zu bytes", payload);
    // a page = 2^j equal blocks of at most 32 KB (page bytes are 17 x 2^m)
    size_t blk = pool->page_bytes;
    int bpp = 1;
    while (blk > (size_t)kBlkMaxBytes && blk % 32 == 0) {
        blk /= 2;
        bpp *= 2;
    }
    if (blk > (size_t)kBlkMaxBytes || blk % 16) return fail(YF_E_UNSUPPORTED, "page of %zu bytes", pool->page_bytes);
    p.blk_words = (int)(blk / 4);
    p.blks_per_page = bpp;
    if (pool->crc_ops.size() != kRecThreads + 2) {  // the record shape is fixed per pool: once
        std::vector<uint32_t> ops(kRecThreads + 2);
        const int nw = p.blk_words;
        for (int t = 0; t < kRecThreads; ++t) {
            const int w1 = (int)((long long)(t + 1) * nw / kRecThreads);
            ops[t] = x8n_mod((unsigned long long)(nw - w1) * 4);
        }
        ops[kRecThreads] = x8n_mod(blk);
        ops[kRecThreads + 1] = gf2_mulmod(x8n_mod(payload), 0xFFFFFFFFu);
        pool->crc_ops.swap(ops);
    }
    for (int t = 0; t < kRecThreads; ++t) p.shift[t] = pool->crc_ops[t];
    p.blk_shift = pool->crc_ops[kRecThreads];
    p.preset = pool->crc_ops[kRecThreads + 1];
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (do_export)
        export_records_kernel<<<n, kRecThreads, 0, s>>>(p);
    else
        import_records_kernel<<<n, kRecThreads, 0, s>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? YF_OK : cuda_fail(e, "snapshot record launch");
}

}  // namespace
}  // namespace yf

using namespace yf;

extern "C" size_t yf_pool_record_bytes(const yf_pool_desc* desc) {
    const size_t per_layer = yf_pool_page_head_bytes(desc) * (desc ? (size_t)desc->n_kv_heads : 0);
    if (!per_layer) return 0;
    return kRecHeader + (size_t)desc->n_layers * per_layer;
}

extern "C" int yf_pool_export_records(yf_pool* pool, int32_t n, const int32_t* d_pages,
                                      const uint64_t* d_chain_hashes, const uint32_t* d_page_indices,
                                      void* d_records, void* stream) {
    return launch_records(pool, n, d_pages, reinterpret_cast<const unsigned long long*>(d_chain_hashes),
                          d_page_indices, d_records, nullptr, true, stream);
}

extern "C" int yf_pool_import_records(yf_pool* pool, int32_t n, const int32_t* d_pages, const void* d_records,
                                      uint32_t* d_ok, void* stream) {
    return launch_records(pool, n, d_pages, nullptr, nullptr, const_cast<void*>(d_records), d_ok, false, stream);
}
