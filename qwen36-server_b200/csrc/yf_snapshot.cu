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
#include <vector>

#include "yf_device.cuh"
#include "yf_internal.h"

namespace yf {
namespace {

constexpr uint32_t kCrcPoly = 0x82F63B78u;
constexpr int kRecThreads = 256;
// CRC combine operators of a pool's records: a shift per thread, the block shift, the preset,
// a shift per token lane and the token block's multiplier (computed when the pool is created)
constexpr size_t kRecOps = kRecThreads + 35;

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
    int P;                 // tokens per page (= token ids per record)
    const int32_t* pages;
    const unsigned long long* hashes;       // export: chain hash per record, or null (0)
    const unsigned long long* prev_hashes;  // export: the previous page's chain hash, or null (0)
    const uint32_t* page_index;             // export: position in the chain, or null (the page id)
    const uint32_t* tokens;                 // export: [n][P] token ids, or null (zeros)
    const unsigned long long* expect_hashes;  // import: chain hash each record must carry, or null
    const uint32_t* expect_tokens;            // import: [n][P] token ids each record must carry, or null
    uint8_t* records;      // export: out; import: in (16-byte aligned, stride rec_bytes)
    uint32_t* ok;
    size_t rec_bytes;
    size_t hdr_bytes;      // 32 + 4 * P
    uint32_t* status;
    int blk_words;         // words of one staged block (a page is 2^j blocks)
    int blks_per_page;
    // x^(8 * bytes of the block after thread t's words) mod P, x^(8 * block bytes) mod P
    uint32_t shift[kRecThreads];
    uint32_t blk_shift;
    // the preset's term 0xFFFFFFFF * x^(8 * (token bytes + payload)) mod P
    uint32_t preset;
    // x^(8 * token bytes after lane l's token words) and x^(8 * payload bytes): the token block's
    // register joined in front of the payload's
    uint32_t tok_shift[32];
    uint32_t tok_mul;
};

// Layout of the record header in 32-bit words.
constexpr int kHdrChain = 0, kHdrPrev = 2, kHdrIndex = 4, kHdrTokens = 5, kHdrLen = 6, kHdrCrc = 7;
constexpr int kHdrWords = 8;

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

// Warp 0: the CRC register (zero preset) of the record's P token words, on every lane.
__device__ __forceinline__ uint32_t token_crc(const uint32_t* tok, int P, const RecParams& p, const uint32_t (*T)[256]) {
    const int lane = threadIdx.x & 31;
    const int w0 = lane * P / 32, w1 = (lane + 1) * P / 32;
    uint32_t c = 0;
    for (int w = w0; w < w1; ++w) c = crc_word(c, tok[w], T);
    uint32_t v = w1 > w0 ? gf2_mulmod(p.tok_shift[lane], c) : 0u;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v ^= __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// One CTA per record: the page's blocks (every layer) are staged through shared memory with
// coalesced 16-byte loads and stores, and each thread checksums a contiguous run of the staged
// words; warp 0 writes and checksums the token ids first.
__global__ void __launch_bounds__(kRecThreads) export_records_kernel(const RecParams p) {
    __shared__ uint32_t T[4][256];
    __shared__ uint32_t red[kRecThreads / 32];
    __shared__ __align__(16) uint32_t blk[kBlkMaxBytes / 4];
    build_tables(T);
    const int r = blockIdx.x;
    const int page = p.pages[r];
    uint8_t* rec = p.records + (size_t)r * p.rec_bytes;
    uint32_t* h = reinterpret_cast<uint32_t*>(rec);
    const size_t payload = (size_t)p.n_layers * p.page_bytes;
    if (page < 0 || page >= p.n_pages) {
        // a header that every import rejects (length 0), so that a reused staging buffer never
        // passes an older record off as this one
        if (threadIdx.x == 0) {
            atomicOr(p.status, YF_DEV_BAD_PAGE);
            for (int k = 0; k < kHdrWords; ++k) h[k] = 0u;
        }
        return;
    }
    uint32_t tok_reg = 0;
    if (threadIdx.x < 32) {
        uint32_t* tw = h + kHdrWords;
        for (int i = threadIdx.x; i < p.P; i += 32) tw[i] = p.tokens ? p.tokens[(size_t)r * p.P + i] : 0u;
        __syncwarp();
        tok_reg = token_crc(tw, p.P, p, T);
    }
    const int nw = p.blk_words;
    uint4* dst = reinterpret_cast<uint4*>(rec + p.hdr_bytes);
    uint32_t acc = 0;  // the payload's CRC register from a zero preset, over the blocks so far
    for (int l = 0; l < p.n_layers; ++l) {
        const uint8_t* pg = p.base + (size_t)l * p.layer_bytes + (size_t)page * p.page_bytes;
        for (int bi = 0; bi < p.blks_per_page; ++bi) {
            const uint4* g = reinterpret_cast<const uint4*>(pg + (size_t)bi * nw * 4);
            uint4* d = dst + ((size_t)l * p.blks_per_page + bi) * (nw / 4);
            for (int k = threadIdx.x; k < nw / 4; k += kRecThreads) {
                const uint4 w = __ldcs(g + k);
                reinterpret_cast<uint4*>(blk)[k] = w;
                d[k] = w;
            }
            __syncthreads();
            const uint32_t b = block_crc(blk, nw, p.shift[threadIdx.x], T, red);
            acc = gf2_mulmod(p.blk_shift, acc) ^ b;
        }
    }
    if (threadIdx.x == 0) {
        const unsigned long long hash = p.hashes ? p.hashes[r] : 0ull;
        const unsigned long long prev = p.prev_hashes ? p.prev_hashes[r] : 0ull;
        h[kHdrChain] = (uint32_t)hash;
        h[kHdrChain + 1] = (uint32_t)(hash >> 32);
        h[kHdrPrev] = (uint32_t)prev;
        h[kHdrPrev + 1] = (uint32_t)(prev >> 32);
        h[kHdrIndex] = p.page_index ? p.page_index[r] : (uint32_t)page;
        h[kHdrTokens] = (uint32_t)p.P;
        h[kHdrLen] = (uint32_t)payload;
        h[kHdrCrc] = p.preset ^ gf2_mulmod(p.tok_mul, tok_reg) ^ acc ^ 0xFFFFFFFFu;
    }
}

__global__ void __launch_bounds__(kRecThreads) import_records_kernel(const RecParams p) {
    __shared__ uint32_t T[4][256];
    __shared__ uint32_t red[kRecThreads / 32];
    __shared__ __align__(16) uint32_t blk[kBlkMaxBytes / 4];
    __shared__ uint32_t s_verdict;
    build_tables(T);
    const int r = blockIdx.x;
    const int page = p.pages[r];
    const uint8_t* rec = p.records + (size_t)r * p.rec_bytes;
    const size_t payload = (size_t)p.n_layers * p.page_bytes;
    const uint32_t* h = reinterpret_cast<const uint32_t*>(rec);
    const uint4* src = reinterpret_cast<const uint4*>(rec + p.hdr_bytes);
    uint32_t tok_reg = 0;
    bool tok_match = true;
    if (threadIdx.x < 32) {
        const uint32_t* tw = h + kHdrWords;
        tok_reg = token_crc(tw, p.P, p, T);
        bool same = true;
        if (p.expect_tokens)
            for (int i = threadIdx.x; i < p.P; i += 32) same &= __ldcg(tw + i) == p.expect_tokens[(size_t)r * p.P + i];
        tok_match = __all_sync(0xffffffffu, same);
    }
    const int nw = p.blk_words;
    const int n_blk = p.n_layers * p.blks_per_page;
    uint32_t acc = 0;
    for (int bi = 0; bi < n_blk; ++bi) {
        const uint4* s4 = src + (size_t)bi * (nw / 4);
        for (int k = threadIdx.x; k < nw / 4; k += kRecThreads) reinterpret_cast<uint4*>(blk)[k] = __ldcg(s4 + k);
        __syncthreads();
        const uint32_t b = block_crc(blk, nw, p.shift[threadIdx.x], T, red);
        acc = gf2_mulmod(p.blk_shift, acc) ^ b;
    }
    if (threadIdx.x == 0) {
        const bool page_ok = page >= 0 && page < p.n_pages;
        if (!page_ok) atomicOr(p.status, YF_DEV_BAD_PAGE);
        const bool intact = h[kHdrLen] == (uint32_t)payload && h[kHdrTokens] == (uint32_t)p.P &&
                            h[kHdrCrc] == (p.preset ^ gf2_mulmod(p.tok_mul, tok_reg) ^ acc ^ 0xFFFFFFFFu);
        const unsigned long long hash = (unsigned long long)h[kHdrChain] | ((unsigned long long)h[kHdrChain + 1] << 32);
        const bool match = tok_match && (!p.expect_hashes || p.expect_hashes[r] == hash);
        const uint32_t v = !(intact && page_ok) ? YF_REC_REJECTED : (match ? YF_REC_RESTORED : YF_REC_MISMATCH);
        p.ok[r] = v;
        s_verdict = v;
    }
    __syncthreads();
    if (s_verdict != YF_REC_RESTORED) return;
    // second pass: the intact payload into the page with 16-byte loads and stores
    for (int l = 0; l < p.n_layers; ++l) {
        uint4* pg = reinterpret_cast<uint4*>(p.base + (size_t)l * p.layer_bytes + (size_t)page * p.page_bytes);
        const uint4* s4 = src + (size_t)l * (p.page_bytes / 16);
        for (size_t k = threadIdx.x; k < p.page_bytes / 16; k += kRecThreads) pg[k] = __ldcg(s4 + k);
    }
}

// Block split of a page: 2^j equal blocks of at most 32 KB (page bytes are 17 x 2^m).
bool record_blocks(size_t page_bytes, size_t* blk_out, int* bpp_out) {
    size_t blk = page_bytes;
    int bpp = 1;
    while (blk > (size_t)kBlkMaxBytes && blk % 32 == 0) {
        blk /= 2;
        bpp *= 2;
    }
    if (blk > (size_t)kBlkMaxBytes || blk % 16) return false;
    *blk_out = blk;
    *bpp_out = bpp;
    return true;
}

int launch_records(yf_pool* pool, int32_t n, const int32_t* pages, const unsigned long long* hashes,
                   const unsigned long long* prev_hashes, const uint32_t* page_index, const uint32_t* tokens,
                   const unsigned long long* expect_hashes, const uint32_t* expect_tokens, void* records,
                   uint32_t* ok, bool do_export, void* stream) {
    if (!pool) return fail(YF_E_INVALID, "pool is null");
    if (!pool->base) return fail(YF_E_INVALID, "host-only pool has no device memory");
    if (n < 0) return fail(YF_E_INVALID, "n %d < 0", n);
    if (n == 0) return YF_OK;
    if (!pages || !records || (!do_export && !ok)) return fail(YF_E_INVALID, "null device pointer");
    if (!aligned(records, 16)) return fail(YF_E_INVALID, "records must be 16-byte aligned");
    if (n > 0x7fffffff / 2) return fail(YF_E_UNSUPPORTED, "too many records");
    if (pool->crc_ops.size() != kRecOps) return fail(YF_E_UNSUPPORTED, "page of %zu bytes", pool->page_bytes);
    RecParams p;
    p.base = pool->base;
    p.layer_bytes = pool->layer_bytes;
    p.page_bytes = pool->page_bytes;
    p.n_layers = pool->desc.n_layers;
    p.n_pages = pool->desc.n_pages;
    p.P = pool->desc.page_size;
    p.pages = pages;
    p.hashes = hashes;
    p.prev_hashes = prev_hashes;
    p.page_index = page_index;
    p.tokens = tokens;
    p.expect_hashes = expect_hashes;
    p.expect_tokens = expect_tokens;
    p.records = static_cast<uint8_t*>(records);
    p.ok = ok;
    p.hdr_bytes = 4 * kHdrWords + 4 * (size_t)p.P;
    p.rec_bytes = p.hdr_bytes + (size_t)pool->desc.n_layers * pool->page_bytes;
    p.status = pool->d_status;
    size_t blk;
    int bpp;
    record_blocks(pool->page_bytes, &blk, &bpp);
    p.blk_words = (int)(blk / 4);
    p.blks_per_page = bpp;
    for (int t = 0; t < kRecThreads; ++t) p.shift[t] = pool->crc_ops[t];
    p.blk_shift = pool->crc_ops[kRecThreads];
    p.preset = pool->crc_ops[kRecThreads + 1];
    for (int l = 0; l < 32; ++l) p.tok_shift[l] = pool->crc_ops[kRecThreads + 2 + l];
    p.tok_mul = pool->crc_ops[kRecThreads + 34];
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (do_export)
        export_records_kernel<<<n, kRecThreads, 0, s>>>(p);
    else
        import_records_kernel<<<n, kRecThreads, 0, s>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? YF_OK : cuda_fail(e, "snapshot record launch");
}

}  // namespace

// The record CRC's combine operators for this pool's page shape (yf_pool_create).
void init_record_ops(yf_pool* pool) {
    pool->crc_ops.clear();
    size_t blk;
    int bpp;
    if (!record_blocks(pool->page_bytes, &blk, &bpp)) return;  // records refused for this shape
    const int P = pool->desc.page_size;
    const size_t payload = (size_t)pool->desc.n_layers * pool->page_bytes;
    std::vector<uint32_t> ops(kRecOps);
    const int nw = (int)(blk / 4);
    for (int t = 0; t < kRecThreads; ++t) {
        const int w1 = (int)((long long)(t + 1) * nw / kRecThreads);
        ops[t] = x8n_mod((unsigned long long)(nw - w1) * 4);
    }
    ops[kRecThreads] = x8n_mod(blk);
    ops[kRecThreads + 1] = gf2_mulmod(x8n_mod(4ull * P + payload), 0xFFFFFFFFu);
    for (int l = 0; l < 32; ++l) {
        const int w1 = (l + 1) * P / 32;
        ops[kRecThreads + 2 + l] = x8n_mod(4ull * (P - w1));
    }
    ops[kRecThreads + 34] = x8n_mod(payload);
    pool->crc_ops.swap(ops);
}

}  // namespace yf

using namespace yf;

extern "C" size_t yf_pool_record_bytes(const yf_pool_desc* desc) {
    const size_t per_layer = yf_pool_page_head_bytes(desc) * (desc ? (size_t)desc->n_kv_heads : 0);
    if (!per_layer) return 0;
    return 4 * (size_t)kHdrWords + 4 * (size_t)desc->page_size + (size_t)desc->n_layers * per_layer;
}

extern "C" int yf_pool_export_records(yf_pool* pool, int32_t n, const int32_t* d_pages,
                                      const uint64_t* d_chain_hashes, const uint64_t* d_prev_hashes,
                                      const uint32_t* d_page_indices, const uint32_t* d_tokens, void* d_records,
                                      void* stream) {
    return launch_records(pool, n, d_pages, reinterpret_cast<const unsigned long long*>(d_chain_hashes),
                          reinterpret_cast<const unsigned long long*>(d_prev_hashes), d_page_indices, d_tokens,
                          nullptr, nullptr, d_records, nullptr, true, stream);
}

extern "C" int yf_pool_import_records(yf_pool* pool, int32_t n, const int32_t* d_pages, const void* d_records,
                                      const uint64_t* d_expect_hashes, const uint32_t* d_expect_tokens,
                                      uint32_t* d_ok, void* stream) {
    return launch_records(pool, n, d_pages, nullptr, nullptr, nullptr, nullptr,
                          reinterpret_cast<const unsigned long long*>(d_expect_hashes), d_expect_tokens,
                          const_cast<void*>(d_records), d_ok, false, stream);
}
