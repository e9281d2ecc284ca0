// Internal declarations shared by the library's translation units.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <vector>

#include "yfattn.h"

namespace yf {

// Tokens per tile: the unit one warp consumes per pipeline step.
constexpr int kTileTokens = 16;
// Units (entry x kv head x row group) whose split-KV partials the attention kernel can merge
// itself; the pool keeps one arrival counter per unit.
constexpr int kMaxCombineUnits = 1 << 16;
// Counters of the first merge level of the persistent decode (groups of pieces of one unit),
// indexed by the group's first partial slot; they follow the per-unit counters.
constexpr int kMaxGroupCounters = 4096;
// Largest batch the persistent decode schedule handles (its tile prefix lives in shared memory).
constexpr int kPersistentMaxBatch = 1024;
// Upper bound of resident split-KV CTAs per SM (sizes the persistent schedule's workspace).
constexpr int kMaxCtasPerSm = 4;
// CTAs per thread-block cluster of the few-long-units decode schedule, and the most units it takes.
constexpr int kClusterCtas = 8;
constexpr int kClusterMaxUnits = 32;
// Dynamic shared memory floor of that schedule's CTAs: above a third of an SM's 228 KB, so no SM
// hosts three of them while others host one (CTAs of equal work then stream at equal rates).
constexpr int kClusterSmemFloor = 80 * 1024;
// Most cluster partials of one unit (sizes the last merge's weight table in shared memory).
constexpr int kClusterMaxParts = 256;

// Byte offsets of the four areas of a 16-token tile (see yf_pool_tile_offset).
struct TileGeom {
    int D;       // head_dim
    int NB;      // scale groups per row (D / group_size)
    int tile;    // whole tile
    int ks_off;  // K scales
    int v_off;   // V values
    int vs_off;  // V scales
};

inline TileGeom tile_geom(int D, int NB) {
    TileGeom g;
    g.D = D;
    g.NB = NB;
    g.ks_off = 16 * D;
    g.v_off = 16 * D + 32 * NB;
    g.vs_off = 32 * D + 32 * NB;
    g.tile = 32 * D + 64 * NB;
    return g;
}

}  // namespace yf

struct yf_pool {
    yf_pool_desc desc;
    uint8_t* base = nullptr;  // device: [n_layers][n_pages][n_kv_heads][page_head_bytes]
    bool owns_mem = false;
    size_t bytes = 0;
    size_t tile_bytes = 0;
    size_t page_head_bytes = 0;
    size_t page_bytes = 0;   // all kv heads of one page in one layer
    size_t layer_bytes = 0;
    uint32_t* d_status = nullptr;  // device status word (YF_DEV_* bits)
    uint32_t* d_counters = nullptr;  // kMaxCombineUnits + kMaxGroupCounters arrival counters, zero between calls
    int sm_count = 148;
    std::vector<int32_t> refcount;
    std::vector<int32_t> free_stack;  // LIFO of free page ids
    // CRC-32C combine operators of this pool's snapshot records (computed when the pool is created)
    std::vector<uint32_t> crc_ops;
    // attention choices every call and the workspace query read (yf_pool_set_options)
    yf_attn_options opts{};
};

namespace yf {

// Records a message for yf_last_error() and returns code.
int fail(int code, const char* fmt, ...);
// Maps a CUDA error to YF_E_CUDA with the call site in the message.
int cuda_fail(cudaError_t e, const char* what);

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Bound of every in-kernel wait of this pool's calls, in nanoseconds.
inline uint64_t wait_limit_ns(const yf_pool* pool) {
    return (uint64_t)(pool->opts.wait_limit_us ? pool->opts.wait_limit_us : 1000000u) * 1000ull;
}

// Per-device launch facts cached behind a mutex (any host thread may launch): the dynamic
// shared memory a kernel was raised to, and the resident CTAs per SM at one size.
struct LaunchCache {
    int smem_set[64] = {};
    int occ_smem[64] = {};
    int occ_val[64] = {};
};
// Raises `kern`'s dynamic shared-memory limit to `smem` once per device.
int raise_smem_attr(const void* kern, int smem, int dev, LaunchCache& c);
// Resident CTAs per SM of `kern` at `threads` x `smem` (cached per device for the last size).
int occupancy(const void* kern, int threads, int smem, int dev, LaunchCache& c, int* out);

// Split-KV plan of one attention call; identical in the workspace query and
// the launch so that the caller's workspace always fits.
struct SplitPlan {
    int rows_per_cta;  // query rows (q heads x query positions) of one CTA: 8 or 16
    int n_row_groups;  // ceil(G * max_seqlen_q / rows_per_cta)
    int chunk_tiles;   // 16-token tiles per CTA
    int max_chunks;    // ceil(max tiles / chunk_tiles)
    int stages;        // bulk-copy stages per warp
    bool fused_combine;  // the last CTA of a unit merges its partials (no combine launch)
    bool persistent;     // decode_persistent_kernel: equal (unit, tile) ranges per CTA
    bool cluster;        // decode_cluster_kernel: max_chunks clusters of chunk_tiles tiles per unit
    int persistent_ctas;  // upper bound of its grid (the launch also caps it by occupancy)
    size_t ws_bytes;   // partial O + lse
};

SplitPlan plan_split(const yf_pool* pool, int n_q_heads, int batch, int max_seqlen_q, int max_seqlen_k,
                     bool tree = false);
// draft rows per entry of a tree verify (a 64-bit ancestor mask per row in the kernel)
constexpr int kMaxTreeRowsHost = 64;

// The exchange of a sharded decode's partial, fused into the cluster decode kernel
// (yf_exchange_decode): every CTA that finishes an output slice of this rank's partial stores it
// as 64-bit (value, step) words into slot `rank` of word buffer step & 1 in every rank's area,
// then polls the same rows of every rank's slot in its own area and merges them into f16 `out`.
// Shared-memory floats are not needed; the bounds below keep the per-thread state small.
constexpr int kXMaxSlices = 256;  // output slices of one call (units x cluster CTAs)
constexpr int kXMaxSeq = 8;       // key ranges merged per head group
struct XFuse {
    const unsigned long long* peers = nullptr;  // device array: every rank's area base (null: off)
    uint8_t* local = nullptr;                   // this rank's area
    int rank = 0, world = 1;
    long long slot_floats = 0;  // words per rank slot (the float slot's layout)
    long long lse_off = 0;      // words: the lse rows inside a slot
    size_t flags_off = 0;       // bytes: the meta words (status at world + 1)
    size_t sstep_off = 0;       // bytes: u32 [kXMaxSlices] step count of every output slice
    size_t words_off = 0;       // bytes: u64 [2][world][slot_floats] word buffers
    int n_hg = 1, n_seq = 1, hq = 1, n_q_heads = 1, rows = 1;
    __half* out = nullptr;  // f16 [rows / hq][n_q_heads][head_dim]
    uint64_t wait_ns = 0;
};

struct AttnArgs {
    const yf_pool* pool;
    int layer;
    const __half* q;
    int n_q_heads;
    const uint32_t* cu_q;  // nullptr for decode (entry b owns query row b)
    const uint32_t* cu_k;
    const uint32_t* block_table;
    int max_blocks;
    int batch;
    int max_seqlen_q;
    int max_seqlen_k;
    float scale;
    __half* out;
    void* workspace;
    size_t workspace_bytes;
    cudaStream_t stream;
    // partial output instead of `out`: normalised f32 O in out's layout and the natural-log
    // sum of exp(scaled logits) per (row, q head), for a later yf_attn_combine
    float* part_o = nullptr;
    float* part_lse = nullptr;
    // tree verify: int32 [total_q][2] inclusive subtree range of every draft row, or null
    const int32_t* trie = nullptr;
    // fused partial exchange (cluster schedule only), or null
    const XFuse* xf = nullptr;
};

// Programmatic stream serialization: the kernel may be scheduled while the previous kernel of
// its stream runs (it calls pdl_wait before touching global memory).
inline void pdl_attr(cudaLaunchAttribute& a) {
    a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    a.val.programmaticStreamSerializationAllowed = 1;
}

// Split-KV attention for decode / verify / small query blocks (yf_decode.cu).
int launch_splitkv(const AttnArgs& a, const SplitPlan& plan);
// A sharded decode's partial with the exchange fused in (yf_pool.cu): *fused = false and nothing
// launched when the cluster schedule does not take this call.
int decode_exchange(yf_pool* pool, int32_t layer, const void* q, int32_t hq, const uint32_t* cu_k, const uint32_t* bt,
                    int32_t max_blocks, int32_t batch, int32_t max_k, float scale, const XFuse& xf, void* ws,
                    size_t ws_bytes, void* stream, bool* fused);
// Clusters of the few-long-units decode kernel that fit on the pool's device at once (one wave),
// for a ring of `stages` copy stages (cached per device; an estimate for a host-only pool).
int cluster_capacity(const yf_pool* pool, int stages);

// Snapshot records: the CRC combine operators of the pool's record shape (yf_snapshot.cu).
void init_record_ops(yf_pool* pool);

// Tensor-core (tcgen05) MTP / tree verify for query blocks of 2..32 rows per kv head
// (yf_verify_tc.cu): keys as the MMA's M, split over CTAs in chunks of key tiles.
struct VerifyPlan {
    int rows;          // N of the MMAs: 16 or 32 query rows per unit
    int chunk_tiles;   // 128-key tiles per CTA
    int max_chunks;
    size_t ws_bytes;   // chunk partials (O + lse), 0 with one chunk per unit
};
bool verify_tc_applies(const yf_pool* pool, int n_q_heads, int max_seqlen_q, bool tree);
VerifyPlan plan_verify(const yf_pool* pool, int n_q_heads, int batch, int max_seqlen_q, int max_seqlen_k);
int launch_verify_tc(const AttnArgs& a, const VerifyPlan& plan);

// Tensor-core (tcgen05) causal prefill for query blocks of >= 128 rows per kv head
// (yf_prefill_tc.cu); needs no workspace.
bool prefill_tc_applies(const yf_pool* pool, int n_q_heads, int max_seqlen_q);
int launch_prefill_tc(const AttnArgs& a);
// The D=256 tcgen05 prefill (yf_prefill_tc256.cu).
bool prefill_tc256_applies(const yf_pool* pool, int n_q_heads, int max_seqlen_q);
int launch_prefill_tc256(const AttnArgs& a);

}  // namespace yf
