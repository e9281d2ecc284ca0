/*
 * yfattn.h — C ABI of the B200 (sm_100a) paged Q8_0 KV attention library.
 *
 * This is the drop-in boundary for the attention path of the yforge engine
 * (askidmobile/qwen36-server) over its persistent paged int8 KV pool
 * (`--kv-pool q8`, src/cli.rs:111-115,286-290).  The engine's Rust side calls
 * the functions below through `extern "C"` with raw device pointers, the way
 * its own `real::paged_attn` call takes raw pool pointers instead of candle
 * tensors (docs/plans/2026-08-24-qwen35-4b-benchmark.md:600-607).
 *
 * Conventions
 *  - Every pointer argument named d_* is device memory of the pool's device.
 *    Host arrays are named h_*.
 *  - The caller owns every buffer passed in.  Calls on the hot path never
 *    allocate; the split-KV workspace size comes from yf_attn_workspace_size.
 *  - Every call is asynchronous on the given CUDA stream (cudaStream_t passed
 *    as void*; NULL is the legacy default stream).
 *  - The return value is YF_OK or a YF_E_* code from host-side validation.
 *    yf_last_error() gives a message for the last failure on this thread.
 *  - Values that only the device knows (page ids in the block table, sequence
 *    lengths) are checked inside the kernels: an out-of-range page or length
 *    is skipped and recorded in the pool's device status word, never trapped.
 *    yf_pool_status() reads and optionally clears that word.
 *  - Distinct pools may be used from distinct threads; one pool is not
 *    internally locked (the engine drives it from one thread).
 *
 * KV pool format ("Q8_0 pages")
 *  - One pool holds n_layers planes.  A page is page_size tokens of every KV
 *    head; pages are shared by all layers (page p of layer l and layer l+1
 *    belong to the same token range), as with the engine's block tables.
 *  - A value group of group_size consecutive head_dim elements (32 = GGML
 *    Q8_0, or head_dim = the engine's own one-scale-per-row int8 pool) is
 *    stored as int8 q and one f16 scale d, value = q * d.  Quantization is
 *    GGML's Q8_0 rule: d = amax/127, q = roundf(x * (1/d)), d stored as f16.
 *    Each q is held as the excess-128 byte q + 128 (its top bit flipped), the
 *    form the kernels turn into f16 with one byte permute.
 *  - Within a layer plane, page p / kv head h is one contiguous block of
 *    page_size/16 "tiles" of 16 tokens.  A tile is
 *        [K int8 16*D][K scales f16 16*(D/G)][V int8 16*D][V scales f16 16*(D/G)]
 *    with the int8 and scale bytes permuted inside the tile so that one
 *    16-byte load per lane delivers tensor-core fragments directly.
 *    yf_pool_tile_offset() states the permutation for any (token, dim).
 */
#ifndef YFATTN_H
#define YFATTN_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define YF_API __attribute__((visibility("default")))
#else
#define YF_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define YFATTN_ABI_VERSION 2

/* Return codes of every entry point. */
#define YF_OK 0
#define YF_E_INVALID 1     /* bad argument: null pointer, negative size, bad alignment */
#define YF_E_UNSUPPORTED 2 /* shape not built (head_dim, page_size, group size, GQA ratio) */
#define YF_E_NOMEM 3       /* device allocation or page allocation failed */
#define YF_E_CUDA 4        /* a CUDA runtime call failed */
#define YF_E_RANGE 5       /* length, layer or page id beyond the pool's capacity */
#define YF_E_WORKSPACE 6   /* workspace smaller than yf_attn_workspace_size */
#define YF_E_STATE 7       /* page allocator misuse: double free, free of a free page */

/* Bits of the pool's device status word (set by kernels, read by yf_pool_status). */
#define YF_DEV_BAD_PAGE 1u     /* a block-table entry was >= n_pages: that page was skipped */
#define YF_DEV_LEN_OVERFLOW 2u /* a sequence length exceeded max_blocks*page_size: clamped */
#define YF_DEV_BAD_POS 4u      /* a KV write position was outside the block table: row skipped */
#define YF_DEV_BAD_ROWS 8u     /* a query-row count exceeded max_seqlen_q (or its keys): rows clamped */
#define YF_DEV_TIMEOUT 16u     /* a bounded wait on a page copy gave up: output of that CTA invalid */
#define YF_DEV_SMEM_ALIGN 32u  /* a kernel found its shared memory misaligned and wrote nothing */
/* With YF_DEV_TIMEOUT set, bits 16-31 of the status word hold a diagnostic tag of the first
 * wait that gave up (kernel-specific: role, barrier, awaited completion). */

typedef struct yf_pool yf_pool;

typedef struct yf_pool_desc {
    int32_t n_layers;   /* layer planes in the pool (>= 1) */
    int32_t n_pages;    /* physical pages per layer plane */
    int32_t n_kv_heads; /* KV heads (Hkv) */
    int32_t head_dim;   /* D: 128 or 256 */
    int32_t page_size;  /* tokens per page: 16 or 64 */
    int32_t group_size; /* quant group along head_dim: 32 (Q8_0) or head_dim (row scale) */
    int32_t device;     /* CUDA device ordinal that owns the pool; < 0 = host-only pool */
    int32_t reserved;
    void* device_mem;   /* optional caller-owned buffer of yf_pool_bytes(desc) bytes, or NULL */
} yf_pool_desc;

/* Thread-local message for the last non-YF_OK return on this thread. */
YF_API const char* yf_last_error(void);
YF_API int yf_abi_version(void);

/* ---- pool: layout and lifetime --------------------------------------------
 * Replaces the engine's PagedKvPool {k, v, k_scale, v_scale}
 * (docs/plans/2026-08-27-tiered-kv-cache.md:352-353) whose size follows
 * src/vram_plan.rs:249-261. */

/* Bytes of one (page, kv head) block and of the whole pool. */
YF_API size_t yf_pool_page_head_bytes(const yf_pool_desc* desc);
YF_API size_t yf_pool_bytes(const yf_pool_desc* desc);
/* Byte offset inside a 16-token tile of the value byte (q + 128) of (token t in 0..15,
 * dim d) for K (is_v=0) or V (is_v=1); the f16 scale offset of (t, group) is
 * returned by yf_pool_scale_offset.  Pure functions of the format. */
YF_API int64_t yf_pool_tile_offset(const yf_pool_desc* desc, int is_v, int t, int d);
YF_API int64_t yf_pool_scale_offset(const yf_pool_desc* desc, int is_v, int t, int group);

/* Creates a pool; allocates device memory unless desc->device_mem is given.
 * The memory is zero-filled.  All pages start free with refcount 0.
 * desc->device < 0 makes a host-only pool: the page allocator alone, with no
 * device memory (every device call on it returns YF_E_INVALID). */
YF_API int yf_pool_create(const yf_pool_desc* desc, yf_pool** out_pool);
YF_API int yf_pool_destroy(yf_pool* pool);
YF_API int yf_pool_get_desc(const yf_pool* pool, yf_pool_desc* out_desc);
/* Device address of a layer plane (for export by the caller, debugging). */
YF_API int yf_pool_layer_ptr(const yf_pool* pool, int32_t layer, void** out_ptr);

/* ---- pool: page allocator (host side) --------------------------------------
 * The engine builds static tables bt[slot*max_blocks+j] = slot*max_blocks+j
 * (docs/plans/2026-08-27-tiered-kv-cache.md:52-58); this allocator replaces
 * that arithmetic with a free list plus refcounts so that pages can be
 * fragmented and shared between slots. */

/* Takes n pages off the free list (refcount 1 each) into h_pages_out.
 * YF_E_NOMEM (and nothing taken) when fewer than n pages are free. */
YF_API int yf_pool_alloc_pages(yf_pool* pool, int32_t n, int32_t* h_pages_out);
/* Adds one reference to each listed page (prefix sharing). */
YF_API int yf_pool_retain_pages(yf_pool* pool, int32_t n, const int32_t* h_pages);
/* Drops one reference; a page whose count reaches 0 returns to the free list.
 * YF_E_STATE if a listed page is already free (nothing is changed then). */
YF_API int yf_pool_free_pages(yf_pool* pool, int32_t n, const int32_t* h_pages);
YF_API int yf_pool_free_count(const yf_pool* pool, int32_t* out_free);
YF_API int yf_pool_refcount(const yf_pool* pool, int32_t page, int32_t* out_refcount);

/* Reads the device status word (synchronizes the pool's device) into
 * *out_bits; clears it when clear != 0.  Clearing a word that holds
 * YF_DEV_TIMEOUT also resets the pool's merge arrival counters (a wait that
 * gave up leaves them mid-count), so the pool is usable again; a pool whose
 * status shows YF_DEV_TIMEOUT must be cleared this way before its next call. */
YF_API int yf_pool_status(yf_pool* pool, uint32_t* out_bits, int clear);

/* ---- pool: attention options ---------------------------------------------------
 * Explicit per-pool choices that every attention call on the pool, and
 * yf_attn_workspace_size, read (the library reads no environment variables).
 * A zero-filled struct is the default.  The engine's counterpart is its
 * command-line / config flags (src/cli.rs), fixed for the life of the pool. */
#define YF_SCHED_AUTO 0        /* cluster schedule for a few long units, persistent for many, else chunked */
#define YF_SCHED_CHUNKED 1     /* always the chunked (unit x chunk grid) split-KV schedule */
#define YF_SCHED_PERSISTENT 2  /* the persistent schedule wherever it applies (no cluster schedule) */
#define YF_MERGE_IN_KERNEL 0   /* split partials merged inside the attention kernel */
#define YF_MERGE_SEPARATE 1    /* chunked schedule: a separate combine launch merges the partials */
#define YF_PREFILL_AUTO 0      /* tcgen05 prefill kernel where it applies (>= 128 rows per kv head) */
#define YF_PREFILL_SPLITKV 1   /* every query block on the split-KV kernel */
#define YF_VERIFY_AUTO 0       /* verify blocks on the split-KV kernel (measured faster at <= 32 rows per kv head) */
#define YF_VERIFY_TCGEN05 1    /* verify blocks of 2..32 rows per kv head (D 128, groups of 32) on the tcgen05 kernel */
/* The persistent decode's CTAs wait for one another's split partials, so all of them must be
 * resident at once.  Its grid never exceeds one resident wave, so against other kernels that
 * finish by themselves (other streams, other pools) a plain launch completes; only kernels that
 * hold SMs indefinitely (another process's persistent kernel under MPS) can starve it, and then
 * its bounded waits flag YF_DEV_TIMEOUT.  A cooperative launch rules that out at launch time and
 * costs 2-3 us per call (measured on B200). */
#define YF_LAUNCH_PLAIN 0        /* plain launch (default) */
#define YF_LAUNCH_COOPERATIVE 1  /* cooperative launch: co-residency guaranteed by the launch */
typedef struct yf_attn_options {
    int32_t schedule;        /* YF_SCHED_* */
    int32_t chunk_tiles;     /* chunked schedule: 16-token tiles per CTA; 0 = sized from the grid */
    int32_t copy_stages;     /* bulk-copy ring depth per warp: 0 = default (4 at D 128, 2 at D 256) or 3 */
    int32_t merge;           /* YF_MERGE_* */
    int32_t prefill_kernel;  /* YF_PREFILL_* */
    uint32_t wait_limit_us;  /* bound of every in-kernel wait (copies, merges); 0 = 1 000 000 (1 s) */
    int32_t launch;          /* YF_LAUNCH_*: how the persistent decode is launched */
    int32_t verify_kernel;   /* YF_VERIFY_* */
    int32_t reserved[8];     /* zero */
} yf_attn_options;
/* Replaces the pool's options (validated: YF_E_INVALID for an unknown value).  Not
 * stream-ordered: set them between calls, not while the pool's kernels run. */
YF_API int yf_pool_set_options(yf_pool* pool, const yf_attn_options* opts);
YF_API int yf_pool_get_options(const yf_pool* pool, yf_attn_options* out_opts);

/* Fault-injection hook for testing the bounded waits (no counterpart in the reference):
 * writes `value` into the pool's merge arrival counter `index` (stream-ordered).  A value of
 * 0xFFFF makes the next merge of that unit wait for parts that never arrive, so the wait runs
 * out after wait_limit_us and flags YF_DEV_TIMEOUT; yf_pool_status(clear) then resets the
 * counters.  index < YF_POOL_COUNTERS. */
#define YF_POOL_COUNTERS (65536 + 4096)
YF_API int yf_pool_plant_counter(yf_pool* pool, int32_t index, uint32_t value, void* stream);

/* ---- KV write: Q8_0 quantize-and-scatter ------------------------------------
 * yf_kv_append_paged replaces kv_append_paged_f16 (fork quantized.cu:6996,
 * cited at docs/plans/2026-08-27-tiered-kv-cache.md:61-64): one new row per
 * batch entry.  d_k, d_v: f16 [B, Hkv, D] contiguous.  Row b is written at
 * token position d_pos[b] of batch entry b, i.e. page
 * d_block_table[b*max_blocks + pos/page_size], slot pos%page_size.
 * A position outside the table is skipped and flags YF_DEV_BAD_POS (the
 * engine instead clamped to window-1 and overwrote the last slot). */
YF_API int yf_kv_append_paged(yf_pool* pool, int32_t layer, const void* d_k, const void* d_v,
                              const int32_t* d_pos, const uint32_t* d_block_table, int32_t max_blocks,
                              int32_t batch, void* stream);

/* Replaces launch_append_multi (fork quantized.cu:7040, called from
 * forward_attn_prefill_paged: docs/plans/2026-08-27-mtp-cuda-graphs.md:132-134):
 * T contiguous rows per batch entry.  d_k, d_v: f16 [total_rows, Hkv, D];
 * rows d_cu_rows[b] .. d_cu_rows[b+1]-1 belong to entry b and go to positions
 * d_start_pos[b] + i.  max_rows bounds d_cu_rows[b+1]-d_cu_rows[b]. */
YF_API int yf_kv_append_paged_multi(yf_pool* pool, int32_t layer, const void* d_k, const void* d_v,
                                    const int32_t* d_cu_rows, const int32_t* d_start_pos,
                                    const uint32_t* d_block_table, int32_t max_blocks, int32_t batch,
                                    int32_t max_rows, void* stream);

/* Fused attention prep + KV append: replaces attn_prepare_decode (RMSNorm of q
 * and k with their own weights, partial RoPE, the gate half of the q projection
 * split out; docs/research/2026-09-16-head-to-head-llamacpp-and-phase-profile.md:181-216)
 * followed by yf_kv_append_paged_multi, in one launch.  Rows as in
 * yf_kv_append_paged_multi (entry b: rows d_cu_rows[b].., positions
 * d_start_pos[b] + i, which are also the RoPE positions).
 * d_qg: f16 [total_rows, Hq, 2*D], per head the q half then the gate half;
 * d_k, d_v: f16 [total_rows, Hkv, D]; d_q_norm_w, d_k_norm_w: f32 [D].
 * q, k: y = x / sqrt(mean(x^2) + eps) * (w + norm_weight_offset) (offset 1 for
 * zero-centred weights), then on dims [0, rope_dim) the rotate-half RoPE
 * y'[i] = y[i] c - y[i+h] s, y'[i+h] = y[i+h] c + y[i] s, h = rope_dim/2,
 * c = d_rope_cos[pos*h + i], s = d_rope_sin[pos*h + i] (f32 [rope_rows, h]).
 * Outputs: d_q_out f16 [total_rows, Hq, D] (normed, rotated q), d_gate_out f16
 * [total_rows, Hq, D] (the gate half as given); K (normed, rotated, rounded to
 * f16) and V are quantized into the pool exactly as yf_kv_append_paged_multi
 * would from those f16 rows.  Every float step is an IEEE round-to-nearest
 * operation in a fixed order (the sum of squares per lane in dim order, then an
 * xor butterfly over the 32 lanes of D/32 dims each, offsets 16..1).
 * rope_dim: 0, or 2*(D/32)*2^k <= D.  Pointers 16-byte aligned.  A position
 * outside [0, rope_rows) or the block table flags YF_DEV_BAD_POS and skips the row. */
YF_API int yf_attn_prepare_append(yf_pool* pool, int32_t layer, int32_t n_q_heads, const void* d_qg,
                                  const void* d_k, const void* d_v, const float* d_q_norm_w,
                                  const float* d_k_norm_w, float eps, int32_t norm_weight_offset,
                                  const float* d_rope_cos, const float* d_rope_sin, int32_t rope_dim,
                                  int32_t rope_rows, const int32_t* d_cu_rows, const int32_t* d_start_pos,
                                  const uint32_t* d_block_table, int32_t max_blocks, int32_t batch,
                                  int32_t max_rows, void* d_q_out, void* d_gate_out, void* stream);

/* ---- attention ---------------------------------------------------------------
 * Split-KV workspace for a call with these shapes (0 is a valid answer). */
YF_API size_t yf_attn_workspace_size(const yf_pool* pool, int32_t n_q_heads, int32_t batch,
                                     int32_t max_seqlen_q, int32_t max_seqlen_k);

/* Batched decode: replaces dispatch_flash_decode_paged(cuda, q, k, v, lens,
 * table, scale) (src/bin/decode_gqa_probe.rs:26,40-46) and the q8 decode
 * branch of real::paged_attn.  d_q: f16 [B, Hq, D]; d_cu_seqlens_k: uint32
 * [B+1] (entry b has d_cu_seqlens_k[b+1]-d_cu_seqlens_k[b] keys, as the probe's
 * `lens`); d_block_table: uint32 [B, max_blocks]; d_out: f16 [B, Hq, D].
 * max_seqlen_k bounds every entry's length (it sizes the split grid).
 * An entry with zero keys produces zeros. */
YF_API int yf_attn_decode(yf_pool* pool, int32_t layer, const void* d_q, int32_t n_q_heads,
                          const uint32_t* d_cu_seqlens_k, const uint32_t* d_block_table,
                          int32_t max_blocks, int32_t batch, int32_t max_seqlen_k, float scale,
                          void* d_out, void* d_workspace, size_t workspace_bytes, void* stream);

/* yf_attn_decode without a workspace argument, for callers that cannot
 * allocate device memory: their memory is planned once at start-up and handed
 * out by an allocator they cannot reach from the FFI layer, so a cudaMalloc
 * of their own would break that budget and may fail mid-request.  No
 * counterpart in the reference.  The split-KV partials go to a 16 MiB array
 * built into the library (held by every GPU that loads it, until exit); a
 * call whose yf_attn_workspace_size exceeds 16 MiB returns YF_E_WORKSPACE.
 * The first call on a device looks up that array's device address, so make
 * it before any stream capture.  All calls share the array: calls whose
 * kernels overlap on the GPU race and must be serialised by the caller.
 * Allocates nothing. */
YF_API int yf_attn_decode_noalloc(yf_pool* pool, int32_t layer, const void* d_q, int32_t n_q_heads,
                                  const uint32_t* d_cu_seqlens_k, const uint32_t* d_block_table,
                                  int32_t max_blocks, int32_t batch, int32_t max_seqlen_k, float scale,
                                  void* d_out, void* stream);

/* Causal chunked prefill and MTP verify: replaces forward_attn_prefill_paged
 * (docs/plans/2026-08-27-mtp-cuda-graphs.md:132,244-248) and
 * forward_verify_paged (:279-284, per_row_gqa at :537-541).
 * d_q: f16 [total_q, Hq, D]; entry b owns query rows d_cu_seqlens_q[b] ..
 * d_cu_seqlens_q[b+1]-1 and Tk_b = d_cu_seqlens_k[b+1]-d_cu_seqlens_k[b]
 * keys already in the pool (prefix plus the new rows).  Query row i of entry
 * b sees keys 0 .. Tk_b - Tq_b + i ("row i sees 0..kv0+i").
 * d_out: f16 [total_q, Hq, D]. */
YF_API int yf_attn_prefill(yf_pool* pool, int32_t layer, const void* d_q, int32_t n_q_heads,
                           const uint32_t* d_cu_seqlens_q, const uint32_t* d_cu_seqlens_k,
                           const uint32_t* d_block_table, int32_t max_blocks, int32_t batch,
                           int32_t max_seqlen_q, int32_t max_seqlen_k, float scale, void* d_out,
                           void* d_workspace, size_t workspace_bytes, void* stream);

/* Tree speculative verify: replaces forward_verify_tree_graphed with its
 * trie_ranges mask (docs/plans/2026-10-09-tree-speculative-decoding.md:26-38).
 * As yf_attn_prefill, but an entry's Tq_b <= 64 draft rows are the nodes of a
 * token trie in depth-first order: d_trie_ranges (int32 [total_q][2], 8-byte
 * aligned) holds for draft row j of an entry the inclusive range [start_j,
 * end_j] of its subtree, as node indices 0 .. Tq_b-1 of that entry.  Row i
 * sees the committed keys 0 .. Tk_b - Tq_b - 1 and draft key Tk_b - Tq_b + j
 * when j <= i and start_j <= i <= end_j (j is i or an ancestor of i).  A chain
 * (start_j = j, end_j = Tq_b - 1) gives yf_attn_prefill's causal rows.  A
 * range outside 0 .. Tq_b-1 is clamped and flags YF_DEV_BAD_ROWS.  Workspace:
 * yf_attn_workspace_size with the same arguments. */
YF_API int yf_attn_verify_tree(yf_pool* pool, int32_t layer, const void* d_q, int32_t n_q_heads,
                               const uint32_t* d_cu_seqlens_q, const uint32_t* d_cu_seqlens_k,
                               const uint32_t* d_block_table, int32_t max_blocks, int32_t batch,
                               int32_t max_seqlen_q, int32_t max_seqlen_k, float scale,
                               const int32_t* d_trie_ranges, void* d_out, void* d_workspace,
                               size_t workspace_bytes, void* stream);

/* Sharded decode, first half: yf_attn_decode over the keys this pool holds
 * (one shard of each sequence and/or a subset of the kv heads), emitting
 * partials instead of f16 output: d_o_part f32 [B, Hq, D] is O normalised
 * over the shard's keys and d_lse_part f32 [B, Hq] is the natural-log
 * log-sum-exp of the shard's scaled logits (-inf, with O = 0, for a shard
 * without keys).  Replaces the partial (o, lse) output of the reference's
 * split-KV kernel that flash_fwd_splitkv_combine_kernel consumes
 * (docs/plans/2026-09-16-prefil-parity-fa2-and-mmq.md:104-107), with the
 * shards on different GPUs.  d_o_part and d_lse_part 16- and 4-byte aligned. */
YF_API int yf_attn_decode_partial(yf_pool* pool, int32_t layer, const void* d_q, int32_t n_q_heads,
                                  const uint32_t* d_cu_seqlens_k, const uint32_t* d_block_table,
                                  int32_t max_blocks, int32_t batch, int32_t max_seqlen_k, float scale,
                                  float* d_o_part, float* d_lse_part, void* d_workspace,
                                  size_t workspace_bytes, void* stream);

/* Sharded decode, second half: merges n_parts partials of `rows` rows into
 * d_out f16 [rows][head_dim].  Part k's O, f32 [rows][head_dim], starts at
 * d_o_parts + k * o_part_stride and its lse, f32 [rows], at d_lse_parts +
 * k * lse_part_stride (strides in floats), so partials packed per rank as
 * one all-gathered buffer are read in place.
 * out = sum_k exp(lse_k - M) o_k / sum_k exp(lse_k - M), M = max_k lse_k
 * (zeros where every lse is -inf).  The LSE merge of
 * flash_fwd_splitkv_combine_kernel (same citation), across GPUs.
 * head_dim a multiple of 4; every O part 16-byte aligned, d_out 8-byte. */
YF_API int yf_attn_combine(const float* d_o_parts, int64_t o_part_stride, const float* d_lse_parts,
                           int64_t lse_part_stride, int32_t n_parts, int32_t rows, int32_t head_dim, void* d_out,
                           void* stream);

/* ---- partial exchange over NVLink peer memory ---------------------------------
 * Replaces, for the kv-head x key-range sharded long decode, the all-gather of the packed
 * partials plus yf_attn_combine (both stand in for flash_fwd_splitkv_combine_kernel across
 * GPUs; same citation): every rank owns an exchange area in its own HBM that the other ranks
 * map once (CUDA IPC, plain peer mappings).  A step is yf_exchange_push (this rank's partial
 * stored into slot `rank` of every rank's area, then a release flag in each) followed, later
 * in the same stream, by yf_exchange_combine (a bounded acquire wait on every rank's flag in
 * the own area, then the LSE merge in place into f16 output).  The reference has no
 * counterpart: its decode runs on one GPU.  Each rank's partial is slot_floats f32, 16-byte
 * aligned: O f32 [rows][head_dim] at offset 0 and lse f32 [rows] at lse_offset.  A wait that
 * runs past the limit (default 1 s) writes nothing and sets YF_DEV_TIMEOUT in the exchange's
 * status. */
typedef struct yf_exchange yf_exchange;
#define YF_EXCHANGE_HANDLE_BYTES 64
YF_API int yf_exchange_create(int32_t device, int32_t rank, int32_t world, int64_t slot_floats,
                              yf_exchange** out);
YF_API int yf_exchange_destroy(yf_exchange* ex);
/* The IPC handle (YF_EXCHANGE_HANDLE_BYTES bytes) of this rank's area, to hand to the others. */
YF_API int yf_exchange_handle(const yf_exchange* ex, void* out_handle);
/* Maps rank `peer`'s area (its handle) into this process. */
YF_API int yf_exchange_open_peer(yf_exchange* ex, int32_t peer, const void* handle);
/* Same-process, same-device peer (tests that emulate ranks on one GPU). */
YF_API int yf_exchange_attach(yf_exchange* ex, int32_t peer, const yf_exchange* other);
/* 0 restores the default limit of one second. */
YF_API int yf_exchange_set_wait_limit(yf_exchange* ex, uint32_t wait_limit_us);
YF_API int yf_exchange_push(yf_exchange* ex, const float* d_partial, void* stream);
/* Ranks s * n_head_groups + g (s < n_seq) hold head group g's key ranges; row i = b * hq + j of
 * a partial is output row b * n_q_heads + g * hq + j, n_q_heads = hq * n_head_groups; d_out f16
 * [rows / hq][n_q_heads][head_dim], 8-byte aligned. */
YF_API int yf_exchange_combine(yf_exchange* ex, int32_t n_head_groups, int32_t n_seq, int32_t rows, int32_t hq,
                               int32_t n_q_heads, int32_t head_dim, int64_t lse_offset, void* d_out,
                               void* stream);
/* One whole step of the sharded decode in one launch where the cluster decode schedule takes it:
 * this rank's partial over its pool (as yf_attn_decode_partial; q [batch][hq][head_dim], the
 * workspace of yf_attn_workspace_size(pool, hq, batch, 1, max_seqlen_k)) is stored straight into
 * every rank's area as (value, step) words, and every CTA that stored a slice polls the same rows
 * of every rank's partial in its own area (bounded) and merges them into d_out (the arithmetic of
 * yf_exchange_combine; 16-byte aligned).  Other
 * schedules run decode_partial, push and combine (three launches, same result).  The slot must
 * hold batch * hq * (head_dim + 1) floats.  For ranks on separate devices: an exchange with
 * attached same-device peers returns YF_E_UNSUPPORTED (those ranks would wait on one another). */
YF_API int yf_exchange_decode(yf_exchange* ex, yf_pool* pool, int32_t layer, const void* d_q, int32_t hq,
                              const uint32_t* d_cu_k, const uint32_t* d_block_table, int32_t max_blocks,
                              int32_t batch, int32_t max_seqlen_k, float scale, int32_t n_head_groups, int32_t n_seq,
                              int32_t n_q_heads, void* d_out, void* d_workspace, size_t workspace_bytes,
                              void* stream);
/* Synchronizes the device, reads the status bits (YF_DEV_TIMEOUT) and clears them if asked. */
YF_API int yf_exchange_status(yf_exchange* ex, uint32_t* out_bits, int clear);

/* ---- prefix snapshot export / restore ----------------------------------------
 * Byte copies of whole pages (all KV heads, one layer) with their scales and
 * no requantization, as StateSnapshot::to_host / to_device do for the int8
 * pool (src/prefix_cache.rs:71-91 and :361; injected by inject_slot_snapshot,
 * src/engine_batched.rs:1724,1738).  The snapshot buffer holds the n pages
 * back to back, yf_pool_page_head_bytes * n_kv_heads bytes each; it may be
 * host (pinned or pageable) or device memory. */
YF_API int yf_pool_export_pages(yf_pool* pool, int32_t layer, int32_t n, const int32_t* h_pages,
                                void* dst, void* stream);
YF_API int yf_pool_restore_pages(yf_pool* pool, int32_t layer, int32_t n, const int32_t* h_pages,
                                 const void* src, void* stream);

/* ---- snapshot wire records ------------------------------------------------------
 * The prefix cache's page records (pages.kv, docs/plans/2026-08-27-tiered-kv-cache.md:141-145,
 * 237-251, whose page entry is { chain_hash, prev_hash, tokens[], payload }): one record per pool
 * page, back to back at a stride of yf_pool_record_bytes,
 *   [u64 chain_hash][u64 prev_hash][u32 page_index][u32 n_tokens][u32 payload_len][u32 crc32c]
 *   [u32 tokens[page_size]][payload]
 * little-endian, packed (32 + 4*page_size header bytes, a multiple of 16); n_tokens = page_size;
 * payload = the page in every layer, layer 0 first (n_layers * yf_pool_page_head_bytes *
 * n_kv_heads bytes); crc32c = CRC-32C (Castagnoli, reflected polynomial 0x82F63B78, preset and
 * final xor 0xFFFFFFFF) of the token ids followed by the payload.  The token ids let a reader
 * tell a chain-hash collision from a hit, as the prefix cache compares tokens before it uses a
 * cached page (src/prefix_cache.rs:347-356). */
#define YF_REC_REJECTED 0  /* corrupt: payload_len, n_tokens or CRC wrong, or a bad page id */
#define YF_REC_RESTORED 1  /* intact and (where expected values were given) the same prefix: restored */
#define YF_REC_MISMATCH 2  /* intact, but its chain hash or token ids differ from the expected ones */
YF_API size_t yf_pool_record_bytes(const yf_pool_desc* desc);
/* Builds n records in device memory d_records (16-byte aligned) from pool pages d_pages[i], with
 * the caller's d_chain_hashes[i] (the prefix chain fingerprint), d_prev_hashes[i] (the previous
 * page's chain hash), d_page_indices[i] (its position in the chain; null: the pool page id) and
 * d_tokens (u32 [n][page_size], the page's token ids); null hash or token arrays write zeros.
 * The CRC is computed in the same pass as the copy.  Device arrays; a page id outside the pool
 * flags YF_DEV_BAD_PAGE and writes a header with payload_len 0, which every import rejects. */
YF_API int yf_pool_export_records(yf_pool* pool, int32_t n, const int32_t* d_pages,
                                  const uint64_t* d_chain_hashes, const uint64_t* d_prev_hashes,
                                  const uint32_t* d_page_indices, const uint32_t* d_tokens, void* d_records,
                                  void* stream);
/* Checks n records in device memory (16-byte aligned): payload_len, n_tokens and the CRC-32C, and,
 * where given, that record i carries d_expect_hashes[i] and the token ids d_expect_tokens[i][*];
 * copies each intact, matching record into pool page d_pages[i] (every layer).  d_ok[i] = one of
 * YF_REC_*; a page not restored is left as it was (the caller then treats the context as a
 * prefill, as the reference does with a record it cannot use). */
YF_API int yf_pool_import_records(yf_pool* pool, int32_t n, const int32_t* d_pages, const void* d_records,
                                  const uint64_t* d_expect_hashes, const uint32_t* d_expect_tokens,
                                  uint32_t* d_ok, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* YFATTN_H */
