// MTP and tree speculative verify on the 5th-generation tensor cores (tcgen05, TMEM accumulators).
//
// Replaces the verify branch of the engine's FA2 split-KV call (forward_verify_paged /
// forward_verify_tree_graphed with per_row_gqa, docs/plans/2026-08-27-mtp-cuda-graphs.md:279-284,
// 537-541; docs/plans/2026-10-09-tree-speculative-decoding.md:26-38): the R = G x Tq query rows
// of one (entry, kv head) -- the G q heads of the kv head times the entry's draft rows -- attend
// to the entry's keys, draft row i seeing keys 0 .. Tk - Tq + i (or, for a tree, the committed
// keys and the draft keys of its ancestors).
//
// A unit (entry, kv head) has R <= 32 rows, too few for the M >= 64 of a tensor-core MMA, so the
// keys are M: per key tile of 128 keys,
//   S^T = K Q^T          tcgen05.mma kind::f16, A = K (128 keys x 128 dims, shared memory,
//                        K-major, 128-byte swizzle), B = Q (N rows x 128 dims), f32 in TMEM:
//                        TMEM lane = key, column = query row (N = 16 or 32);
//   P^T                  softmax thread = key (TMEM lane) over its N row values; the row maxima
//                        are kept per row and moved only when a tile's value exceeds them by 2^8
//                        (one CTA vote per tile decides); P^T is written as f16 into shared
//                        memory (B operand: N rows x 128 keys);
//   O^T += V^T P^T       tcgen05.mma, A = V^T (128 dims x 128 keys), B = P^T, f32 in TMEM:
//                        lane = dim, column = query row.
// S is double-buffered (TMEM columns [0, N) and [N, 2N)), so QK of tile j+1 runs while the
// softmax of tile j works; O is columns [2N, 3N).  The unit's key tiles are split into chunks of
// chunk_tiles, one CTA each; a chunk writes a normalised partial and the unit's last chunk to
// arrive merges them (an arrival counter per unit in the pool).
//
// Warp roles (10 warps), handing buffers to each other through mbarriers, every wait bounded:
//   warps 0-3 softmax (thread = key = TMEM lane; at the end thread = dim for O),
//   warps 4-7 dequant of the pool tiles into f16 K [key][dim] and V^T [dim][key],
//   warp 8 control (one lane issues every MMA and commit, polling its barriers),
//   warp 9 copies (one lane: bulk copies of the eight 16-token pool tiles of a key tile).
#include <cstdint>

#include "yf_device.cuh"
#include "yf_internal.h"
#include "yf_tc.cuh"

namespace yf {
namespace {

constexpr int kVtKeys = 128;                 // keys per key tile
constexpr int kVtD = 128;                    // head dim
constexpr int kVtPoolTiles = kVtKeys / 16;   // 16-token pool tiles per key tile
constexpr int kVtRawTile = 4352;             // one pool tile (D 128, Q8_0 groups of 32)
constexpr int kVtRawPitch = 4368;            // staged 16 B apart modulo 128 B: spreads banks
constexpr int kVtWarps = 10;
constexpr int kVtBlock = kVtWarps * 32;
constexpr int kVtCtl = 8, kVtCopy = 9;
constexpr float kVtRescale = 8.0f;           // lazy rescale threshold (base 2)
constexpr int kVtMaxTree = 64;               // draft rows of a tree entry (64-bit ancestor masks)
constexpr int kVtMaxChunkTiles = 64;         // key tiles of one CTA (its page ids live in shared memory)

// Shared-memory map (bytes from a 1024-aligned base) for N query rows per unit.
template <int N>
struct VtMap {
    static constexpr int Q = 0;                                 // [N rows][128 dims] SW128
    static constexpr int K = 8192;                              // [2 stages][128 keys][128 dims]
    static constexpr int VT = K + 2 * 32768;                    // [2 stages][128 dims][128 keys]
    static constexpr int P = VT + 2 * 32768;                    // [2 buffers][N rows][128 keys]
    static constexpr int RAW = P + 2 * N * 256;                 // [2 stages][8 pool tiles]
    static constexpr int MISC = RAW + 2 * kVtPoolTiles * kVtRawPitch;
    static constexpr int ANC = MISC + 512;                      // [64] ancestor masks (tree)
    static constexpr int RED = ANC + kVtMaxTree * 8;            // [4 warps][N] row scratch
    static constexpr int PGS = RED + 4 * N * 4;                 // [64 key tiles x 8] page ids of the chunk
    static constexpr int ALLOC = PGS + kVtMaxChunkTiles * kVtPoolTiles * 4;
    static_assert(ALLOC <= 232448, "shared memory");
};

struct VtBars {
    uint64_t raw_full[2], raw_free[2];  // pool tiles of a key tile staged / released
    uint64_t k_full[2], k_free[2];      // K stage written by the dequant warps / read by its QK
    uint64_t v_full[2], v_free[2];      // V^T stage written / read by its PV
    uint64_t s_full[2], s_free[2];      // S buffer written by QK / read by the softmax
    uint64_t p_full[2], p_free[2];      // P buffer written by the softmax / read by PV (and O updated)
    uint64_t o_done, drain;
};
static_assert(sizeof(VtBars) <= 256, "barrier area");

struct VerifyParams {
    const uint8_t* layer_base;
    int n_pages;
    int H;
    int G;
    int Hq;
    long long phb;
    int tpp;                 // 16-token tiles per page
    const __half* q;
    const uint32_t* cu_q;
    const uint32_t* cu_k;
    const uint32_t* bt;
    int max_blocks;
    int max_seqlen_q;
    int chunk_tiles;         // key tiles (128 keys) per CTA
    int max_chunks;
    float scale_log2;
    __half* out;
    float* ws_o;             // [units * max_chunks][N][128] normalised partial O
    float* ws_lse;           // [units * max_chunks][N] base-2 lse
    uint32_t* counters;      // per-unit arrival counters
    uint32_t* status;
    const int2* trie;        // tree verify: inclusive subtree range of every draft row, or null
    uint64_t wait_ns;
};

__device__ __forceinline__ void vt_give_up(volatile int* abort, uint32_t* status) {
    *abort = 1;
    atomicOr(status, YF_DEV_TIMEOUT);
}

// Bounded wait for the use-th completion (0-based) of `bar`; gives up on the CTA's abort flag.
__device__ __forceinline__ bool vt_wait(uint64_t* bar, int use, volatile int* abort, uint32_t* status,
                                       uint64_t limit_ns) {
    if (*abort) return false;
    if (mbar_try_wait(bar, (uint32_t)use & 1u)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, (uint32_t)use & 1u)) return true;
        if ((i & 7u) == 0) {
            if (*abort) return false;
            if (globaltimer_ns() - t0 > limit_ns) break;
        }
    }
    vt_give_up(abort, status);
    return false;
}

// OR of `pred` over the 128 softmax threads (named barrier 1).
__device__ __forceinline__ bool softmax_any(bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\tbar.red.or.pred po, 1, 128, pi;\n\t"
        "selp.u32 %0, 1, 0, po;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)pred)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ void softmax_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
__device__ __forceinline__ void dequant_sync() { asm volatile("bar.sync 2, 128;" ::: "memory"); }

// Per-row reduction over the 128 softmax threads: max (kMax) or sum of v[r]; every thread gets
// the N results.
template <int N, bool kMax>
__device__ __forceinline__ void rows_reduce(float (&v)[N], float* red, int warp, int lane) {
#pragma unroll
    for (int r = 0; r < N; ++r) {
        float x = v[r];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float y = __shfl_xor_sync(0xffffffffu, x, off);
            x = kMax ? fmaxf(x, y) : x + y;
        }
        if (lane == 0) red[warp * N + r] = x;
    }
    softmax_sync();
#pragma unroll
    for (int r = 0; r < N; ++r) {
        const float a = red[r], b = red[N + r], c = red[2 * N + r], d = red[3 * N + r];
        v[r] = kMax ? fmaxf(fmaxf(a, b), fmaxf(c, d)) : (a + b) + (c + d);
    }
    softmax_sync();  // red is reused
}

template <int N, bool TREE>
__global__ void __launch_bounds__(kVtBlock, 1) verify_tc_kernel(const VerifyParams p) {
    using Map = VtMap<N>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* base = smem_raw;
    const uint32_t sbase = smem_u32(smem_raw);
    VtBars* bars = reinterpret_cast<VtBars*>(base + Map::MISC);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + Map::MISC + 256);
    uint8_t* s_valid = base + Map::MISC + 264;  // [2][8] staged pool-tile flags
    volatile int* s_abort = reinterpret_cast<volatile int*>(base + Map::MISC + 280);
    int* s_last = reinterpret_cast<int*>(base + Map::MISC + 284);
    unsigned long long* anc = reinterpret_cast<unsigned long long*>(base + Map::ANC);
    float* red = reinterpret_cast<float*>(base + Map::RED);
    uint32_t* pgs = reinterpret_cast<uint32_t*>(base + Map::PGS);  // page id of every pool tile of the chunk

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;

    // ---- geometry (the split-KV kernels' clamps)
    const int cap = p.max_blocks * p.tpp * 16;
    const uint32_t tk_u = p.cu_k[b + 1] - p.cu_k[b];
    const int Tk = tk_u > (uint32_t)cap ? cap : (int)tk_u;
    const uint32_t tq_u = p.cu_q[b + 1] - p.cu_q[b];
    const int Tq = tq_u > (uint32_t)p.max_seqlen_q ? p.max_seqlen_q : (int)tq_u;
    if (tid == 0 && c == 0) {
        if (tk_u > (uint32_t)cap) atomicOr(p.status, YF_DEV_LEN_OVERFLOW);
        if (tq_u > (uint32_t)p.max_seqlen_q || Tq > Tk) atomicOr(p.status, YF_DEV_BAD_ROWS);
    }
    const int R = min(p.G * Tq, N);  // rows of the unit
    const int kv0 = Tk - Tq;         // first draft key
    const int n_kt = (Tk + kVtKeys - 1) / kVtKeys;
    const int n_ch = max(1, (n_kt + p.chunk_tiles - 1) / p.chunk_tiles);
    if (c >= n_ch) return;
    const int kt0 = c * p.chunk_tiles;
    const int n = max(0, min(p.chunk_tiles, n_kt - kt0));  // key tiles of this CTA
    if (sbase & 1023u) {
        if (tid == 0) atomicOr(p.status, YF_DEV_SMEM_ALIGN);
        return;
    }
    const int qrow0 = (int)p.cu_q[b];
    const int pt_total = (Tk + 15) / 16;
    const uint32_t* btrow = p.bt + (size_t)b * p.max_blocks;
    const uint8_t* head_base = p.layer_base + (size_t)h * p.phb;
    const long long page_stride = p.phb * p.H;

    // ---- set-up
    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bars->raw_full[i], 1);
            mbar_init(&bars->raw_free[i], 4);
            mbar_init(&bars->k_full[i], 4);
            mbar_init(&bars->k_free[i], 1);
            mbar_init(&bars->v_full[i], 4);
            mbar_init(&bars->v_free[i], 1);
            mbar_init(&bars->s_full[i], 1);
            mbar_init(&bars->s_free[i], 4);
            mbar_init(&bars->p_full[i], 4);
            mbar_init(&bars->p_free[i], 1);
        }
        mbar_init(&bars->o_done, 1);
        mbar_init(&bars->drain, 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == kVtCtl) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(N == 16 ? 64 : 128)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    int bad = 0;
    if (warp < 4) {
        // Q row r (draft r / G, q head h*G + r % G) into the SW128 B operand; rows >= R are zero
        const int r = tid;
        if (r < N) {
            const bool live = r < R;
            const uint4* qp =
                live ? reinterpret_cast<const uint4*>(p.q + ((size_t)(qrow0 + r / p.G) * p.Hq + (size_t)h * p.G + r % p.G) * kVtD)
                     : nullptr;
#pragma unroll
            for (int cc = 0; cc < 16; ++cc)
                sts128(sbase + Map::Q + sw128_off(r, cc, N), live ? __ldg(qp + cc) : make_uint4(0, 0, 0, 0));
        }
        fence_proxy_async_smem();
        // the page id of every pool tile of the chunk, read once: the copy warp then issues each
        // key tile's copies without a dependent global load; every page the CTA reads exists in
        // the common case, which skips per-key page checks
        for (int i = tid; i < n * kVtPoolTiles; i += 128) {
            const int pt = kt0 * kVtPoolTiles + i;
            const uint32_t pg = pt < pt_total ? __ldg(btrow + pt / p.tpp) : (uint32_t)p.n_pages;
            pgs[i] = pg;
            if (pt < pt_total && pg >= (uint32_t)p.n_pages) bad = 1;
        }
        if constexpr (TREE) {
            // ancestor masks of the entry's draft nodes from their subtree ranges (clamped to the
            // block; a range outside it flags YF_DEV_BAD_ROWS)
            for (int i = tid; i < kVtMaxTree; i += 128) anc[i] = 0ull;
            softmax_sync();
            for (int j = tid; j < Tq; j += 128) {
                const int2 rg = p.trie[qrow0 + j];
                if (rg.x < 0 || rg.y >= Tq || rg.x > rg.y) atomicOr(p.status, YF_DEV_BAD_ROWS);
                const int lo = max(max(rg.x, j), 0), hi = min(rg.y, Tq - 1);
                for (int i = lo; i <= hi; ++i) atomicOr(&anc[i], 1ull << j);
            }
        }
    }
    tc_fence_before();
    const bool pages_ok = __syncthreads_or(bad) == 0;
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    constexpr uint32_t IDESC = umma_idesc_f16(128, N);

    if (warp == kVtCtl) {
        // ================= control: every MMA and commit =================
        if (lane == 0 && n > 0) {
            int qk = 0, pv = 0;
            uint32_t idle = 0;
            uint64_t idle_t0 = 0;
            while (pv < n && !*s_abort) {
                bool prog = false;
                // QK(qk) into S buffer qk & 1, once the softmax has read QK(qk - 2) from it
                if (qk < n && (qk < 2 || mbar_test(&bars->s_free[qk & 1], (qk >> 1) - 1)) &&
                    mbar_test(&bars->k_full[qk & 1], qk >> 1)) {
                    tc_fence_after();
#pragma unroll
                    for (int ks = 0; ks < kVtD / 16; ++ks) {
                        const uint64_t a =
                            umma_desc_sw128(sbase + Map::K + (qk & 1) * 32768 + (ks >> 2) * 16384 + (ks & 3) * 32);
                        const uint64_t bd = umma_desc_sw128(sbase + Map::Q + (ks >> 2) * (N * 128) + (ks & 3) * 32);
                        umma_ss(tmem + (qk & 1) * N, a, bd, IDESC, ks > 0);
                    }
                    umma_commit(&bars->s_full[qk & 1]);
                    umma_commit(&bars->k_free[qk & 1]);
                    ++qk;
                    prog = true;
                }
                // PV(pv) once its P and V^T are written
                if (pv < qk && mbar_test(&bars->p_full[pv & 1], pv >> 1) && mbar_test(&bars->v_full[pv & 1], pv >> 1)) {
                    tc_fence_after();
#pragma unroll
                    for (int ks = 0; ks < kVtKeys / 16; ++ks) {
                        const uint64_t a =
                            umma_desc_sw128(sbase + Map::VT + (pv & 1) * 32768 + (ks >> 2) * 16384 + (ks & 3) * 32);
                        const uint64_t bd =
                            umma_desc_sw128(sbase + Map::P + (pv & 1) * (N * 256) + (ks >> 2) * (N * 128) + (ks & 3) * 32);
                        umma_ss(tmem + 2 * N, a, bd, IDESC, (pv > 0 || ks > 0) ? 1u : 0u);
                    }
                    umma_commit(&bars->p_free[pv & 1]);
                    umma_commit(&bars->v_free[pv & 1]);
                    if (pv == n - 1) umma_commit(&bars->o_done);
                    ++pv;
                    prog = true;
                }
                if (prog) {
                    idle = 0;
                } else if (++idle == 1) {
                    idle_t0 = globaltimer_ns();
                } else if ((idle & 63u) == 0 && globaltimer_ns() - idle_t0 > p.wait_ns) {
                    vt_give_up(s_abort, p.status);
                }
            }
            umma_commit(&bars->drain);  // every MMA has completed before TMEM is released
            if (!mbar_wait(&bars->drain, 0u, p.wait_ns)) vt_give_up(s_abort, p.status);
        }
        __syncwarp();
    } else if (warp == kVtCopy) {
        // ================= copies: the 8 pool tiles of a key tile into the raw ring =================
        if (lane == 0) {
            for (int i = 0; i < n; ++i) {
                const int kt = kt0 + i, slot = i & 1;
                uint32_t cur[kVtPoolTiles];
#pragma unroll
                for (int j = 0; j < kVtPoolTiles; ++j) cur[j] = pgs[i * kVtPoolTiles + j];
                if (i >= 2 && !vt_wait(&bars->raw_free[slot], (i >> 1) - 1, s_abort, p.status, p.wait_ns)) break;
                uint8_t* dst = base + Map::RAW + slot * kVtPoolTiles * kVtRawPitch;
                uint32_t bytes = 0;
                const uint8_t* src[kVtPoolTiles];
#pragma unroll
                for (int j = 0; j < kVtPoolTiles; ++j) {
                    const int pt = kt * kVtPoolTiles + j;
                    src[j] = nullptr;
                    if (cur[j] < (uint32_t)p.n_pages)
                        src[j] = head_base + (size_t)cur[j] * page_stride + (pt % p.tpp) * kVtRawTile;
                    else if (pt < pt_total)
                        atomicOr(p.status, YF_DEV_BAD_PAGE);
                    s_valid[slot * kVtPoolTiles + j] = src[j] != nullptr;
                    bytes += src[j] ? kVtRawTile : 0;
                }
                mbar_arrive_expect_tx(&bars->raw_full[slot], bytes);
#pragma unroll
                for (int j = 0; j < kVtPoolTiles; ++j)
                    if (src[j]) bulk_g2s(dst + j * kVtRawPitch, src[j], kVtRawTile, &bars->raw_full[slot]);
            }
        }
        __syncwarp();
    } else if (warp >= 4) {
        // ================= dequant: raw pool tiles -> f16 K [key][dim] and V^T [dim][key] =================
        const int t = tid - 128, dw = t >> 5;  // dw: this warp's 32-dim block (K) / dim bits 5-6 (V)
        // K: lane -> (token g, dim octet tig) of a 512-byte block, paired so that each
        // quarter-warp's loads and swizzled stores hit eight distinct 16-byte bank groups
        const int qw = lane >> 3, k8 = lane & 7;
        const int kg = (k8 < 4) ? qw : (qw ^ 5), ktig = k8 & 3;
        // V: lane -> (dim bits 4, 3, 0; pool tile of the half); the step gives dim bits 1-2
        const int vm1 = lane >> 4, vdh = (lane >> 3) & 1, vjt = (lane >> 1) & 3, vg1 = lane & 1;
        for (int i = 0; i < n; ++i) {
            const int slot = i & 1;
            (void)vt_wait(&bars->raw_full[slot], i >> 1, s_abort, p.status, p.wait_ns);
            if (i >= 2) (void)vt_wait(&bars->k_free[slot], (i >> 1) - 1, s_abort, p.status, p.wait_ns);
            const uint8_t* raw = base + Map::RAW + slot * kVtPoolTiles * kVtRawPitch;
            const uint32_t kdst = sbase + Map::K + slot * 32768;
#pragma unroll
            for (int jt = 0; jt < kVtPoolTiles; ++jt) {
                // K: tokens kg, kg+8 x dims 32dw + 8ktig .. +7 of pool tile jt
                const uint8_t* T = raw + jt * kVtRawPitch;
                uint4 o0 = make_uint4(0, 0, 0, 0), o1 = make_uint4(0, 0, 0, 0);
                if (s_valid[slot * kVtPoolTiles + jt]) {
                    const uint4 kw = lds128(T + dw * 512 + (kg * 4 + ktig) * 16);
                    const uint16_t s0 = *reinterpret_cast<const uint16_t*>(T + 16 * kVtD + 2 * ((kg * 2) * 4 + dw));
                    const uint16_t s1 = *reinterpret_cast<const uint16_t*>(T + 16 * kVtD + 2 * ((kg * 2 + 1) * 4 + dw));
                    const uint32_t d0 = (uint32_t)s0 | ((uint32_t)s0 << 16), d1 = (uint32_t)s1 | ((uint32_t)s1 << 16);
                    o0 = make_uint4(dq2(kw.x, 0, d0), dq2(kw.x, 1, d0), dq2(kw.y, 0, d0), dq2(kw.y, 1, d0));
                    o1 = make_uint4(dq2(kw.z, 0, d1), dq2(kw.z, 1, d1), dq2(kw.w, 0, d1), dq2(kw.w, 1, d1));
                }
                const int key = jt * 16 + kg, cc = dw * 4 + ktig;
                sts128(kdst + sw128_off(key, cc, kVtKeys), o0);
                sts128(kdst + sw128_off(key + 8, cc, kVtKeys), o1);
            }
            fence_proxy_async_smem();
            dequant_sync();
            if (lane == 0) mbar_arrive(&bars->k_full[slot]);
            if (i >= 2) (void)vt_wait(&bars->v_free[slot], (i >> 1) - 1, s_abort, p.status, p.wait_ns);
#pragma unroll
            for (int e = 0; e < 2; ++e) {  // key halves 0-63, 64-127: V^T column blocks
                const int jt = e * 4 + vjt;
                const uint8_t* TV = raw + jt * kVtRawPitch;
                const bool vvalid = s_valid[slot * kVtPoolTiles + jt] != 0;
                const uint32_t vdst = sbase + Map::VT + slot * 32768 + e * 16384;
                uint32_t sp[8];  // (token 2k, 2k+1) scale pairs for k = 0..7
                if (vvalid) {
                    const uint8_t* vsc = TV + 32 * kVtD + 128 + dw * 8;
#pragma unroll
                    for (int qq = 0; qq < 4; ++qq) {
                        const uint2 pr = lds64(vsc + qq * 32);
                        sp[qq] = __byte_perm(pr.x, pr.y, 0x5410);
                        sp[4 + qq] = __byte_perm(pr.x, pr.y, 0x7632);
                    }
                }
#pragma unroll
                for (int st = 0; st < 4; ++st) {
                    const int d = 32 * dw + 16 * vm1 + 8 * vdh + 2 * st + vg1;
                    const int m = d >> 4, gp = d & 7;
                    uint4 lo = make_uint4(0, 0, 0, 0), hi = make_uint4(0, 0, 0, 0);
                    if (vvalid) {
                        const uint8_t* vb = TV + 16 * kVtD + 128 + (m >> 1) * 512 + ((m & 1) * 2 + vdh) * 4;
                        uint32_t wv[4];
#pragma unroll
                        for (int qq = 0; qq < 4; ++qq) wv[qq] = lds32(vb + (gp * 4 + qq) * 16);
                        const uint32_t k03 = __byte_perm(wv[0], wv[1], 0x6420), k47 = __byte_perm(wv[2], wv[3], 0x6420);
                        const uint32_t k8b = __byte_perm(wv[0], wv[1], 0x7531), kcf = __byte_perm(wv[2], wv[3], 0x7531);
                        lo = make_uint4(dq2(k03, 0, sp[0]), dq2(k03, 1, sp[1]), dq2(k47, 0, sp[2]), dq2(k47, 1, sp[3]));
                        hi = make_uint4(dq2(k8b, 0, sp[4]), dq2(k8b, 1, sp[5]), dq2(kcf, 0, sp[6]), dq2(kcf, 1, sp[7]));
                    }
                    sts128(vdst + sw128_off(d, 2 * vjt, kVtD), lo);
                    sts128(vdst + sw128_off(d, 2 * vjt + 1, kVtD), hi);
                }
            }
            fence_proxy_async_smem();
            dequant_sync();
            if (lane == 0) {
                mbar_arrive(&bars->v_full[slot]);
                mbar_arrive(&bars->raw_free[slot]);
            }
        }
    } else {
        // ================= softmax: thread = key (TMEM lane) =================
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        const float sl2 = p.scale_log2;
        float m_run[N], l_part[N];
#pragma unroll
        for (int r = 0; r < N; ++r) {
            m_run[r] = -INFINITY;
            l_part[r] = 0.f;
        }
        for (int i = 0; i < n; ++i) {
            const int kt = kt0 + i, key = kt * kVtKeys + tid;
            (void)vt_wait(&bars->s_full[i & 1], i >> 1, s_abort, p.status, p.wait_ns);
            __syncwarp();
            tc_fence_after();
            float v[N];
            if constexpr (N == 16) {
                tmem_ld16(tmem + (i & 1) * N + lane_off, v);
            } else {
                tmem_ld32(tmem + (i & 1) * N + lane_off, v);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->s_free[i & 1]);
            bool key_live = key < Tk;
            if (!pages_ok && key_live) key_live = pgs[i * kVtPoolTiles + (tid >> 4)] < (uint32_t)p.n_pages;
            bool need = false;
            // draft row j = r / G sees keys < kv0 + j + 1; rows past the unit's R see none
            const int kq = key - kv0;  // >= 0 only for draft keys
#pragma unroll
            for (int r = 0; r < N; ++r) {
                bool vis = key_live && r < R && kq <= r / p.G;
                if constexpr (TREE) {
                    if (vis && kq >= 0) vis = (anc[r / p.G] >> kq) & 1ull;
                }
                v[r] = vis ? v[r] * sl2 : -INFINITY;
                need |= v[r] > m_run[r] + kVtRescale;
            }
            if (softmax_any(need)) {
                float mt[N];
#pragma unroll
                for (int r = 0; r < N; ++r) mt[r] = v[r];
                rows_reduce<N, true>(mt, red, warp, lane);
                float alpha[N];
                bool any_scale = false;
#pragma unroll
                for (int r = 0; r < N; ++r) {
                    alpha[r] = 1.f;
                    if (mt[r] > m_run[r] + kVtRescale) {
                        alpha[r] = fast_exp2(m_run[r] - mt[r]);  // 0 while nothing is accumulated
                        m_run[r] = mt[r];
                        l_part[r] *= alpha[r];
                        any_scale = true;
                    }
                }
                if (any_scale && i > 0) {
                    // O holds PV(i-1) once it completes (PV(i) waits for this tile's P)
                    (void)vt_wait(&bars->p_free[(i - 1) & 1], (i - 1) >> 1, s_abort, p.status, p.wait_ns);
                    __syncwarp();
                    tc_fence_after();
                    float o[N];
                    uint32_t ob[N];
                    if constexpr (N == 16) {
                        tmem_ld16(tmem + 2 * N + lane_off, o);
                    } else {
                        tmem_ld32(tmem + 2 * N + lane_off, o);
                    }
#pragma unroll
                    for (int r = 0; r < N; ++r) ob[r] = __float_as_uint(o[r] * alpha[r]);
                    if constexpr (N == 16) {
                        tmem_st16(tmem + 2 * N + lane_off, ob);
                    } else {
                        tmem_st32(tmem + 2 * N + lane_off, ob);
                    }
                    tmem_wait_st();
                    tc_fence_before();
                }
            }
            // P buffer i & 1 was last read by PV(i - 2)
            if (i >= 2) (void)vt_wait(&bars->p_free[i & 1], (i >> 1) - 1, s_abort, p.status, p.wait_ns);
            const uint32_t pdst = sbase + Map::P + (i & 1) * (N * 256) + (tid & 7) * 2;
#pragma unroll
            for (int r = 0; r < N; ++r) {
                const float pr = m_run[r] == -INFINITY ? 0.f : fast_exp2(v[r] - m_run[r]);
                l_part[r] += pr;
                const __half hp = __float2half_rn(pr);
                asm volatile("st.shared.u16 [%0], %1;" ::"r"(pdst + sw128_off(r, tid >> 3, N)),
                             "h"(__half_as_ushort(hp))
                             : "memory");
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->p_full[i & 1]);
        }
        // ---- epilogue: row sums, then thread = dim reads its O^T lane
        rows_reduce<N, false>(l_part, red, warp, lane);
        float o[N];
        if (n > 0) {
            (void)vt_wait(&bars->o_done, 0, s_abort, p.status, p.wait_ns);
            __syncwarp();
            tc_fence_after();
            if constexpr (N == 16) {
                tmem_ld16(tmem + 2 * N + lane_off, o);
            } else {
                tmem_ld32(tmem + 2 * N + lane_off, o);
            }
        } else {
#pragma unroll
            for (int r = 0; r < N; ++r) o[r] = 0.f;
        }
        const int d = tid;
        const size_t unit = (size_t)b * p.H + h;
        if (n_ch == 1) {
#pragma unroll
            for (int r = 0; r < N; ++r) {
                if (r >= R) break;
                const float inv = l_part[r] > 0.f ? 1.f / l_part[r] : 0.f;
                p.out[((size_t)(qrow0 + r / p.G) * p.Hq + (size_t)h * p.G + r % p.G) * kVtD + d] = __float2half_rn(o[r] * inv);
            }
        } else {
            const size_t item = unit * p.max_chunks + c;
#pragma unroll
            for (int r = 0; r < N; ++r) {
                const float inv = l_part[r] > 0.f ? 1.f / l_part[r] : 0.f;
                __stcg(p.ws_o + (item * N + r) * kVtD + d, o[r] * inv);
                if (d == 0) __stcg(p.ws_lse + item * N + r, l_part[r] > 0.f ? m_run[r] + __log2f(l_part[r]) : -INFINITY);
            }
            __threadfence();
            softmax_sync();
            if (tid == 0) *s_last = atomicAdd(&p.counters[unit], 1u) == (uint32_t)n_ch - 1;
            softmax_sync();
            if (*s_last) {
                __threadfence();
                // the unit's chunks merged: thread = dim, every row
                for (int r = 0; r < R; ++r) {
                    float M = -INFINITY;
                    for (int k = 0; k < n_ch; ++k) M = fmaxf(M, __ldcg(p.ws_lse + (unit * p.max_chunks + k) * N + r));
                    float L = 0.f, acc = 0.f;
                    for (int k0 = 0; k0 < n_ch; k0 += 8) {
                        float lv[8], ov[8];
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            lv[j] = -INFINITY;
                            ov[j] = 0.f;
                            if (k0 + j < n_ch) {
                                const size_t it = unit * p.max_chunks + k0 + j;
                                lv[j] = __ldcg(p.ws_lse + it * N + r);
                                ov[j] = __ldcg(p.ws_o + (it * N + r) * kVtD + d);
                            }
                        }
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            if (lv[j] == -INFINITY) continue;
                            const float f = fast_exp2(lv[j] - M);
                            L += f;
                            acc = fmaf(f, ov[j], acc);
                        }
                    }
                    p.out[((size_t)(qrow0 + r / p.G) * p.Hq + (size_t)h * p.G + r % p.G) * kVtD + d] =
                        __float2half_rn(L > 0.f ? acc / L : 0.f);
                }
                if (tid == 0) p.counters[unit] = 0;  // ready for the next call on this pool
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kVtCtl) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(N == 16 ? 64 : 128)
                     : "memory");
    }
}

template <int N, bool TREE>
int launch_t(const AttnArgs& a, const VerifyParams& p, int max_chunks) {
    auto kern = verify_tc_kernel<N, TREE>;
    static LaunchCache cache;
    const int rc = raise_smem_attr((const void*)kern, VtMap<N>::ALLOC, a.pool->desc.device, cache);
    if (rc) return rc;
    const dim3 grid((unsigned)max_chunks, a.pool->desc.n_kv_heads, a.batch);
    kern<<<grid, kVtBlock, VtMap<N>::ALLOC, a.stream>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? YF_OK : cuda_fail(e, "verify_tc launch");
}

}  // namespace

bool verify_tc_applies(const yf_pool* pool, int n_q_heads, int max_seqlen_q, bool tree) {
    if (pool->opts.verify_kernel != YF_VERIFY_TCGEN05) return false;
    const yf_pool_desc& d = pool->desc;
    const int G = n_q_heads / d.n_kv_heads;
    const int rows = G * max_seqlen_q;
    return d.head_dim == kVtD && d.group_size == 32 && max_seqlen_q > 1 && rows <= 32 &&
           (!tree || max_seqlen_q <= kVtMaxTree);
}

VerifyPlan plan_verify(const yf_pool* pool, int n_q_heads, int batch, int max_seqlen_q, int max_seqlen_k) {
    VerifyPlan v;
    const int G = n_q_heads / pool->desc.n_kv_heads;
    v.rows = G * max_seqlen_q <= 16 ? 16 : 32;
    const long long units = (long long)batch * pool->desc.n_kv_heads;
    const int max_kt = (max_seqlen_k + kVtKeys - 1) / kVtKeys;
    // 16 to 64 key tiles per CTA: enough CTAs for ~8 waves over the SMs, few enough that the
    // per-CTA set-up and the merge stay small against the stream
    long long ct = (units * max_kt + (long long)pool->sm_count * 8 - 1) / ((long long)pool->sm_count * 8);
    ct = std::max<long long>(16, std::min<long long>(kVtMaxChunkTiles, ct));
    v.chunk_tiles = (int)ct;
    v.max_chunks = std::max(1, (max_kt + v.chunk_tiles - 1) / v.chunk_tiles);
    v.ws_bytes = v.max_chunks > 1 ? (size_t)units * v.max_chunks * v.rows * (kVtD + 1) * sizeof(float) : 0;
    return v;
}

int launch_verify_tc(const AttnArgs& a, const VerifyPlan& plan) {
    const yf_pool_desc& d = a.pool->desc;
    VerifyParams p;
    p.layer_base = a.pool->base + (size_t)a.layer * a.pool->layer_bytes;
    p.n_pages = d.n_pages;
    p.H = d.n_kv_heads;
    p.G = a.n_q_heads / d.n_kv_heads;
    p.Hq = a.n_q_heads;
    p.phb = (long long)a.pool->page_head_bytes;
    p.tpp = d.page_size / 16;
    p.q = a.q;
    p.cu_q = a.cu_q;
    p.cu_k = a.cu_k;
    p.bt = a.block_table;
    p.max_blocks = a.max_blocks;
    p.max_seqlen_q = a.max_seqlen_q;
    p.chunk_tiles = plan.chunk_tiles;
    p.max_chunks = plan.max_chunks;
    p.scale_log2 = a.scale * 1.4426950408889634f;
    p.out = a.out;
    p.ws_o = static_cast<float*>(a.workspace);
    const size_t items = (size_t)a.batch * d.n_kv_heads * plan.max_chunks;
    p.ws_lse = plan.ws_bytes ? p.ws_o + items * plan.rows * kVtD : nullptr;
    p.counters = a.pool->d_counters;
    p.status = a.pool->d_status;
    p.trie = reinterpret_cast<const int2*>(a.trie);
    p.wait_ns = wait_limit_ns(a.pool);
    if ((size_t)a.batch * d.n_kv_heads > (size_t)kMaxCombineUnits)
        return fail(YF_E_UNSUPPORTED, "tensor-core verify of more than %d units", kMaxCombineUnits);
    if (p.trie) return plan.rows == 16 ? launch_t<16, true>(a, p, plan.max_chunks) : launch_t<32, true>(a, p, plan.max_chunks);
    return plan.rows == 16 ? launch_t<16, false>(a, p, plan.max_chunks) : launch_t<32, false>(a, p, plan.max_chunks);
}

}  // namespace yf
