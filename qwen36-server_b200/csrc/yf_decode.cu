// Split-KV paged Q8_0 attention for decode, MTP verify and other small query
// blocks, plus the log-sum-exp merge of split partials.
//
// Replaces the int8-pool decode/verify branch of the engine's FA2 split-KV
// kernel (compute_attn_1rowblock_splitkv with Is_kv_q8, described at
// docs/research/2026-09-16-head-to-head-llamacpp-and-phase-profile.md:3469-3481)
// and flash_fwd_splitkv_combine_kernel (docs/plans/2026-09-16-prefil-parity-fa2-and-mmq.md:104-107).
//
// A "unit" is (entry b, kv head h, group of 8 or 16 query rows): the G = Hq/Hkv
// q heads of kv head h times the entry's query positions, folded into the MMA
// N dimension so every K/V byte is read once per unit.  The unit's keys are
// 16-token tiles, each one contiguous block of the pool (K int8 + scales +
// V int8 + scales).  Each of a CTA's 4 warps streams its own tiles: lane 0
// issues a 1-D bulk copy (cp.async.bulk into this CTA only) of the whole tile into
// a per-warp ring of shared-memory stages, completing on an mbarrier, and
// loads the next tile's page id one tile ahead.  The tile bytes are laid out
// so that each lane's 16-byte shared load is exactly its mma.sync fragment:
// K feeds S^T = K Q^T (tokens in M), V feeds O^T = V^T P^T (dims in M); int8
// is unpacked to exact f16 in registers and the Q8_0 group scales multiply
// the per-group partial dot products (K) and P (V).  Softmax is online, base
// 2, with warp-shuffle row maxima and a lazy rescale; the 4 warps of a CTA
// merge through shared memory.
//
// Two schedules share that tile code:
//  * decode_persistent_kernel (one row group per entry, B <= 1024): a grid of
//    (SMs x resident CTAs) splits the global sequence of (unit, tile) into
//    equal contiguous ranges, so every CTA streams the same number of bytes
//    and no SM idles at the tail.  A range covers whole units (written
//    directly) and at most two unit pieces (written as partials); the CTA that
//    finishes a unit's last piece merges the pieces (an arrival counter per
//    unit in the pool).
//  * splitkv_kernel (everything else): a 3-D grid of (unit, chunk of tiles)
//    with the same last-arrival merge, or the separate splitkv_combine launch.
// Calls on one pool must be stream-ordered (the counters belong to the pool).
#include <algorithm>
#include <cfloat>
#include <mutex>

#include "yf_device.cuh"
#include "yf_internal.h"
#include "yf_xchg.cuh"

namespace yf {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kHdrBytes = 256;  // mbarriers + per-stage page-valid flags
constexpr int kMaxTreeRows = 64;  // draft rows per entry of a tree verify (one 64-bit mask each)
// 16-row units (two n-tiles) are bound by instruction issue rather than by HBM: their QK feeds
// K as the f16 values 1152 + k and starts each scale group's accumulator at -1152 x (the row's q
// summed over the group), read per warp from shared memory: [group][tig][n-tile][4] floats.
template <int NT>
constexpr bool kbias_in_acc() { return NT == 2; }
template <int NB, int NT, bool TREE = false>
constexpr int hdr_bytes() {
    return kHdrBytes + (kbias_in_acc<NT>() ? kWarps * NB * 4 * NT * 16 : 0) + (TREE ? kMaxTreeRows * 8 : 0);
}
template <int NB, int NT>
__device__ __forceinline__ float* kbias_area(uint8_t* smem, int warp) {
    return reinterpret_cast<float*>(smem + kHdrBytes) + warp * NB * 4 * NT * 4;
}
// Lazy softmax rescale: the running max only moves when a tile's max exceeds it by
// more than 8 (base 2), so most tiles skip the O rescale and p stays <= 256.
constexpr float kRescaleThresh = 8.0f;
static_assert(kWarps * 32 * 128 * kMaxCtasPerSm <= 65536, "register budget of the resident CTAs");

struct SplitParams {
    const uint8_t* layer_base;
    int n_pages;
    int H;  // kv heads
    int G;  // q heads per kv head
    int Hq;
    int B;
    long long phb;  // bytes of one (page, kv head)
    const __half* q;
    const uint32_t* cu_q;  // null for decode
    const uint32_t* cu_k;
    const uint32_t* bt;
    int max_blocks;
    int max_seqlen_q;
    int n_row_groups;
    int chunk_tiles;
    int max_chunks;
    float scale_log2;
    __half* out;
    float* part_o;    // partial output (f32 O + natural-log lse) instead of `out`, or null
    float* part_lse;
    float* ws_o;
    float* ws_lse;
    uint32_t* counters;  // per-unit arrival counters for the merge, or null (separate combine)
    uint32_t* status;
    const int2* trie;    // tree verify: inclusive subtree range of every draft row, or null
    uint64_t wait_ns;    // bound of every wait (copies, merge arrivals)
    XFuse x;             // fused partial exchange (cluster schedule), x.peers null when off
};

// Tree verify: the draft rows of an entry are the nodes of a token trie in depth-first order;
// row i sees the committed keys and draft key j when j <= i and i lies in node j's subtree
// range (j is i or an ancestor).  anc[i] has bit j set for those j.
struct TreeCtx {
    const unsigned long long* anc;  // [Tq] in shared memory
    int kv0;                        // first draft key (Tk - Tq)
    int row0;                       // first row of the unit
    int G;
};

// Geometry of one unit, computed identically everywhere.
struct UnitGeom {
    int Tk, Tq, qrow0, rows_total, row_begin, n_tiles, n_chunks;
};

template <int TPP, int RPC>
__device__ __forceinline__ bool unit_geom(const SplitParams& p, int b, int rg, UnitGeom& u, bool flag) {
    const int cap = p.max_blocks * (TPP * kTileTokens);
    const uint32_t tk = p.cu_k[b + 1] - p.cu_k[b];
    u.Tk = tk > (uint32_t)cap ? cap : (int)tk;
    if (flag && tk > (uint32_t)cap) atomicOr(p.status, YF_DEV_LEN_OVERFLOW);
    u.Tq = 1;
    u.qrow0 = b;
    if (p.cu_q) {
        const uint32_t tq = p.cu_q[b + 1] - p.cu_q[b];
        u.Tq = tq > (uint32_t)p.max_seqlen_q ? p.max_seqlen_q : (int)tq;
        u.qrow0 = (int)p.cu_q[b];
        if (flag && (tq > (uint32_t)p.max_seqlen_q || u.Tq > u.Tk)) atomicOr(p.status, YF_DEV_BAD_ROWS);
    }
    u.rows_total = p.G * u.Tq;
    u.row_begin = rg * RPC;
    if (u.row_begin >= u.rows_total) return false;
    const int row_end = min(u.row_begin + RPC, u.rows_total);
    int kv_hi = u.Tk - u.Tq + (row_end - 1) / p.G + 1;
    kv_hi = max(0, min(kv_hi, u.Tk));
    u.n_tiles = (kv_hi + kTileTokens - 1) / kTileTokens;
    u.n_chunks = max(1, (u.n_tiles + p.chunk_tiles - 1) / p.chunk_tiles);
    return true;
}

// Offset (in halves) of query / output row `row` of unit u (q and out share the layout).
__device__ __forceinline__ size_t row_offset(const SplitParams& p, const UnitGeom& u, int h, int row, int D) {
    const int j = row / p.G, gi = row % p.G;
    return ((size_t)(u.qrow0 + j) * p.Hq + (size_t)h * p.G + gi) * D;
}

// Final output of dims d4 .. d4+3 of `row` (kv head h of unit u): normalised O `v` and the
// row's base-2 lse `lse2` (-inf without keys).  f16 into out, or with partial output on, f32
// O into part_o (same layout) and the natural-log lse into part_lse[row][q head].
__device__ __forceinline__ void store_row4(const SplitParams& p, const UnitGeom& u, int h, int row, int d4, int D,
                                           float4 v, float lse2) {
    const size_t off = row_offset(p, u, h, row, D);
    if (p.part_o) {
        *reinterpret_cast<float4*>(p.part_o + off + d4) = v;
        if (d4 == 0) p.part_lse[off / D] = lse2 * 0.6931471805599453f;
    } else {
        uint2 pk;
        pk.x = pack_h2(v.x, v.y);
        pk.y = pack_h2(v.z, v.w);
        *reinterpret_cast<uint2*>(p.out + off + d4) = pk;
    }
}

// Final output of a cluster-decode row slice: store_row4, or with the fused exchange on, the
// f32 O and natural-log lse as (value, xstep) words into slot `rank` of word buffer xstep & 1 of
// every rank's area (the partial layout of part_o / part_lse, lse rows at x.lse_off).
__device__ __forceinline__ void store_out4(const SplitParams& p, const UnitGeom& u, int h, int row, int d4, int D,
                                           float4 v, float lse2, uint32_t xstep) {
    if (!p.x.peers) {
        store_row4(p, u, h, row, d4, D, v, lse2);
        return;
    }
    const size_t off = row_offset(p, u, h, row, D);
    const unsigned long long lse = ll_word(lse2 * 0.6931471805599453f, xstep);
    const unsigned long long w0 = ll_word(v.x, xstep), w1 = ll_word(v.y, xstep), w2 = ll_word(v.z, xstep),
                             w3 = ll_word(v.w, xstep);
    const long long slot0 = ((long long)(xstep & 1u) * p.x.world + p.x.rank) * p.x.slot_floats;
    for (int k = 0; k < p.x.world; ++k) {
        unsigned long long* wd = reinterpret_cast<unsigned long long*>(p.x.peers[k] + p.x.words_off) + slot0;
        st_ll2(wd + off + d4, w0, w1);
        st_ll2(wd + off + d4 + 2, w2, w3);
        if (d4 == 0) st_ll1(wd + p.x.lse_off + off / D, lse);
    }
}

// The fused exchange's merge, by the CTA that stored output row `row` (of unit u) of this rank's
// partial: the same partial row of every rank arrives in the own area's word buffer xstep & 1
// (polled, bounded by x.wait_ns); head group g's output row merges ranks s * n_hg + g, s < n_seq,
// with xmerge4's arithmetic.  One thread per (head group, float4 column).  A wait that runs out
// sets YF_DEV_TIMEOUT in the area's status word and leaves the element unwritten.
template <int D>
__device__ __forceinline__ void exchange_merge_row(const SplitParams& p, const UnitGeom& u, int h, int row,
                                                   uint32_t xstep) {
    const XFuse& x = p.x;
    constexpr int d4n = D / 4;
    const size_t pr = row_offset(p, u, h, row, D) / D;  // partial row
    const unsigned long long* wd = reinterpret_cast<const unsigned long long*>(x.local + x.words_off) +
                                   (long long)(xstep & 1u) * x.world * x.slot_floats;
    const uint64_t t0 = globaltimer_ns();
    for (int e = threadIdx.x; e < x.n_hg * d4n; e += kThreads) {
        const int g = e / d4n, c = e % d4n;
        float lv[kXMaxSeq];
        bool ok = true;
        float M = -INFINITY;
        for (int s = 0; s < x.n_seq && ok; ++s) {
            ok = ll_wait1(wd + (long long)(s * x.n_hg + g) * x.slot_floats + x.lse_off + pr, xstep, t0, x.wait_ns, lv[s]);
            M = fmaxf(M, lv[s]);
        }
        float L = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s = 0; s < x.n_seq && ok; ++s) {
            float4 v;
            const unsigned long long* src = wd + (long long)(s * x.n_hg + g) * x.slot_floats + pr * D + 4 * c;
            ok = ll_wait2(src, xstep, t0, x.wait_ns, v.x, v.y) && ll_wait2(src + 2, xstep, t0, x.wait_ns, v.z, v.w);
            if (!ok || M == -INFINITY || lv[s] == -INFINITY) continue;
            const float w = fast_exp2((lv[s] - M) * 1.4426950408889634f);
            L += w;
            acc.x = fmaf(w, v.x, acc.x);
            acc.y = fmaf(w, v.y, acc.y);
            acc.z = fmaf(w, v.z, acc.z);
            acc.w = fmaf(w, v.w, acc.w);
        }
        if (!ok) {
            atomicOr(xmeta(x.local, x.flags_off) + x.world + 1, YF_DEV_TIMEOUT);
            continue;
        }
        const float inv = L > 0.f ? 1.f / L : 0.f;
        const int b = (int)(pr / x.hq), j = (int)(pr % x.hq);
        uint2 pk;
        pk.x = pack_h2(acc.x * inv, acc.y * inv);
        pk.y = pack_h2(acc.z * inv, acc.w * inv);
        reinterpret_cast<uint2*>(x.out + ((size_t)b * x.n_q_heads + (size_t)g * x.hq + j) * D)[c] = pk;
    }
}

// After this CTA's slice stores (all threads): merges each live row of slice r and records the
// slice's step.
template <int D, int RPC, int CL>
__device__ __forceinline__ void exchange_finish(const SplitParams& p, const UnitGeom& u, int h, int r, int si,
                                                uint32_t xstep) {
    constexpr int RS = RPC / CL;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < RS; ++i) {
        const int row = u.row_begin + r * RS + i;
        if (row < u.rows_total) exchange_merge_row<D>(p, u, h, row, xstep);
    }
    if (threadIdx.x == 0)
        reinterpret_cast<uint32_t*>(p.x.local + p.x.sstep_off)[si] = xstep;  // this slice's step, for the next call
}

// mma.sync m16n8k16 f16 x f16 -> f32, D = A B + C (C may differ from D).
__device__ __forceinline__ void mma_acc(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_init(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1, const uint4 c) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(__uint_as_float(c.x)),
          "f"(__uint_as_float(c.y)), "f"(__uint_as_float(c.z)), "f"(__uint_as_float(c.w)));
}
// bytes 0,1 / 2,3 of a pool word -> f16x2 of 1152 + x (the magic value before its subtraction)
__device__ __forceinline__ uint32_t s8lo_to_h2_biased(uint32_t wb) { return __byte_perm(wb, 0x64646464u, 0x4140); }
__device__ __forceinline__ uint32_t s8hi_to_h2_biased(uint32_t wb) { return __byte_perm(wb, 0x64646464u, 0x4342); }

// ---- per-warp state and tile math ------------------------------------------------------

template <int D, int NT>
struct WarpAcc {
    float m[NT][2];
    float l[NT][2];
    float o[D / 16][NT][4];

    __device__ __forceinline__ void reset() {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            m[nt][0] = m[nt][1] = -INFINITY;
            l[nt][0] = l[nt][1] = 0.f;
        }
#pragma unroll
        for (int mt = 0; mt < D / 16; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) o[mt][nt][e] = 0.f;
    }
};

// Q^T fragments of a unit: lane holds Q[row nt*8+g][32cb + 8tig .. +7] for every chunk cb;
// and the key count each of the lane's softmax rows (2tig, 2tig+1 of each n-tile) sees.
template <int D, int NT, int NBG>
__device__ __forceinline__ void load_unit_q(const SplitParams& p, const UnitGeom& u, int h, int lane,
                                            uint4 (&qf)[NT][D / 32], int (&kvlen)[NT][2], int& kv_min,
                                            float* cw) {
    const int g = lane >> 2, tig = lane & 3;
    int km = 0x7fffffff;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int r = u.row_begin + nt * 8 + g;
        if (r < u.rows_total) {
            const uint4* qp = reinterpret_cast<const uint4*>(p.q + row_offset(p, u, h, r, D));
#pragma unroll
            for (int cb = 0; cb < D / 32; ++cb) qf[nt][cb] = __ldg(qp + cb * 4 + tig);
        } else {
#pragma unroll
            for (int cb = 0; cb < D / 32; ++cb) qf[nt][cb] = make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int col = 0; col < 2; ++col) {
            const int rr = u.row_begin + nt * 8 + 2 * tig + col;
            const int kl = u.Tk - u.Tq + rr / p.G + 1;
            kvlen[nt][col] = rr < u.rows_total ? max(0, min(kl, u.Tk)) : 0;
            if (rr < u.rows_total) km = min(km, kvlen[nt][col]);
        }
    }
    kv_min = __reduce_min_sync(0xffffffffu, km);
    if constexpr (!kbias_in_acc<NT>()) return;
    // lane (g, tig) reads {c(2tig), c(2tig+1), c(2tig), c(2tig+1)} per n-tile and group
    __syncwarp();
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int s = 0; s < NBG; ++s) {
            float sum = 0.f;
#pragma unroll
            for (int cc = 0; cc < D / 32 / NBG; ++cc) {
                const uint4 w = qf[nt][s * (D / 32 / NBG) + cc];
                const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&ww[k]));
                    sum += f.x + f.y;
                }
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            if (tig == 0) {
                float* c = cw + ((s * 4 + (g >> 1)) * NT + nt) * 4;
                c[g & 1] = -1152.f * sum;
                c[2 + (g & 1)] = -1152.f * sum;
            }
        }
    __syncwarp();
}

// One 16-token tile (already in shared memory at T) into the warp's running softmax state.
template <int D, int NB, int NT, bool TREE = false>
__device__ __forceinline__ void tile_math(const uint8_t* T, int kt, const uint4 (&qf)[NT][D / 32],
                                          const int (&kvlen)[NT][2], int kv_min, const float* cw,
                                          float scale_log2, WarpAcc<D, NT>& a, int lane, const TreeCtx& tc) {
    constexpr int KS_OFF = 16 * D;
    constexpr int V_OFF = 16 * D + 32 * NB;
    constexpr int VS_OFF = 32 * D + 32 * NB;
    constexpr int CH = D / 32;
    constexpr int CPG = CH / NB;
    constexpr int MT = D / 16;
    constexpr int MPG = MT / NB;
    static_assert(MPG % 2 == 0, "m-tiles come in pairs per 16-byte V word");
    const int g = lane >> 2, tig = lane & 3;

    // ---- K scales of tokens g and g+8
    float ks0[NB], ks1[NB];
    if constexpr (NB == 1) {
        const uint32_t w = lds32(T + KS_OFF + 4 * g);
        ks0[0] = h2f((uint16_t)(w & 0xffff));
        ks1[0] = h2f((uint16_t)(w >> 16));
    } else {
#pragma unroll
        for (int q4 = 0; q4 < NB / 4; ++q4) {
            const uint4 w = lds128(T + KS_OFF + 4 * NB * g + 16 * q4);
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int idx = q4 * 8 + k;  // f16 index within the lane's 2*NB values
                const float v = h2f((uint16_t)((ww[k / 2] >> (16 * (k & 1))) & 0xffff));
                if (idx < NB)
                    ks0[idx] = v;
                else
                    ks1[idx - NB] = v;
            }
        }
    }
    // ---- S^T = K Q^T, per scale group
    float sacc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) sacc[nt][e] = 0.f;
#pragma unroll
    for (int s = 0; s < NB; ++s) {
        float acc[NT][4];
        if constexpr (kbias_in_acc<NT>()) {
            uint4 cst[NT];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) cst[nt] = lds128(cw + ((s * 4 + tig) * NT + nt) * 4);
#pragma unroll
            for (int cc = 0; cc < CPG; ++cc) {
                const int cb = s * CPG + cc;
                const uint4 kw = lds128(T + cb * 512 + lane * 16);
                const uint32_t x0 = kw.x, x1 = kw.y, z0 = kw.z, z1 = kw.w;
                uint32_t a0 = s8lo_to_h2_biased(x0), a1 = s8lo_to_h2_biased(z0), a2 = s8hi_to_h2_biased(x0),
                         a3 = s8hi_to_h2_biased(z0);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    if (cc == 0)
                        mma_init(acc[nt], a0, a1, a2, a3, qf[nt][cb].x, qf[nt][cb].y, cst[nt]);
                    else
                        mma_acc(acc[nt], a0, a1, a2, a3, qf[nt][cb].x, qf[nt][cb].y);
                }
                a0 = s8lo_to_h2_biased(x1);
                a1 = s8lo_to_h2_biased(z1);
                a2 = s8hi_to_h2_biased(x1);
                a3 = s8hi_to_h2_biased(z1);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) mma_acc(acc[nt], a0, a1, a2, a3, qf[nt][cb].z, qf[nt][cb].w);
            }
        } else {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
#pragma unroll
            for (int cc = 0; cc < CPG; ++cc) {
                const int cb = s * CPG + cc;
                const uint4 kw = lds128(T + cb * 512 + lane * 16);
                const uint32_t x0 = kw.x, x1 = kw.y, z0 = kw.z, z1 = kw.w;
                uint32_t a0 = s8lo_to_h2(x0), a1 = s8lo_to_h2(z0), a2 = s8hi_to_h2(x0), a3 = s8hi_to_h2(z0);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) mma16816(acc[nt], a0, a1, a2, a3, qf[nt][cb].x, qf[nt][cb].y);
                a0 = s8lo_to_h2(x1);
                a1 = s8lo_to_h2(z1);
                a2 = s8hi_to_h2(x1);
                a3 = s8hi_to_h2(z1);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) mma16816(acc[nt], a0, a1, a2, a3, qf[nt][cb].z, qf[nt][cb].w);
            }
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            sacc[nt][0] = fmaf(ks0[s], acc[nt][0], sacc[nt][0]);
            sacc[nt][1] = fmaf(ks0[s], acc[nt][1], sacc[nt][1]);
            sacc[nt][2] = fmaf(ks1[s], acc[nt][2], sacc[nt][2]);
            sacc[nt][3] = fmaf(ks1[s], acc[nt][3], sacc[nt][3]);
        }
    }
    // ---- online softmax (base 2) on rows 2tig, 2tig+1 of each n-tile.  The running max m of a
    // row only moves when the tile's max exceeds it by kRescaleThresh, so the exact row max
    // (shuffles across the row's 8 lanes) and the O rescale are needed only when some lane's
    // own values cross that bound: one vote per tile decides.
    const int tok0 = kt * kTileTokens + g, tok1 = tok0 + 8;
    float v[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) v[nt][e] = sacc[nt][e] * scale_log2;
    if (kt * kTileTokens + kTileTokens > kv_min) {  // some row ends inside this tile (warp-uniform)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int col = 0; col < 2; ++col) {
                if (tok0 >= kvlen[nt][col]) v[nt][col] = -INFINITY;
                if (tok1 >= kvlen[nt][col]) v[nt][2 + col] = -INFINITY;
                if constexpr (TREE) {
                    // kvlen[] > 0 only for real rows; draft keys j = tok - kv0 < kvlen - kv0 <= 64
                    if (kvlen[nt][col] > 0) {
                        const unsigned long long anc = tc.anc[(tc.row0 + nt * 8 + 2 * tig + col) / tc.G];
                        if (tok0 >= tc.kv0 && tok0 < kvlen[nt][col] && !((anc >> (tok0 - tc.kv0)) & 1ull))
                            v[nt][col] = -INFINITY;
                        if (tok1 >= tc.kv0 && tok1 < kvlen[nt][col] && !((anc >> (tok1 - tc.kv0)) & 1ull))
                            v[nt][2 + col] = -INFINITY;
                    }
                }
            }
    }
    bool need = false;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int col = 0; col < 2; ++col)
            need |= fmaxf(v[nt][col], v[nt][2 + col]) > a.m[nt][col] + kRescaleThresh;
    if (__any_sync(0xffffffffu, need)) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            float alpha[2];
#pragma unroll
            for (int col = 0; col < 2; ++col) {
                float mx = fmaxf(v[nt][col], v[nt][2 + col]);
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                alpha[col] = 1.f;
                if (mx > a.m[nt][col] + kRescaleThresh) {
                    // a.m == -inf gives alpha = exp2(-inf) = 0: nothing accumulated yet
                    alpha[col] = fast_exp2(a.m[nt][col] - mx);
                    a.m[nt][col] = mx;
                    a.l[nt][col] *= alpha[col];
                }
            }
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                a.o[mt][nt][0] *= alpha[0];
                a.o[mt][nt][2] *= alpha[0];
                a.o[mt][nt][1] *= alpha[1];
                a.o[mt][nt][3] *= alpha[1];
            }
        }
    }
    uint32_t pb01[NT], pb23[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        float pr[2][2];
#pragma unroll
        for (int col = 0; col < 2; ++col) {
            const float muse = a.m[nt][col] == -INFINITY ? 0.f : a.m[nt][col];
            pr[col][0] = fast_exp2(v[nt][col] - muse);
            pr[col][1] = fast_exp2(v[nt][2 + col] - muse);
            a.l[nt][col] += pr[col][0] + pr[col][1];
        }
        // P^T B-fragment: lane (g, tig) needs P[tok 2tig, 2tig+8][row g] and
        // P[tok 2tig+1, 2tig+9][row g]; lane (g', tig') holds tokens g', g'+8 of
        // rows 2tig', 2tig'+1.
        const uint32_t X = pack_h2(pr[0][0], pr[0][1]);
        const uint32_t Y = pack_h2(pr[1][0], pr[1][1]);
        const int src0 = (2 * tig) * 4 + (g >> 1), src1 = src0 + 4;
        const uint32_t x0 = __shfl_sync(0xffffffffu, X, src0);
        const uint32_t y0 = __shfl_sync(0xffffffffu, Y, src0);
        const uint32_t x1 = __shfl_sync(0xffffffffu, X, src1);
        const uint32_t y1 = __shfl_sync(0xffffffffu, Y, src1);
        pb01[nt] = (g & 1) ? y0 : x0;
        pb23[nt] = (g & 1) ? y1 : x1;
    }
    // ---- O^T += V^T P^T with the V group scales folded into P
#pragma unroll
    for (int s = 0; s < NB; ++s) {
        const uint2 vsw = lds64(T + VS_OFF + (tig * NB + s) * 8);
        uint32_t b0[NT], b1[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            b0[nt] = h2mul(pb01[nt], vsw.x);
            b1[nt] = h2mul(pb23[nt], vsw.y);
        }
#pragma unroll
        for (int mp = 0; mp < MPG / 2; ++mp) {
            const int mt0 = s * MPG + 2 * mp;
            const uint4 vw = lds128(T + V_OFF + (mt0 / 2) * 512 + lane * 16);
            uint32_t w0 = vw.x, w1 = vw.y;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
                mma16816(a.o[mt0][nt], s8lo_to_h2(w0), s8lo_to_h2(w1), s8hi_to_h2(w0), s8hi_to_h2(w1), b0[nt], b1[nt]);
            w0 = vw.z;
            w1 = vw.w;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
                mma16816(a.o[mt0 + 1][nt], s8lo_to_h2(w0), s8lo_to_h2(w1), s8hi_to_h2(w0), s8hi_to_h2(w1), b0[nt],
                         b1[nt]);
        }
    }
}

// ---- per-warp tile stream -----------------------------------------------------------------

// A warp's ring of tile stages.  The warp's n-th tile overall goes to slot n % STAGES with
// phase (n / STAGES) & 1, so the ring continues across units without re-initialisation.
template <int TB, int STAGES>
struct TileRing {
    uint64_t* bar;
    uint8_t* stage;
    uint8_t* flag;
    int base;  // tiles this warp consumed before the current run

    __device__ __forceinline__ void init(uint8_t* smem_hdr, uint8_t* smem_stages, int warp, int lane) {
        bar = reinterpret_cast<uint64_t*>(smem_hdr) + warp * STAGES;
        flag = smem_hdr + kWarps * STAGES * 8 + warp * STAGES;
        stage = smem_stages + (size_t)warp * STAGES * TB;
        base = 0;
        if (lane == 0) {
#pragma unroll
            for (int s = 0; s < STAGES; ++s) mbar_init(&bar[s], 1);
            fence_mbar_init();
        }
        __syncwarp();
    }

    // lane 0 only: copy the tile at `src` (null = a page id past the pool) into run position i.
    __device__ __forceinline__ void issue(int i, const uint8_t* src, uint32_t* status) {
        const int slot = (base + i) % STAGES;
        if (src) {
            flag[slot] = 1;
            mbar_arrive_expect_tx(&bar[slot], TB);
            bulk_g2s(stage + slot * TB, src, TB, &bar[slot]);
        } else {
            flag[slot] = 0;
            atomicOr(status, YF_DEV_BAD_PAGE);
            mbar_arrive(&bar[slot]);
        }
    }
};

// Streams tiles t0 + warp + 4i (i < this warp's share of n_seg tiles) of unit (b, h) through
// the warp's ring into `a`.  A bounded wait that gives up flags YF_DEV_TIMEOUT.
template <int D, int NB, int NT, int TPP, int STAGES, bool TREE = false>
__device__ __forceinline__ void stream_unit(const SplitParams& p, TileRing<32 * D + 64 * NB, STAGES>& ring, int b,
                                            int h, int t0, int n_seg, const uint4 (&qf)[NT][D / 32],
                                            const int (&kvlen)[NT][2], int kv_min, const float* cw,
                                            WarpAcc<D, NT>& a, int warp, int lane, const TreeCtx& tc) {
    constexpr int TB = 32 * D + 64 * NB;
    const int my_n = n_seg > warp ? (n_seg - warp + kWarps - 1) / kWarps : 0;
    const uint32_t* btrow = p.bt + (size_t)b * p.max_blocks;
    const uint8_t* head_base = p.layer_base + (size_t)h * p.phb;
    const long long page_stride = p.phb * p.H;
    auto tile_of = [&](int i) { return t0 + warp + i * kWarps; };
    auto src_of = [&](int kt, uint32_t page) -> const uint8_t* {
        return page < (uint32_t)p.n_pages ? head_base + (size_t)page * page_stride + (kt % TPP) * TB : nullptr;
    };
    uint32_t next_page = 0;  // lane 0: page id of the next tile to issue, loaded one tile ahead
    if (lane == 0) {
        for (int s = 0; s < STAGES && s < my_n; ++s)
            ring.issue(s, src_of(tile_of(s), __ldg(btrow + tile_of(s) / TPP)), p.status);
        if (STAGES < my_n) next_page = __ldg(btrow + tile_of(STAGES) / TPP);
    }
    __syncwarp();
    int done = 0;
    bool ok = true;
    for (int i = 0; i < my_n; ++i) {
        const int pos = ring.base + i;
        const int slot = pos % STAGES;
        if (!__all_sync(0xffffffffu, mbar_wait(&ring.bar[slot], (uint32_t)(pos / STAGES) & 1u, p.wait_ns))) {
            if (lane == 0) atomicOr(p.status, YF_DEV_TIMEOUT);
            ok = false;
            break;
        }
        done = i + 1;
        if (ring.flag[slot])
            tile_math<D, NB, NT, TREE>(ring.stage + slot * TB, tile_of(i), qf, kvlen, kv_min, cw, p.scale_log2, a,
                                       lane, tc);
        __syncwarp();
        if (lane == 0 && i + STAGES < my_n) {
            ring.issue(i + STAGES, src_of(tile_of(i + STAGES), next_page), p.status);
            if (i + STAGES + 1 < my_n) next_page = __ldg(btrow + tile_of(i + STAGES + 1) / TPP);
        }
    }
    if (!ok) {  // wait (bounded) for the copies still in flight before the ring is reused
        for (int i = done; i < my_n && i < done + STAGES; ++i)
            (void)mbar_wait(&ring.bar[(ring.base + i) % STAGES], (uint32_t)((ring.base + i) / STAGES) & 1u, p.wait_ns);
    }
    ring.base += my_n;
}

// ---- 4-warp merge --------------------------------------------------------------------------

// Writes each warp's (m, l, O) to shared memory (reusing the stage area: every copy of the
// CTA is complete once all warps arrive) and synchronises the CTA.
template <int D, int NT>
__device__ __forceinline__ void stash_warp(uint8_t* area, WarpAcc<D, NT>& a, int warp, int lane) {
    constexpr int RPC = 8 * NT, DP = D + 4;
    const int g = lane >> 2, tig = lane & 3;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int col = 0; col < 2; ++col) {
            float l = a.l[nt][col];
            l += __shfl_xor_sync(0xffffffffu, l, 4);
            l += __shfl_xor_sync(0xffffffffu, l, 8);
            l += __shfl_xor_sync(0xffffffffu, l, 16);
            a.l[nt][col] = l;
        }
    __syncthreads();  // every warp is done reading its stages
    float* mw = reinterpret_cast<float*>(area);
    float* lw = mw + kWarps * RPC;
    float* ow = lw + kWarps * RPC;
    if (g == 0) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int col = 0; col < 2; ++col) {
                mw[warp * RPC + nt * 8 + 2 * tig + col] = a.m[nt][col];
                lw[warp * RPC + nt * 8 + 2 * tig + col] = a.l[nt][col];
            }
    }
#pragma unroll
    for (int mt = 0; mt < D / 16; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int r = nt * 8 + 2 * tig + (e & 1);
                const int d = 16 * mt + g + 8 * (e >> 1);
                ow[(warp * RPC + r) * DP + d] = a.o[mt][nt][e];
            }
    __syncthreads();
}

// Merges the stashed warps of one unit: f16 output when `direct`, else the normalised
// partial O and base-2 lse into workspace item `item`.
template <int D, int NT>
__device__ __forceinline__ void emit_unit(const SplitParams& p, const UnitGeom& u, int h, const uint8_t* area,
                                          bool direct, size_t item) {
    constexpr int RPC = 8 * NT, DP = D + 4;
    const float* mw = reinterpret_cast<const float*>(area);
    const float* lw = mw + kWarps * RPC;
    const float* ow = lw + kWarps * RPC;
    for (int e = threadIdx.x; e < RPC * (D / 4); e += kThreads) {
        const int r = e / (D / 4), d4 = (e % (D / 4)) * 4;
        const int row = u.row_begin + r;
        if (row >= u.rows_total) continue;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, mw[w * RPC + r]);
        float L = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            const float mv = mw[w * RPC + r];
            if (mv == -INFINITY) continue;
            const float f = fast_exp2(mv - M);
            L = fmaf(f, lw[w * RPC + r], L);
            const float4 ov = *reinterpret_cast<const float4*>(&ow[(w * RPC + r) * DP + d4]);
            acc.x = fmaf(f, ov.x, acc.x);
            acc.y = fmaf(f, ov.y, acc.y);
            acc.z = fmaf(f, ov.z, acc.z);
            acc.w = fmaf(f, ov.w, acc.w);
        }
        const float inv = L > 0.f ? 1.f / L : 0.f;
        acc.x *= inv;
        acc.y *= inv;
        acc.z *= inv;
        acc.w *= inv;
        if (direct) {
            store_row4(p, u, h, row, d4, D, acc, L > 0.f ? M + __log2f(L) : -INFINITY);
        } else {
            *reinterpret_cast<float4*>(p.ws_o + (item * RPC + r) * D + d4) = acc;
            if (d4 == 0) p.ws_lse[item * RPC + r] = L > 0.f ? M + __log2f(L) : -INFINITY;
        }
    }
}

// Merges n partials (items item_of(0..n-1)) of one unit into f16 output; loads through L2
// (the partials were written by other CTAs).
template <int D, int RPC, typename ItemOf>
__device__ __forceinline__ void combine_items(const SplitParams& p, const UnitGeom& u, int h, int n, ItemOf item_of) {
    for (int e = threadIdx.x; e < RPC * (D / 4); e += kThreads) {
        const int r = e / (D / 4), d4 = (e % (D / 4)) * 4;
        const int row = u.row_begin + r;
        if (row >= u.rows_total) continue;
        float M = -INFINITY;
        for (int c = 0; c < n; ++c) M = fmaxf(M, __ldcg(p.ws_lse + item_of(c) * RPC + r));
        float L = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int c = 0; c < n; ++c) {
            const size_t it = item_of(c);
            const float lv = __ldcg(p.ws_lse + it * RPC + r);
            if (lv == -INFINITY) continue;
            const float f = fast_exp2(lv - M);
            L += f;
            const float4 ov = __ldcg(reinterpret_cast<const float4*>(p.ws_o + (it * RPC + r) * D + d4));
            acc.x = fmaf(f, ov.x, acc.x);
            acc.y = fmaf(f, ov.y, acc.y);
            acc.z = fmaf(f, ov.z, acc.z);
            acc.w = fmaf(f, ov.w, acc.w);
        }
        const float inv = L > 0.f ? 1.f / L : 0.f;
        store_row4(p, u, h, row, d4, D, make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv),
                   L > 0.f ? M + __log2f(L) : -INFINITY);
    }
}

// Merges n partials of one unit (workspace items item_of(0..n-1)) in three parallel phases:
// every lse is loaded at once, turned into normalised per-row weights in shared memory (wsm:
// n*RPC + RPC floats), then each thread accumulates its O elements with independent loads.
// Writes f16 output when dst_item < 0, else a partial (normalised O, base-2 lse) into
// dst_item, which may be one of the inputs (each element is read before it is written, by
// the same thread).
template <int D, int RPC, typename ItemOf>
__device__ __forceinline__ void merge_parts(const SplitParams& p, const UnitGeom& u, int h, int n, ItemOf item_of,
                                            float* wsm, long long dst_item) {
    float* w = wsm;
    float* lse_out = wsm + n * RPC;
    for (int idx = threadIdx.x; idx < n * RPC; idx += kThreads)
        w[idx] = __ldcg(p.ws_lse + item_of(idx / RPC) * RPC + idx % RPC);
    __syncthreads();
    for (int r = threadIdx.x; r < RPC; r += kThreads) {
        float M = -INFINITY;
        for (int k = 0; k < n; ++k) M = fmaxf(M, w[k * RPC + r]);
        float L = 0.f;
        for (int k = 0; k < n; ++k) {
            const float lv = w[k * RPC + r];
            const float f = lv == -INFINITY ? 0.f : fast_exp2(lv - M);
            w[k * RPC + r] = f;
            L += f;
        }
        const float inv = L > 0.f ? 1.f / L : 0.f;
        for (int k = 0; k < n; ++k) w[k * RPC + r] *= inv;
        lse_out[r] = L > 0.f ? M + __log2f(L) : -INFINITY;
    }
    __syncthreads();
    // every thread owns EPT float4 elements; per batch of PB parts it issues all EPT*PB loads
    // before the first use, so the merge pays a few L2 round trips, not one per part
    constexpr int EPT = (RPC * (D / 4) + kThreads - 1) / kThreads;
    constexpr int PB = EPT >= 4 ? 2 : 4;
    float4 acc[EPT];
    bool live[EPT];
    size_t eoff[EPT];
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
        const int e = threadIdx.x + i * kThreads;
        const int r = e / (D / 4), d4 = (e % (D / 4)) * 4;
        live[i] = e < RPC * (D / 4) && u.row_begin + r < u.rows_total;
        eoff[i] = (size_t)r * D + d4;
        acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int k0 = 0; k0 < n; k0 += PB) {
        float4 ov[EPT][PB];
#pragma unroll
        for (int j = 0; j < PB; ++j) {
            const size_t base = k0 + j < n ? item_of(k0 + j) * RPC * D : 0;
#pragma unroll
            for (int i = 0; i < EPT; ++i)
                ov[i][j] = (live[i] && k0 + j < n) ? __ldcg(reinterpret_cast<const float4*>(p.ws_o + base + eoff[i]))
                                                   : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int j = 0; j < PB; ++j) {
            if (k0 + j >= n) break;
#pragma unroll
            for (int i = 0; i < EPT; ++i) {
                const int r = (threadIdx.x + i * kThreads) / (D / 4);
                const float f = live[i] ? w[(k0 + j) * RPC + r] : 0.f;
                acc[i].x = fmaf(f, ov[i][j].x, acc[i].x);
                acc[i].y = fmaf(f, ov[i][j].y, acc[i].y);
                acc[i].z = fmaf(f, ov[i][j].z, acc[i].z);
                acc[i].w = fmaf(f, ov[i][j].w, acc[i].w);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
        if (!live[i]) continue;
        const int e = threadIdx.x + i * kThreads;
        const int r = e / (D / 4), d4 = (e % (D / 4)) * 4;
        if (dst_item < 0) {
            store_row4(p, u, h, u.row_begin + r, d4, D, acc[i], lse_out[r]);
        } else {
            __stcg(reinterpret_cast<float4*>(p.ws_o + (size_t)dst_item * RPC * D + eoff[i]), acc[i]);
        }
    }
    if (dst_item >= 0)
        for (int r = threadIdx.x; r < RPC; r += kThreads) __stcg(p.ws_lse + (size_t)dst_item * RPC + r, lse_out[r]);
}

// Counts this CTA's arrival on counter `ctr` (one of `n_arrivals`); true for the last one,
// which then owns the merge and resets the counter.
__device__ __forceinline__ bool arrive_last(uint32_t* ctr, int n_arrivals, int* s_flag) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) *s_flag = atomicAdd(ctr, 1u) == (uint32_t)n_arrivals - 1;
    __syncthreads();
    const bool last = *s_flag;
    if (last) __threadfence();
    return last;
}

// Single-level merge: the last of the unit's n_parts arrivals merges every part into the output.
template <int D, int RPC, typename ItemOf>
__device__ __forceinline__ void arrive_and_merge(const SplitParams& p, const UnitGeom& u, int h, size_t unit,
                                                 int n_parts, ItemOf item_of, float* wsm, int* s_flag) {
    if (!arrive_last(&p.counters[unit], n_parts, s_flag)) return;
    merge_parts<D, RPC>(p, u, h, n_parts, item_of, wsm, -1);
    if (threadIdx.x == 0) p.counters[unit] = 0;  // ready for the next call on this pool
}

// ---- cooperative merge of the persistent schedule ------------------------------------------
// Every CTA of a split unit arrives on the unit's counter (low 16 bits); the CTAs whose range
// ends inside the unit then wait for all of the unit's parts and merge one slice each of the
// unit's output columns (all of a slice's loads in flight at once), and count their
// departure (high 16 bits); the last to leave resets the counter for the next call.  A CTA
// that goes on to the next unit only arrives.  The grid is a single resident wave, so the
// waits end; each is bounded by the call's wait limit and flags YF_DEV_TIMEOUT if it gives up.

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* ptr) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
    return v;
}

// Online merge of one (base-2 lse, normalised O) part into (m, l, o).
__device__ __forceinline__ void merge_in(float lv, float4 ov, float& m, float& l, float4& o) {
    if (lv == -INFINITY) return;
    if (lv > m) {
        const float f = m == -INFINITY ? 0.f : fast_exp2(m - lv);
        l *= f;
        o.x *= f;
        o.y *= f;
        o.z *= f;
        o.w *= f;
        m = lv;
    }
    const float w = fast_exp2(lv - m);
    l += w;
    o.x = fmaf(w, ov.x, o.x);
    o.y = fmaf(w, ov.y, o.y);
    o.z = fmaf(w, ov.z, o.z);
    o.w = fmaf(w, ov.w, o.w);
}

// Slice `slice` of `n_slices` of the unit's RPC x D/4 output columns (float4), merged over the
// n parts whose workspace items are items[0..n-1].
template <int D, int RPC>
__device__ __forceinline__ void merge_slice(const SplitParams& p, const UnitGeom& u, int h, int n,
                                            const uint32_t* items, int slice, int n_slices) {
    constexpr int COLS = RPC * (D / 4);
    constexpr int PB = 8;  // parts per lane (or thread) loaded together
    const int c0 = (int)((long long)slice * COLS / n_slices), c1 = (int)((long long)(slice + 1) * COLS / n_slices);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    if (n >= 32) {
        // a warp per column, its lanes over the parts, then the lanes' states merged
        for (int col = c0 + warp; col < c1; col += kWarps) {
            const int r = col / (D / 4), d4 = (col % (D / 4)) * 4;
            if (u.row_begin + r >= u.rows_total) continue;
            float m = -INFINITY, l = 0.f;
            float4 o = zero;
            for (int k0 = lane; k0 < n; k0 += 32 * PB) {
                float lv[PB];
                float4 ov[PB];
#pragma unroll
                for (int j = 0; j < PB; ++j) {
                    const int k = k0 + 32 * j;
                    lv[j] = -INFINITY;
                    ov[j] = zero;
                    if (k < n) {
                        const size_t it = items[k];
                        lv[j] = __ldcg(p.ws_lse + it * RPC + r);
                        ov[j] = __ldcg(reinterpret_cast<const float4*>(p.ws_o + (it * RPC + r) * D + d4));
                    }
                }
#pragma unroll
                for (int j = 0; j < PB; ++j) merge_in(lv[j], ov[j], m, l, o);
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
                const float l2 = __shfl_xor_sync(0xffffffffu, l, off);
                float4 o2;
                o2.x = __shfl_xor_sync(0xffffffffu, o.x, off);
                o2.y = __shfl_xor_sync(0xffffffffu, o.y, off);
                o2.z = __shfl_xor_sync(0xffffffffu, o.z, off);
                o2.w = __shfl_xor_sync(0xffffffffu, o.w, off);
                const float M = fmaxf(m, m2);
                if (M != -INFINITY) {
                    const float f1 = m == -INFINITY ? 0.f : fast_exp2(m - M);
                    const float f2 = m2 == -INFINITY ? 0.f : fast_exp2(m2 - M);
                    l = l * f1 + l2 * f2;
                    o.x = o.x * f1 + o2.x * f2;
                    o.y = o.y * f1 + o2.y * f2;
                    o.z = o.z * f1 + o2.z * f2;
                    o.w = o.w * f1 + o2.w * f2;
                    m = M;
                }
            }
            if (lane == 0) {
                const float inv = l > 0.f ? 1.f / l : 0.f;
                store_row4(p, u, h, u.row_begin + r, d4, D, make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv),
                           l > 0.f ? m + __log2f(l) : -INFINITY);
            }
        }
    } else {
        // a thread per column, over every part
        for (int col = c0 + threadIdx.x; col < c1; col += kThreads) {
            const int r = col / (D / 4), d4 = (col % (D / 4)) * 4;
            if (u.row_begin + r >= u.rows_total) continue;
            float m = -INFINITY, l = 0.f;
            float4 o = zero;
            for (int k0 = 0; k0 < n; k0 += PB) {
                float lv[PB];
                float4 ov[PB];
#pragma unroll
                for (int j = 0; j < PB; ++j) {
                    lv[j] = -INFINITY;
                    ov[j] = zero;
                    if (k0 + j < n) {
                        const size_t it = items[k0 + j];
                        lv[j] = __ldcg(p.ws_lse + it * RPC + r);
                        ov[j] = __ldcg(reinterpret_cast<const float4*>(p.ws_o + (it * RPC + r) * D + d4));
                    }
                }
#pragma unroll
                for (int j = 0; j < PB; ++j) merge_in(lv[j], ov[j], m, l, o);
            }
            const float inv = l > 0.f ? 1.f / l : 0.f;
            store_row4(p, u, h, u.row_begin + r, d4, D, make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv),
                       l > 0.f ? m + __log2f(l) : -INFINITY);
        }
    }
}

template <int D, int RPC, typename ItemOf>
__device__ __forceinline__ void cooperative_merge(const SplitParams& p, const UnitGeom& u, int h, size_t unit,
                                                  int n_parts, ItemOf item_of, bool merger, int slice, int n_slices,
                                                  uint32_t* s_items, int* s_flag) {
    uint32_t* ctr = &p.counters[unit];
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) atomicAdd(ctr, 1u);
    if (!merger) return;
    if (threadIdx.x == 0) {
        bool ok = true;
        if ((ld_acquire_u32(ctr) & 0xFFFFu) < (uint32_t)n_parts) {
            const uint64_t t0 = globaltimer_ns();
            for (uint32_t i = 0;; ++i) {
                if ((ld_acquire_u32(ctr) & 0xFFFFu) >= (uint32_t)n_parts) break;
                if ((i & 63u) == 63u && globaltimer_ns() - t0 > p.wait_ns) {
                    ok = false;
                    break;
                }
                __nanosleep(32);
            }
        }
        if (!ok) atomicOr(p.status, YF_DEV_TIMEOUT);
        *s_flag = ok;
    }
    for (int k = threadIdx.x; k < n_parts; k += kThreads) s_items[k] = (uint32_t)item_of(k);
    __syncthreads();
    __threadfence();
    if (*s_flag) merge_slice<D, RPC>(p, u, h, n_parts, s_items, slice, n_slices);
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t old = atomicAdd(ctr, 0x10000u);
        if ((old >> 16) == (uint32_t)n_slices - 1) atomicExch(ctr, 0u);  // the last merger leaves
    }
}

// ---- schedule 1: persistent, equal contiguous ranges of (unit, tile) ------------------------

// Resident CTAs per SM the register allocation must allow (the wide variants would
// otherwise take ~200 registers and fit only 2).
template <int D, int NT>
constexpr int min_ctas() { return (D == 128 && NT == 1) ? 4 : 3; }

template <int D, int NB, int NT, int TPP, int STAGES>
__global__ void __launch_bounds__(kThreads, min_ctas<D, NT>()) decode_persistent_kernel(const SplitParams p) {
    constexpr int TB = 32 * D + 64 * NB;
    constexpr int RPC = 8 * NT;
    constexpr int DP = D + 4;
    static_assert(kHdrBytes >= kWarps * STAGES * 9, "header area too small");
    static_assert(kWarps * STAGES * TB >= 2 * kWarps * RPC * 4 + kWarps * RPC * DP * 4, "merge area too small");
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* stages = smem + hdr_bytes<NB, NT>();
    long long* sP = reinterpret_cast<long long*>(stages + kWarps * STAGES * TB);  // [B+1] tile prefix
    __shared__ int s_last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = p.H, B = p.B;

    // Tiles per head of every entry and their prefix over (entry, head): unit (b, h) owns the
    // linear tiles [sP[b] + h*E_b, sP[b] + (h+1)*E_b), E_b = (sP[b+1]-sP[b]) / H.
    if (warp == 0) {
        long long carry = 0;
        for (int base = 0; base < B; base += 32) {
            const int b = base + lane;
            long long e = 0;
            UnitGeom u;
            if (b < B && unit_geom<TPP, RPC>(p, b, 0, u, blockIdx.x == 0)) e = u.n_tiles;
            long long v = e;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const long long t = __shfl_up_sync(0xffffffffu, v, off);
                if (lane >= off) v += t;
            }
            if (b < B) sP[b] = (carry + v - e) * H;
            carry += __shfl_sync(0xffffffffu, v, 31);
        }
        if (lane == 0) sP[B] = carry * H;
    }
    __syncthreads();
    const long long T = sP[B];
    // N <= T: every CTA of the partition owns at least one tile, so the CTAs that meet a unit
    // are exactly the parts its merge counts
    const long long N = T < (long long)gridDim.x ? T : (long long)gridDim.x;
    const bool in_partition = (long long)blockIdx.x < N;
    const long long s = in_partition ? (long long)blockIdx.x * T / N : 0;
    const long long e_end = in_partition ? ((long long)blockIdx.x + 1) * T / N : 0;
    auto start_of = [&](long long c) { return c * T / N; };
    auto cta_of = [&](long long x) { return ((x + 1) * N - 1) / T; };  // largest c with start_of(c) <= x

    // Entries without keys get zero rows (no tile belongs to them).
    for (int b = blockIdx.x; b < B; b += gridDim.x) {
        if (sP[b + 1] != sP[b]) continue;
        UnitGeom u;
        if (!unit_geom<TPP, RPC>(p, b, 0, u, false)) continue;
        for (int e = threadIdx.x; e < u.rows_total * H * (D / 4); e += kThreads) {
            const int d4 = (e % (D / 4)) * 4, rh = e / (D / 4);
            const int row = rh % u.rows_total, h = rh / u.rows_total;
            store_row4(p, u, h, row, d4, D, make_float4(0.f, 0.f, 0.f, 0.f), -INFINITY);
        }
    }
    if (s >= e_end) return;

    TileRing<TB, STAGES> ring;
    ring.init(smem, stages, warp, lane);
    WarpAcc<D, NT> acc;
    uint4 qf[NT][D / 32];
    int kvlen[NT][2], kv_min;

    long long x = s;
    while (x < e_end) {
        // entry of linear tile x: the largest b with sP[b] <= x (entries without tiles have
        // sP[b] == sP[b+1], so the search passes over them)
        int lo = 0, hi = B - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (sP[mid] <= x)
                lo = mid;
            else
                hi = mid - 1;
        }
        const int b = lo;
        const long long E = (sP[b + 1] - sP[b]) / H;
        const long long off = x - sP[b];
        const int h = (int)(off / E);
        const int t0 = (int)(off % E);
        const long long Us = sP[b] + (long long)h * E, Ue = Us + E;
        const long long seg_e = e_end < Ue ? e_end : Ue;
        UnitGeom u;
        unit_geom<TPP, RPC>(p, b, 0, u, false);
        load_unit_q<D, NT, NB>(p, u, h, lane, qf, kvlen, kv_min, kbias_area<NB, NT>(smem, warp));
        acc.reset();
        stream_unit<D, NB, NT, TPP, STAGES>(p, ring, b, h, t0, (int)(seg_e - x), qf, kvlen, kv_min,
                                            kbias_area<NB, NT>(smem, warp), acc, warp, lane, TreeCtx{});
        stash_warp<D, NT>(stages, acc, warp, lane);
        const bool whole = x == Us && seg_e == Ue;
        // partial slots: 2 per CTA; slot 1 when the CTA began inside an earlier unit
        const size_t item = (size_t)blockIdx.x * 2 + (s < Us ? 1 : 0);
        emit_unit<D, NT>(p, u, h, stages, whole, item);
        if (!whole) {
            const long long c_lo = cta_of(Us), c_hi = cta_of(Ue - 1);
            // partial slot of part k (CTA c_lo + k): only the unit's first CTA can have begun
            // inside an earlier unit (slot 1)
            const size_t item0 = (size_t)c_lo * 2 + (start_of(c_lo) < Us ? 1 : 0);
            auto item_of = [&](int k) -> size_t { return k == 0 ? item0 : (size_t)(c_lo + k) * 2; };
            // mergers: the unit's CTAs whose range ends inside it (all but c_hi, and c_hi too when
            // its range ends exactly at the unit's end)
            const long long p_hi = start_of(c_hi + 1) == Ue ? c_hi : c_hi - 1;
            cooperative_merge<D, RPC>(p, u, h, (size_t)b * H + h, (int)(c_hi - c_lo + 1), item_of, e_end <= Ue,
                                      (int)(blockIdx.x - c_lo), (int)(p_hi - c_lo + 1),
                                      reinterpret_cast<uint32_t*>(stages), &s_last);
        }
        // the merge area is the next unit's stage area: order its generic accesses before the
        // bulk copies that will overwrite it
        fence_proxy_async_smem();
        __syncthreads();
        x = seg_e;
    }
}

// ---- schedule 3: few long units over thread-block clusters ----------------------------------
//
// For a handful of long units (the long-context decode, a small decode, one rank's shard) every
// unit gets whole clusters of kClusterCtas CTAs; cluster lc of a unit streams tiles
// [lc * tpc, (lc + 1) * tpc) of it, split evenly over its CTAs.  Each CTA merges its 4 warps into
// a normalised partial in its own shared memory; after a cluster barrier, CTA rank r merges
// column slice r of the unit's output over the cluster's CTAs by distributed shared-memory loads.
// A unit held by one cluster writes its output there.  Otherwise each cluster writes its slices
// as a partial and counts an arrival per slice; the CTA that arrives last for slice r merges the
// unit's cluster partials of that slice from L2 and writes the output (its counter back to zero).
// No CTA ever waits for another cluster, so the grid needs no co-residency beyond the cluster,
// which the hardware schedules as one.

template <int D>
constexpr int cluster_part_off() {  // the CTA partial, after the 4-warp stash in the stage area
    return ((2 * kWarps * 8 * 4 + kWarps * 8 * (D + 4) * 4) + 127) / 128 * 128;
}

// The last arrival's merge of slice r (RPC / CL rows) over the unit's n cluster partials, workspace
// items item0 .. item0 + n - 1.  Weights first: warp j < RS takes row j's n lse values, their max
// and w_k = 2^(lse_k - max) (0 for a part without keys) into shared memory, with their sum reduced
// in a fixed lane order.  Then every thread adds w_k o_k of its column over parts k = ph, ph + TPC,
// ... (TPC threads per column), with the loads of an unrolled run of parts in flight together,
// and the TPC shares are added in phase order.  `area` is the CTA's stage area (free again once
// the cluster's reads of this CTA's partial are over).
template <int D, int RPC, int CL>
__device__ __forceinline__ void last_merge(const SplitParams& p, const UnitGeom& u, int h, int r, int n,
                                           size_t item0, uint8_t* area, uint32_t xstep) {
    constexpr int C4 = D / 4;               // float4 columns of a row
    constexpr int SLICE = RPC * C4 / CL;    // float4 columns of a slice
    constexpr int RS = RPC / CL;            // rows of a slice
    constexpr int TPC = kThreads / SLICE;   // threads per column
    static_assert(RPC % CL == 0 && RS <= kWarps && kThreads % SLICE == 0, "slice geometry");
    float* wts = reinterpret_cast<float*>(area);                 // [n][RS]
    float* rowm = wts + kClusterMaxParts * RS;                   // [RS] max lse
    float* rowl = rowm + 4;                                      // [RS] sum of weights
    float4* share = reinterpret_cast<float4*>(rowl + 4);         // [kThreads]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = r * RS;
    if (warp < RS) {
        float M = -INFINITY;
        for (int k = lane; k < n; k += 32) {
            const float lv = __ldcg(p.ws_lse + (item0 + k) * RPC + row0 + warp);
            wts[k * RS + warp] = lv;
            M = fmaxf(M, lv);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float L = 0.f;
        for (int k = lane; k < n; k += 32) {
            const float lv = wts[k * RS + warp];
            const float w = lv == -INFINITY ? 0.f : fast_exp2(lv - M);
            wts[k * RS + warp] = w;
            L += w;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
        if (lane == 0) {
            rowm[warp] = M;
            rowl[warp] = L;
        }
    }
    __syncthreads();
    const int c = threadIdx.x % SLICE, ph = threadIdx.x / SLICE;
    const int col = r * SLICE + c, row = col / C4, d4 = (col % C4) * 4, rr = row - row0;
    const float4* src = reinterpret_cast<const float4*>(p.ws_o) + (item0 * RPC + row) * C4 + col % C4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int k = ph; k < n; k += TPC) {
        const float w = wts[k * RS + rr];
        const float4 v = __ldcg(src + (size_t)k * RPC * C4);
        acc.x = fmaf(w, v.x, acc.x);
        acc.y = fmaf(w, v.y, acc.y);
        acc.z = fmaf(w, v.z, acc.z);
        acc.w = fmaf(w, v.w, acc.w);
    }
    if constexpr (TPC > 1) {
        share[threadIdx.x] = acc;
        __syncthreads();
    }
    if (ph == 0 && u.row_begin + row < u.rows_total) {
#pragma unroll
        for (int q = 1; q < TPC; ++q) {
            const float4 v = share[q * SLICE + c];
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        const float L = rowl[rr], inv = L > 0.f ? 1.f / L : 0.f;
        store_out4(p, u, h, u.row_begin + row, d4, D, make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv),
                   L > 0.f ? rowm[rr] + __log2f(L) : -INFINITY, xstep);
    }
}

template <int D, int NB, int TPP, int STAGES>
__global__ void __cluster_dims__(kClusterCtas, 1, 1) __launch_bounds__(kThreads, 2)  // 2 per SM: kClusterSmemFloor
    decode_cluster_kernel(const SplitParams p) {
    pdl_wait();  // before any global access: the previous kernel (a KV write) has completed
    constexpr int NT = 1, RPC = 8, CL = kClusterCtas;
    constexpr int TB = 32 * D + 64 * NB;
    constexpr int DP = D + 4;
    constexpr int COLS = RPC * (D / 4);  // float4 columns of a unit's output
    constexpr int SLICE = COLS / CL;
    static_assert(SLICE <= kThreads && COLS % CL == 0, "one column per thread in a slice");
    static_assert(cluster_part_off<D>() + RPC * (D + 1) * 4 <= kWarps * STAGES * TB, "partial area");
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* stages = smem + hdr_bytes<NB, NT>();
    float* part_lse = reinterpret_cast<float*>(stages + cluster_part_off<D>());  // [RPC] base-2 lse
    float* part_o = part_lse + RPC;                                               // [RPC][D] normalised
    __shared__ int s_last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = (int)cluster_rank();
    const int cid = blockIdx.x / CL;
    const int cpu = p.max_chunks, tpc = p.chunk_tiles;  // clusters per unit, tiles per cluster
    const int uidx = cid / cpu, lc = cid % cpu;
    const int b = uidx / p.H, h = uidx % p.H;
    UnitGeom u;
    unit_geom<TPP, RPC>(p, b, 0, u, lc == 0 && r == 0 && threadIdx.x == 0);
    const int n_u = max(1, (u.n_tiles + tpc - 1) / tpc);  // clusters this unit uses
    if (lc >= n_u) return;                               // the whole cluster leaves together
    const int c0 = lc * tpc, c1 = min(c0 + tpc, u.n_tiles), len = max(c1 - c0, 0);
    const int t0 = c0 + r * len / CL, t1 = c0 + (r + 1) * len / CL;

    TileRing<TB, STAGES> ring;
    ring.init(smem, stages, warp, lane);
    WarpAcc<D, NT> acc;
    uint4 qf[NT][D / 32];
    int kvlen[NT][2], kv_min;
    load_unit_q<D, NT, NB>(p, u, h, lane, qf, kvlen, kv_min, kbias_area<NB, NT>(smem, warp));
    acc.reset();
    stream_unit<D, NB, NT, TPP, STAGES>(p, ring, b, h, t0, t1 - t0, qf, kvlen, kv_min, kbias_area<NB, NT>(smem, warp),
                                        acc, warp, lane, TreeCtx{});
    stash_warp<D, NT>(stages, acc, warp, lane);
    {  // the 4 warps into this CTA's partial
        const float* mw = reinterpret_cast<const float*>(stages);
        const float* lw = mw + kWarps * RPC;
        const float* ow = lw + kWarps * RPC;
        for (int e = threadIdx.x; e < RPC * (D / 4); e += kThreads) {
            const int row = e / (D / 4), d4 = (e % (D / 4)) * 4;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) M = fmaxf(M, mw[w * RPC + row]);
            float L = 0.f;
            float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int w = 0; w < kWarps; ++w) {
                const float mv = mw[w * RPC + row];
                if (mv == -INFINITY) continue;
                const float f = fast_exp2(mv - M);
                L = fmaf(f, lw[w * RPC + row], L);
                const float4 ov = *reinterpret_cast<const float4*>(&ow[(w * RPC + row) * DP + d4]);
                o.x = fmaf(f, ov.x, o.x);
                o.y = fmaf(f, ov.y, o.y);
                o.z = fmaf(f, ov.z, o.z);
                o.w = fmaf(f, ov.w, o.w);
            }
            const float inv = L > 0.f ? 1.f / L : 0.f;
            *reinterpret_cast<float4*>(&part_o[row * D + d4]) = make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
            if (d4 == 0) part_lse[row] = L > 0.f ? M + __log2f(L) : -INFINITY;
        }
    }
    cluster_barrier();  // every CTA's partial is in its shared memory
    // slice r of the columns, merged over the cluster's CTAs through distributed shared memory
    const int col = r * SLICE + threadIdx.x;
    const int row = col / (D / 4), d4 = (col % (D / 4)) * 4;
    float m = -INFINITY, l = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    if (threadIdx.x < SLICE) {
        float lv[CL];
        float4 ov[CL];
#pragma unroll
        for (int q = 0; q < CL; ++q) {
            lv[q] = ld_dsmem_f32(dsmem_addr(&part_lse[row], q));
            ov[q] = ld_dsmem_f32x4(dsmem_addr(&part_o[row * D + d4], q));
        }
#pragma unroll
        for (int q = 0; q < CL; ++q) merge_in(lv[q], ov[q], m, l, o);
    }
    cluster_barrier();  // no CTA leaves, or reuses its shared memory, while a peer still reads it
    const bool live_row = threadIdx.x < SLICE && u.row_begin + row < u.rows_total;
    // fused exchange: this slice's step (its previous call's + 1; only this CTA role touches it)
    const int xsi = uidx * CL + r;
    const uint32_t xstep = p.x.peers ? reinterpret_cast<const uint32_t*>(p.x.local + p.x.sstep_off)[xsi] + 1u : 0u;
    if (n_u == 1) {
        if (live_row) {
            const float inv = l > 0.f ? 1.f / l : 0.f;
            store_out4(p, u, h, u.row_begin + row, d4, D, make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv),
                       l > 0.f ? m + __log2f(l) : -INFINITY, xstep);
        }
        if (p.x.peers) exchange_finish<D, RPC, CL>(p, u, h, r, xsi, xstep);
        return;
    }
    // this cluster's partial of slice r, then the slice's arrival
    const size_t item = (size_t)uidx * cpu + lc;
    if (threadIdx.x < SLICE) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
        __stcg(reinterpret_cast<float4*>(p.ws_o + (item * RPC + row) * D + d4),
               make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv));
        if (d4 == 0) __stcg(p.ws_lse + item * RPC + row, l > 0.f ? m + __log2f(l) : -INFINITY);
    }
    uint32_t* ctr = &p.counters[(size_t)uidx * CL + r];
    if (!arrive_last(ctr, n_u, &s_last)) return;
    last_merge<D, RPC, CL>(p, u, h, r, n_u, (size_t)uidx * cpu, stages, xstep);
    if (threadIdx.x == 0) *ctr = 0;  // ready for the next call on this pool
    if (p.x.peers) exchange_finish<D, RPC, CL>(p, u, h, r, xsi, xstep);
}

// ---- schedule 2: a 3-D grid of (unit, chunk of tiles) ----------------------------------------

template <int D, int NB, int NT, int TPP, int STAGES, bool TREE = false>
__global__ void __launch_bounds__(kThreads) splitkv_kernel(const SplitParams p) {
    pdl_wait();  // before any global access: the previous kernel (a KV write) has completed
    constexpr int TB = 32 * D + 64 * NB;
    constexpr int RPC = 8 * NT;
    constexpr int DP = D + 4;
    static_assert(kHdrBytes >= kWarps * STAGES * 9, "header area too small");
    static_assert(kWarps * STAGES * TB >= 2 * kWarps * RPC * 4 + kWarps * RPC * DP * 4, "merge area too small");
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* stages = smem + hdr_bytes<NB, NT, TREE>();
    __shared__ int s_last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // chunk index is the slowest grid dimension: every unit's first chunks are dispatched first
    const int c = blockIdx.z, b = blockIdx.y;
    const int h = blockIdx.x % p.H, rg = blockIdx.x / p.H;

    UnitGeom u;
    if (!unit_geom<TPP, RPC>(p, b, rg, u, threadIdx.x == 0 && c == 0)) return;
    if (c >= u.n_chunks) return;
    const int tile_begin = c * p.chunk_tiles;
    const int tile_end = min(tile_begin + p.chunk_tiles, u.n_tiles);

    uint4 qf[NT][D / 32];
    int kvlen[NT][2], kv_min;
    load_unit_q<D, NT, NB>(p, u, h, lane, qf, kvlen, kv_min, kbias_area<NB, NT>(smem, warp));
    TreeCtx tc{};
    if constexpr (TREE) {
        // ancestor masks of the entry's draft rows from the subtree ranges (clamped to the block;
        // a range outside it flags YF_DEV_BAD_ROWS)
        unsigned long long* anc = reinterpret_cast<unsigned long long*>(smem + hdr_bytes<NB, NT>());
        for (int i = threadIdx.x; i < kMaxTreeRows; i += kThreads) anc[i] = 0ull;
        __syncthreads();
        for (int j = threadIdx.x; j < u.Tq; j += kThreads) {
            const int2 r = p.trie[u.qrow0 + j];
            if (r.x < 0 || r.y >= u.Tq || r.x > r.y) atomicOr(p.status, YF_DEV_BAD_ROWS);
            const int lo = max(max(r.x, j), 0), hi = min(r.y, u.Tq - 1);
            for (int i = lo; i <= hi; ++i) atomicOr(&anc[i], 1ull << j);
        }
        __syncthreads();
        tc = TreeCtx{anc, u.Tk - u.Tq, u.row_begin, p.G};
        kv_min = min(kv_min, u.Tk - u.Tq);  // every tile holding a draft key takes the mask
    }
    TileRing<TB, STAGES> ring;
    ring.init(smem, stages, warp, lane);
    WarpAcc<D, NT> acc;
    acc.reset();
    stream_unit<D, NB, NT, TPP, STAGES, TREE>(p, ring, b, h, tile_begin, tile_end - tile_begin, qf, kvlen, kv_min,
                                              kbias_area<NB, NT>(smem, warp), acc, warp, lane, tc);
    stash_warp<D, NT>(stages, acc, warp, lane);

    const bool direct = u.n_chunks == 1;
    const size_t unit = ((size_t)b * p.H + h) * p.n_row_groups + rg;
    emit_unit<D, NT>(p, u, h, stages, direct, unit * p.max_chunks + c);
    if (direct || !p.counters) return;
    auto item_of = [&](int k) -> size_t { return unit * p.max_chunks + k; };
    if ((u.n_chunks + 1) * RPC * 4 <= kWarps * STAGES * TB)
        arrive_and_merge<D, RPC>(p, u, h, unit, u.n_chunks, item_of, reinterpret_cast<float*>(stages), &s_last);
    else if (arrive_last(&p.counters[unit], u.n_chunks, &s_last)) {
        combine_items<D, RPC>(p, u, h, u.n_chunks, item_of);
        if (threadIdx.x == 0) p.counters[unit] = 0;
    }
}

// Separate merge launch for schedule 2 when the pool's counters cannot be used.
template <int D, int TPP, int RPC>
__global__ void __launch_bounds__(kThreads) splitkv_combine(const SplitParams p) {
    const int b = blockIdx.y;
    const int h = blockIdx.x % p.H, rg = blockIdx.x / p.H;
    UnitGeom u;
    if (!unit_geom<TPP, RPC>(p, b, rg, u, false)) return;
    if (u.n_chunks <= 1) return;
    const size_t unit = ((size_t)b * p.H + h) * p.n_row_groups + rg;
    auto item_of = [&](int k) -> size_t { return unit * p.max_chunks + k; };
    combine_items<D, RPC>(p, u, h, u.n_chunks, item_of);
}

// ---- launch ----------------------------------------------------------------------------------

template <int D, int NB, int NT, int TPP, int STAGES, bool TREE = false>
static int launch_t(const AttnArgs& a, const SplitPlan& plan, const SplitParams& p) {
    constexpr int TB = 32 * D + 64 * NB;
    constexpr int SMEM = hdr_bytes<NB, NT, TREE>() + kWarps * STAGES * TB;
    const int dev = a.pool->desc.device;
    cudaError_t e;
    if constexpr (!TREE && NT == 1) {
        if (plan.cluster) {
            auto kern = decode_cluster_kernel<D, NB, TPP, STAGES>;
            static LaunchCache ccache;
            constexpr int SMEM_C = SMEM > kClusterSmemFloor ? SMEM : kClusterSmemFloor;
            const int rc = raise_smem_attr((const void*)kern, SMEM_C, dev, ccache);
            if (rc) return rc;
            const long long units = (long long)a.batch * a.pool->desc.n_kv_heads;
            const long long ctas = units * plan.max_chunks * kClusterCtas;
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3((unsigned)ctas);
            cfg.blockDim = dim3(kThreads);
            cfg.dynamicSmemBytes = SMEM_C;
            cfg.stream = a.stream;
            cudaLaunchAttribute attr[1];
            pdl_attr(attr[0]);
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            e = cudaLaunchKernelEx(&cfg, kern, p);
            if (e == cudaSuccess) e = cudaGetLastError();
            return e == cudaSuccess ? YF_OK : cuda_fail(e, "decode_cluster launch");
        }
    }
    if (!TREE && plan.persistent) {
        auto kern = decode_persistent_kernel<D, NB, NT, TPP, STAGES>;
        static LaunchCache cache;
        const int smem = SMEM + (a.batch + 1) * (int)sizeof(long long);
        int rc = raise_smem_attr((const void*)kern, SMEM + (kPersistentMaxBatch + 1) * (int)sizeof(long long), dev,
                                 cache);
        if (rc) return rc;
        // every CTA must be resident at once (mergers wait for the parts of other CTAs): the grid
        // is capped by the occupancy at this shared-memory size; with YF_LAUNCH_COOPERATIVE the
        // launch itself guarantees co-residency (a grid that cannot be co-resident is deferred or
        // refused instead of stalling its mergers), at 2-3 us per call
        int occ = 0;
        rc = occupancy((const void*)kern, kThreads, smem, dev, cache, &occ);
        if (rc) return rc;
        int ctas = std::max(1, std::min(plan.persistent_ctas, occ * a.pool->sm_count));
        // a few units over many CTAs: a multiple of the unit count puts the boundaries of
        // equal-length units on CTA boundaries (no CTA switches units and joins two merges)
        const long long units = (long long)a.batch * a.pool->desc.n_kv_heads * plan.n_row_groups;
        if (units > 1 && ctas >= 16 * units) ctas -= (int)(ctas % units);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(ctas);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = a.stream;
        // no programmatic (early) launch here: the grid is sized to exactly one resident wave, and
        // CTAs launched while the previous kernel still holds SMs start late and end late
        // (decode_batch's step: 112.7 against 108.5 us)
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = a.pool->opts.launch == YF_LAUNCH_COOPERATIVE ? 1 : 0;
        e = cudaLaunchKernelEx(&cfg, kern, p);
        if (e == cudaSuccess) e = cudaGetLastError();
        return e == cudaSuccess ? YF_OK : cuda_fail(e, "decode_persistent launch");
    }
    auto kern = splitkv_kernel<D, NB, NT, TPP, STAGES, TREE>;
    static LaunchCache cache2;
    const int rc = raise_smem_attr((const void*)kern, SMEM, dev, cache2);
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.pool->desc.n_kv_heads * plan.n_row_groups, a.batch, plan.max_chunks);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = SMEM;
    cfg.stream = a.stream;
    cudaLaunchAttribute attr[1];
    pdl_attr(attr[0]);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "splitkv launch");
    if (plan.max_chunks > 1 && !p.counters) {
        const dim3 cg(a.pool->desc.n_kv_heads * plan.n_row_groups, a.batch);
        splitkv_combine<D, TPP, 8 * NT><<<cg, kThreads, 0, a.stream>>>(p);
        e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_fail(e, "combine launch");
    }
    return YF_OK;
}

template <int D, int NB, int NT, int TPP>
static int launch_st(const AttnArgs& a, const SplitPlan& plan, const SplitParams& p) {
    if (p.trie) {  // tree verify: the chunked schedule at the default depth
        if constexpr (D == 128)
            return launch_t<D, NB, NT, TPP, 4, true>(a, plan, p);
        else
            return launch_t<D, NB, NT, TPP, 2, true>(a, plan, p);
    }
    if (plan.stages == 3) return launch_t<D, NB, NT, TPP, 3>(a, plan, p);
    if constexpr (D == 128)
        return launch_t<D, NB, NT, TPP, 4>(a, plan, p);
    else
        return launch_t<D, NB, NT, TPP, 2>(a, plan, p);
}

template <int D, int NB, int NT>
static int launch_tpp(const AttnArgs& a, const SplitPlan& plan, const SplitParams& p) {
    if (a.pool->desc.page_size == 16) return launch_st<D, NB, NT, 1>(a, plan, p);
    return launch_st<D, NB, NT, 4>(a, plan, p);
}

// ---- cluster capacity of decode_cluster_kernel ------------------------------------------------

namespace {
std::mutex g_cluster_mu;
}

template <int D, int NB, int TPP, int STAGES>
static int cluster_capacity_t(int dev, int sm_count) {
    static int cached[64] = {};
    constexpr int TB = 32 * D + 64 * NB;
    constexpr int SMEM0 = hdr_bytes<NB, 1>() + kWarps * STAGES * TB;
    constexpr int SMEM = SMEM0 > kClusterSmemFloor ? SMEM0 : kClusterSmemFloor;  // as launched
    const int fallback = std::max(1, sm_count * 2 / kClusterCtas);
    if (dev < 0 || dev >= 64) return fallback;
    std::lock_guard<std::mutex> lock(g_cluster_mu);
    if (cached[dev] > 0) return cached[dev];
    auto kern = decode_cluster_kernel<D, NB, TPP, STAGES>;
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) return fallback;
    if (prev != dev && cudaSetDevice(dev) != cudaSuccess) return fallback;
    int n = 0;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (e == cudaSuccess) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(kClusterCtas * 256);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = SMEM;
        e = cudaOccupancyMaxActiveClusters(&n, (const void*)kern, &cfg);
    }
    if (prev != dev) cudaSetDevice(prev);
    if (e != cudaSuccess || n <= 0) {
        cudaGetLastError();
        return fallback;
    }
    cached[dev] = n;
    return n;
}

template <int D, int NB, int TPP>
static int cluster_capacity_st(int dev, int sm, int stages) {
    if (stages == 3) return cluster_capacity_t<D, NB, TPP, 3>(dev, sm);
    if constexpr (D == 128)
        return cluster_capacity_t<D, NB, TPP, 4>(dev, sm);
    else
        return cluster_capacity_t<D, NB, TPP, 2>(dev, sm);
}

int cluster_capacity(const yf_pool* pool, int stages) {
    const yf_pool_desc& d = pool->desc;
    const int dev = pool->base ? d.device : -1;
    const bool rs = d.group_size == d.head_dim, p16 = d.page_size == 16;
    if (d.head_dim == 128) {
        if (rs) return p16 ? cluster_capacity_st<128, 1, 1>(dev, pool->sm_count, stages)
                           : cluster_capacity_st<128, 1, 4>(dev, pool->sm_count, stages);
        return p16 ? cluster_capacity_st<128, 4, 1>(dev, pool->sm_count, stages)
                   : cluster_capacity_st<128, 4, 4>(dev, pool->sm_count, stages);
    }
    if (rs) return p16 ? cluster_capacity_st<256, 1, 1>(dev, pool->sm_count, stages)
                       : cluster_capacity_st<256, 1, 4>(dev, pool->sm_count, stages);
    return p16 ? cluster_capacity_st<256, 8, 1>(dev, pool->sm_count, stages)
               : cluster_capacity_st<256, 8, 4>(dev, pool->sm_count, stages);
}

int launch_splitkv(const AttnArgs& a, const SplitPlan& plan) {
    const yf_pool_desc& d = a.pool->desc;
    SplitParams p;
    p.layer_base = a.pool->base + (size_t)a.layer * a.pool->layer_bytes;
    p.n_pages = d.n_pages;
    p.H = d.n_kv_heads;
    p.G = a.n_q_heads / d.n_kv_heads;
    p.Hq = a.n_q_heads;
    p.B = a.batch;
    p.phb = (long long)a.pool->page_head_bytes;
    p.q = a.q;
    p.cu_q = a.cu_q;
    p.cu_k = a.cu_k;
    p.bt = a.block_table;
    p.max_blocks = a.max_blocks;
    p.max_seqlen_q = a.max_seqlen_q;
    p.n_row_groups = plan.n_row_groups;
    p.chunk_tiles = plan.chunk_tiles;
    p.max_chunks = plan.max_chunks;
    p.scale_log2 = a.scale * 1.4426950408889634f;
    p.out = a.out;
    p.part_o = a.part_o;
    p.part_lse = a.part_lse;
    p.status = a.pool->d_status;
    p.trie = reinterpret_cast<const int2*>(a.trie);
    p.wait_ns = wait_limit_ns(a.pool);
    p.x = a.xf ? *a.xf : XFuse{};
    if (p.x.peers && !plan.cluster) return fail(YF_E_UNSUPPORTED, "the fused exchange needs the cluster schedule");
    if (p.trie && plan.persistent) return fail(YF_E_UNSUPPORTED, "tree verify needs the chunked schedule");
    const size_t units = (size_t)a.batch * d.n_kv_heads * plan.n_row_groups;
    p.counters = (plan.fused_combine && units <= (size_t)kMaxCombineUnits) ? a.pool->d_counters : nullptr;
    if (plan.persistent && !p.counters) return fail(YF_E_UNSUPPORTED, "persistent decode needs the merge counters");
    if (plan.ws_bytes > 0) {
        const size_t items = plan.persistent ? (size_t)plan.persistent_ctas * 2 : units * plan.max_chunks;  // cluster: units x clusters
        p.ws_o = static_cast<float*>(a.workspace);
        p.ws_lse = p.ws_o + items * plan.rows_per_cta * d.head_dim;
    } else {
        p.ws_o = nullptr;
        p.ws_lse = nullptr;
    }
    const bool row_scale = d.group_size == d.head_dim;
    if (d.head_dim == 128) {
        if (plan.rows_per_cta == 8)
            return row_scale ? launch_tpp<128, 1, 1>(a, plan, p) : launch_tpp<128, 4, 1>(a, plan, p);
        return row_scale ? launch_tpp<128, 1, 2>(a, plan, p) : launch_tpp<128, 4, 2>(a, plan, p);
    }
    return row_scale ? launch_tpp<256, 1, 1>(a, plan, p) : launch_tpp<256, 8, 1>(a, plan, p);
}

}  // namespace yf
