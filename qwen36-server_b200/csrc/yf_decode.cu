// Split-KV paged Q8_0 attention for decode, MTP verify and other small query
// blocks, plus the log-sum-exp combine of the split partials.
//
// Replaces the int8-pool decode/verify branch of the engine's FA2 split-KV
// kernel (compute_attn_1rowblock_splitkv with Is_kv_q8, described at
// docs/research/2026-09-16-head-to-head-llamacpp-and-phase-profile.md:3469-3481)
// and flash_fwd_splitkv_combine_kernel (docs/plans/2026-09-16-prefil-parity-fa2-and-mmq.md:104-107).
//
// One CTA = (entry b, kv head h, group of 8 or 16 query rows, chunk of
// 16-token tiles).  The query rows are the G = Hq/Hkv q heads of kv head h
// times the query positions (GQA folded into the MMA N dimension), so every
// K/V byte is read once per CTA.  Each of the 4 warps streams its own tiles:
// lane 0 issues a 1-D bulk copy (cp.async.bulk, no multicast) of the whole
// tile (K int8 + scales + V int8 + scales, one contiguous block of the pool)
// into a per-warp ring of shared-memory stages, completing on an mbarrier.
// The tile bytes are laid out so that each lane's 16-byte shared load is
// exactly its mma.sync fragment: K feeds S^T = K Q^T (tokens in M), V feeds
// O^T = V^T P^T (dims in M); int8 is unpacked to exact f16 in registers and
// the Q8_0 group scales are applied to the per-group partial dot products (K)
// and to P (V), so the tensor cores see only exact integers.  Softmax is
// online, base 2, with warp-shuffle row maxima and a lazy rescale; rows of one
// CTA end in a shared-memory merge of the 4 warps.  A unit that needs one
// chunk writes f16 output directly; otherwise normalised partials + lse go to
// the workspace and the CTA that finishes the unit's last chunk (an arrival
// counter in the pool) merges them, so no second launch is needed.  Lane 0
// loads each tile's page id one tile ahead so the block-table read stays off
// the copy's critical path.  Calls on one pool must be stream-ordered (the
// counters are per pool).
#include <cfloat>

#include "yf_device.cuh"
#include "yf_internal.h"

namespace yf {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kHdrBytes = 256;  // mbarriers + per-stage page-valid flags
// Lazy softmax rescale: the running max only moves when a tile's max exceeds it by
// more than 2^8 in probability terms, so most tiles skip the O rescale; p <= 256.
constexpr float kRescaleThresh = 8.0f;

struct SplitParams {
    const uint8_t* layer_base;
    int n_pages;
    int H;   // kv heads
    int G;   // q heads per kv head
    int Hq;
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
    float* ws_o;
    float* ws_lse;
    uint32_t* counters;  // per-unit arrival counters for the fused combine, or null
    uint32_t* status;
};

// Geometry of one CTA's unit, computed identically by both kernels.
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

// Merges the n_chunks partials (normalised O, base-2 lse) of one unit into f16 output.
// Loads go through L2 (ld.global.cg): the partials were written by other CTAs.
template <int D, int RPC>
__device__ __forceinline__ void combine_unit(const SplitParams& p, const UnitGeom& u, int h, size_t item0, int tid,
                                             int nthreads) {
    for (int e = tid; e < RPC * (D / 4); e += nthreads) {
        const int r = e / (D / 4), d4 = (e % (D / 4)) * 4;
        const int row = u.row_begin + r;
        if (row >= u.rows_total) continue;
        float M = -INFINITY;
        for (int c = 0; c < u.n_chunks; ++c) M = fmaxf(M, __ldcg(p.ws_lse + (item0 + c) * RPC + r));
        float L = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int c = 0; c < u.n_chunks; ++c) {
            const float lv = __ldcg(p.ws_lse + (item0 + c) * RPC + r);
            if (lv == -INFINITY) continue;
            const float f = fast_exp2(lv - M);
            L += f;
            const float4 ov = __ldcg(reinterpret_cast<const float4*>(p.ws_o + ((item0 + c) * RPC + r) * D + d4));
            acc.x = fmaf(f, ov.x, acc.x);
            acc.y = fmaf(f, ov.y, acc.y);
            acc.z = fmaf(f, ov.z, acc.z);
            acc.w = fmaf(f, ov.w, acc.w);
        }
        const float inv = L > 0.f ? 1.f / L : 0.f;
        const int j = row / p.G, gi = row % p.G;
        __half* op = p.out + ((size_t)(u.qrow0 + j) * p.Hq + (size_t)h * p.G + gi) * D + d4;
        uint2 pk;
        pk.x = pack_h2(acc.x * inv, acc.y * inv);
        pk.y = pack_h2(acc.z * inv, acc.w * inv);
        *reinterpret_cast<uint2*>(op) = pk;
    }
}

template <int D, int NB, int NT, int TPP, int STAGES>
__global__ void __launch_bounds__(kThreads) splitkv_kernel(const SplitParams p) {
    constexpr int TB = 32 * D + 64 * NB;  // tile bytes
    constexpr int KS_OFF = 16 * D;
    constexpr int V_OFF = 16 * D + 32 * NB;
    constexpr int VS_OFF = 32 * D + 32 * NB;
    constexpr int CH = D / 32;    // 32-dim chunks (one 16-byte K word per lane each)
    constexpr int CPG = CH / NB;  // chunks per scale group
    constexpr int MT = D / 16;    // 16-dim m-tiles of O^T
    constexpr int MPG = MT / NB;  // m-tiles per scale group
    constexpr int RPC = 8 * NT;   // query rows per CTA
    constexpr int DP = D + 4;     // padded row stride of the merge buffer
    static_assert(MPG % 2 == 0, "m-tiles come in pairs per 16-byte V word");
    static_assert(kHdrBytes >= kWarps * STAGES * 9, "header area too small");
    static_assert(kWarps * STAGES * TB >= 2 * kWarps * RPC * 4 + kWarps * RPC * DP * 4, "merge area too small");

    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
    uint8_t* sflag = smem + kWarps * STAGES * 8;
    uint8_t* stages = smem + kHdrBytes;
    __shared__ int s_last;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, tig = lane & 3;
    // chunk index is the slowest grid dimension: every unit's first chunks are dispatched first
    const int c = blockIdx.z, b = blockIdx.y;
    const int h = blockIdx.x % p.H, rg = blockIdx.x / p.H;

    UnitGeom u;
    if (!unit_geom<TPP, RPC>(p, b, rg, u, threadIdx.x == 0 && c == 0)) return;
    if (c >= u.n_chunks) return;
    const int tile_begin = c * p.chunk_tiles;
    const int tile_end = min(tile_begin + p.chunk_tiles, u.n_tiles);

    // Keys visible to the softmax rows this lane owns (columns 2tig, 2tig+1 of each n-tile).
    int kvlen[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int col = 0; col < 2; ++col) {
            const int r = u.row_begin + nt * 8 + 2 * tig + col;
            const int kl = u.Tk - u.Tq + r / p.G + 1;
            kvlen[nt][col] = r < u.rows_total ? max(0, min(kl, u.Tk)) : 0;
        }

    // Q^T fragments: lane holds Q[row nt*8+g][32cb + 8tig .. +7] for every chunk.
    uint4 qf[NT][CH];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int r = u.row_begin + nt * 8 + g;
        if (r < u.rows_total) {
            const int j = r / p.G, gi = r % p.G;
            const uint4* qp = reinterpret_cast<const uint4*>(
                p.q + ((size_t)(u.qrow0 + j) * p.Hq + (size_t)h * p.G + gi) * D);
#pragma unroll
            for (int cb = 0; cb < CH; ++cb) qf[nt][cb] = __ldg(qp + cb * 4 + tig);
        } else {
#pragma unroll
            for (int cb = 0; cb < CH; ++cb) qf[nt][cb] = make_uint4(0, 0, 0, 0);
        }
    }

    // Per-warp ring of tile stages.
    uint64_t* mybar = bars + warp * STAGES;
    uint8_t* mystage = stages + (size_t)warp * STAGES * TB;
    const int span = tile_end - tile_begin;
    const int my_n = span > warp ? (span - warp + kWarps - 1) / kWarps : 0;
    const uint32_t* btrow = p.bt + (size_t)b * p.max_blocks;
    const uint8_t* head_base = p.layer_base + (size_t)h * p.phb;
    const long long page_stride = p.phb * p.H;

    uint8_t* myflag = sflag + warp * STAGES;
    // lane 0 only: copy tile kt (page id already loaded) into `slot`; a page id past the pool
    // completes the stage without a copy and marks it invalid.
    auto issue = [&](int slot, int kt, uint32_t page) {
        if (page < (uint32_t)p.n_pages) {
            myflag[slot] = 1;
            mbar_arrive_expect_tx(&mybar[slot], TB);
            bulk_g2s(mystage + slot * TB, head_base + (size_t)page * page_stride + (kt % TPP) * TB, TB,
                     &mybar[slot]);
        } else {
            myflag[slot] = 0;
            atomicOr(p.status, YF_DEV_BAD_PAGE);
            mbar_arrive(&mybar[slot]);
        }
    };
    auto tile_of = [&](int i) { return tile_begin + warp + i * kWarps; };

    uint32_t next_page = 0;  // lane 0: page id of the next tile to issue, loaded one tile ahead
    if (lane == 0) {
#pragma unroll
        for (int s = 0; s < STAGES; ++s) mbar_init(&mybar[s], 1);
        fence_mbar_init();
        for (int s = 0; s < STAGES && s < my_n; ++s) issue(s, tile_of(s), __ldg(btrow + tile_of(s) / TPP));
        if (STAGES < my_n) next_page = __ldg(btrow + tile_of(STAGES) / TPP);
    }
    __syncwarp();

    float m_run[NT][2], l_run[NT][2];
    float o[MT][NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        m_run[nt][0] = m_run[nt][1] = -INFINITY;
        l_run[nt][0] = l_run[nt][1] = 0.f;
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) o[mt][nt][e] = 0.f;

    int done = 0;
    for (int i = 0; i < my_n; ++i) {
        const int slot = i % STAGES;
        const uint32_t parity = (uint32_t)(i / STAGES) & 1u;
        const int kt = tile_of(i);
        const bool arrived = __all_sync(0xffffffffu, mbar_wait(&mybar[slot], parity));
        if (!arrived) {
            if (lane == 0) atomicOr(p.status, YF_DEV_TIMEOUT);
            break;
        }
        done = i + 1;
        if (myflag[slot]) {
            const uint8_t* T = mystage + slot * TB;
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
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
#pragma unroll
                for (int cc = 0; cc < CPG; ++cc) {
                    const int cb = s * CPG + cc;
                    const uint4 kw = lds128(T + cb * 512 + lane * 16);
                    const uint32_t x0 = bias8(kw.x), x1 = bias8(kw.y), z0 = bias8(kw.z), z1 = bias8(kw.w);
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
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    sacc[nt][0] = fmaf(ks0[s], acc[nt][0], sacc[nt][0]);
                    sacc[nt][1] = fmaf(ks0[s], acc[nt][1], sacc[nt][1]);
                    sacc[nt][2] = fmaf(ks1[s], acc[nt][2], sacc[nt][2]);
                    sacc[nt][3] = fmaf(ks1[s], acc[nt][3], sacc[nt][3]);
                }
            }
            // ---- online softmax (base 2) on rows 2tig, 2tig+1 of each n-tile
            const int tok0 = kt * kTileTokens + g, tok1 = tok0 + 8;
            uint32_t pb01[NT], pb23[NT];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                float pr[2][2];
#pragma unroll
                bool need = false;
                float alpha[2];
#pragma unroll
                for (int col = 0; col < 2; ++col) {
                    float v0 = sacc[nt][col] * p.scale_log2;
                    float v1 = sacc[nt][2 + col] * p.scale_log2;
                    if (tok0 >= kvlen[nt][col]) v0 = -INFINITY;
                    if (tok1 >= kvlen[nt][col]) v1 = -INFINITY;
                    float mx = fmaxf(v0, v1);
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                    alpha[col] = 1.f;
                    if (mx > m_run[nt][col] + kRescaleThresh) {
                        // m_run == -inf gives alpha = exp2(-inf) = 0 (nothing accumulated yet)
                        alpha[col] = fast_exp2(m_run[nt][col] - mx);
                        m_run[nt][col] = mx;
                        l_run[nt][col] *= alpha[col];
                        need = true;
                    }
                    const float muse = m_run[nt][col] == -INFINITY ? 0.f : m_run[nt][col];
                    pr[col][0] = fast_exp2(v0 - muse);
                    pr[col][1] = fast_exp2(v1 - muse);
                    l_run[nt][col] += pr[col][0] + pr[col][1];
                }
                if (__any_sync(0xffffffffu, need)) {
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        o[mt][nt][0] *= alpha[0];
                        o[mt][nt][2] *= alpha[0];
                        o[mt][nt][1] *= alpha[1];
                        o[mt][nt][3] *= alpha[1];
                    }
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
                    uint32_t w0 = bias8(vw.x), w1 = bias8(vw.y);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
                        mma16816(o[mt0][nt], s8lo_to_h2(w0), s8lo_to_h2(w1), s8hi_to_h2(w0), s8hi_to_h2(w1), b0[nt],
                                 b1[nt]);
                    w0 = bias8(vw.z);
                    w1 = bias8(vw.w);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
                        mma16816(o[mt0 + 1][nt], s8lo_to_h2(w0), s8lo_to_h2(w1), s8hi_to_h2(w0), s8hi_to_h2(w1),
                                 b0[nt], b1[nt]);
                }
            }
        }
        __syncwarp();
        if (lane == 0 && i + STAGES < my_n) {
            issue(slot, tile_of(i + STAGES), next_page);
            if (i + STAGES + 1 < my_n) next_page = __ldg(btrow + tile_of(i + STAGES + 1) / TPP);
        }
    }
    // A warp that gave up waits (bounded) for the copies it still has in flight.
    if (done < my_n) {
        for (int i = done; i < my_n && i < done + STAGES; ++i)
            (void)mbar_wait(&mybar[i % STAGES], (uint32_t)(i / STAGES) & 1u);
    }

    // ---- merge the 4 warps
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int col = 0; col < 2; ++col) {
            float l = l_run[nt][col];
            l += __shfl_xor_sync(0xffffffffu, l, 4);
            l += __shfl_xor_sync(0xffffffffu, l, 8);
            l += __shfl_xor_sync(0xffffffffu, l, 16);
            l_run[nt][col] = l;
        }
    __syncthreads();
    float* mw = reinterpret_cast<float*>(stages);
    float* lw = mw + kWarps * RPC;
    float* ow = lw + kWarps * RPC;
    if (g == 0) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int col = 0; col < 2; ++col) {
                mw[warp * RPC + nt * 8 + 2 * tig + col] = m_run[nt][col];
                lw[warp * RPC + nt * 8 + 2 * tig + col] = l_run[nt][col];
            }
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int r = nt * 8 + 2 * tig + (e & 1);
                const int d = 16 * mt + g + 8 * (e >> 1);
                ow[(warp * RPC + r) * DP + d] = o[mt][nt][e];
            }
    __syncthreads();

    const bool direct = u.n_chunks == 1;
    const size_t unit = ((size_t)b * p.H + h) * p.n_row_groups + rg;
    const size_t item = unit * p.max_chunks + c;
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
            const int j = row / p.G, gi = row % p.G;
            __half* op = p.out + ((size_t)(u.qrow0 + j) * p.Hq + (size_t)h * p.G + gi) * D + d4;
            uint2 pk;
            pk.x = pack_h2(acc.x, acc.y);
            pk.y = pack_h2(acc.z, acc.w);
            *reinterpret_cast<uint2*>(op) = pk;
        } else {
            *reinterpret_cast<float4*>(p.ws_o + (item * RPC + r) * D + d4) = acc;
            if (d4 == 0) p.ws_lse[item * RPC + r] = L > 0.f ? M + __log2f(L) : -INFINITY;
        }
    }
    if (direct || !p.counters) return;

    // Fused combine: the CTA that finishes a unit's last chunk merges all its partials.
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t prev = atomicAdd(&p.counters[unit], 1u);
        s_last = prev == (uint32_t)u.n_chunks - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    combine_unit<D, RPC>(p, u, h, unit * p.max_chunks, threadIdx.x, kThreads);
    if (threadIdx.x == 0) p.counters[unit] = 0;  // ready for the next call on this pool
}

// Log-sum-exp merge of the chunk partials of one (entry, kv head, row group).
template <int D, int TPP, int RPC>
__global__ void __launch_bounds__(kThreads) splitkv_combine(const SplitParams p) {
    const int b = blockIdx.y;
    const int h = blockIdx.x % p.H, rg = blockIdx.x / p.H;
    UnitGeom u;
    if (!unit_geom<TPP, RPC>(p, b, rg, u, false)) return;
    if (u.n_chunks <= 1) return;
    const size_t unit = ((size_t)b * p.H + h) * p.n_row_groups + rg;
    combine_unit<D, RPC>(p, u, h, unit * p.max_chunks, threadIdx.x, kThreads);
}

template <int D, int NB, int NT, int TPP, int STAGES>
static int launch_t(const AttnArgs& a, const SplitPlan& plan, const SplitParams& p) {
    constexpr int TB = 32 * D + 64 * NB;
    constexpr int SMEM = kHdrBytes + kWarps * STAGES * TB;
    auto kern = splitkv_kernel<D, NB, NT, TPP, STAGES>;
    static bool attr_set[64] = {};
    const int dev = a.pool->desc.device;
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(splitkv)");
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    const dim3 grid(a.pool->desc.n_kv_heads * plan.n_row_groups, a.batch, plan.max_chunks);
    kern<<<grid, kThreads, SMEM, a.stream>>>(p);
    cudaError_t e = cudaGetLastError();
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
    if (plan.stages == 3) return launch_t<D, NB, NT, TPP, 3>(a, plan, p);
    return launch_t<D, NB, NT, TPP, (D == 128 ? 4 : 3)>(a, plan, p);
}

template <int D, int NB, int NT>
static int launch_tpp(const AttnArgs& a, const SplitPlan& plan, const SplitParams& p) {
    if (a.pool->desc.page_size == 16) return launch_st<D, NB, NT, 1>(a, plan, p);
    return launch_st<D, NB, NT, 4>(a, plan, p);
}

int launch_splitkv(const AttnArgs& a, const SplitPlan& plan) {
    const yf_pool_desc& d = a.pool->desc;
    SplitParams p;
    p.layer_base = a.pool->base + (size_t)a.layer * a.pool->layer_bytes;
    p.n_pages = d.n_pages;
    p.H = d.n_kv_heads;
    p.G = a.n_q_heads / d.n_kv_heads;
    p.Hq = a.n_q_heads;
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
    p.status = a.pool->d_status;
    const size_t units = (size_t)a.batch * d.n_kv_heads * plan.n_row_groups;
    p.counters = (plan.fused_combine && units <= (size_t)kMaxCombineUnits) ? a.pool->d_counters : nullptr;
    if (plan.max_chunks > 1) {
        const size_t items = (size_t)a.batch * d.n_kv_heads * plan.n_row_groups * plan.max_chunks;
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
