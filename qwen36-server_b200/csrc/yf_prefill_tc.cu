// Causal chunked-prefill attention over the paged Q8_0 pool on the 5th-generation
// tensor cores (tcgen05, TMEM accumulators).
//
// Replaces the prefill branch of the engine's FA2 varlen split-KV call from
// forward_attn_prefill_paged (docs/plans/2026-08-27-mtp-cuda-graphs.md:132,244-248;
// QK_INT8_PREFILL described at docs/research/2026-09-16-head-to-head-llamacpp-and-phase-profile.md:3627-3634):
// query row i of an entry sees keys 0 .. Tk - Tq + i.
//
// One CTA = one entry, one kv head and two query tiles of 128 rows (256/G query positions x
// the G q heads of the kv head: GQA folded into M).  CTAs come in clusters of two covering
// adjacent row blocks of the same (entry, kv head): each CTA of the pair copies and
// dequantizes one 64-key half of every key tile and writes the f16 result into both CTAs'
// shared memory (distributed shared memory), so each pool byte is copied and dequantized once
// for 512 rows.  Keys advance in tiles of 128.  Per key tile j and query tile i:
//   S_i = Q_i K_j^T      tcgen05.mma kind::f16, A = Q_i and B = K_j from shared memory
//                        (K-major, 128-byte swizzle), M = 128 rows, N = 128 keys, f32 in TMEM;
//   P_i = softmax part   written back into TMEM as f16 over the upper half of S_i's columns;
//   O_i += P_i V_j       tcgen05.mma with A = P_i read from TMEM, B = V_j^T from shared
//                        memory, M = 128 rows, N = 128 dims, f32 accumulator in TMEM.
// TMEM (512 columns): O_0 [0,128), O_1 [128,256), S_0 [256,384), S_1 [384,512).
//
// Warp roles (14 warps), handing buffers to each other through mbarriers:
//   * warps 0-3 / 4-7, softmax of query tile 0 / 1: thread r owns row r (TMEM lane r):
//     row max, lazy base-2 rescale of the running max (O_i rescaled in TMEM by the same
//     thread, only when the max grew by more than 2^8), exponentials, f16 P into TMEM;
//   * warps 8-11, dequant: this CTA's half of each key tile, int8 pool tiles staged by bulk
//     copies -> f16 K [key][dim] and V^T [dim][key] in the swizzled layouts the MMA descriptors
//     describe, stored locally and into the peer CTA;
//   * warp 12, control (one lane): every MMA and commit, polling its barriers, and the report
//     to the peer that a K/V^T stage is no longer read here;
//   * warp 13, copies (one lane): bulk copies of this CTA's 64-key half of each key tile (K+V
//     int8 and scales, one 4352-byte block per 16-token tile), page ids read one half ahead.
// At the end thread r reads row r of O_i and writes out[row] / l[row].
// Pools with 32-dim scale groups (4352-byte tiles) and with one scale per row (4160-byte tiles,
// the engine's own int8 pool format) are both read; only the dequant's scale indexing differs.
#include <cstdint>
#include <cstdlib>

#include "yf_device.cuh"
#include "yf_internal.h"
#include "yf_pfcommon.cuh"
#include "yf_tc.cuh"

namespace yf {
namespace {

constexpr int kPfRows = 128;      // query rows per query tile (M of both MMAs)
constexpr int kPfTiles = 2;       // query tiles per CTA
constexpr int kPfKeys = 128;      // keys per key tile (N of S, K of PV)
constexpr int kPfD = 128;         // head dim (K of S, N of PV)
constexpr int kPfTmemCols = 512;
constexpr float kPfRescale = 8.0f;  // lazy rescale threshold (base 2), as in the decode kernels

// one 16-token pool tile at D=128: 4352 B with 32-dim scale groups (NB = 4), 4160 B with one
// scale per row (NB = 1)
template <int NB>
constexpr int raw_tile_bytes() { return 32 * 128 + 64 * NB; }
constexpr int kRawPitch = 4368;       // staged tiles 16 B apart modulo 128 B: spreads banks
constexpr int kRawHalf = 4 * kRawPitch;  // 64 keys

// shared-memory map (bytes from the 1024-aligned dynamic shared memory base)
constexpr int kSmQ = 0;                         // Q   [2 tiles][2 col blocks of 64 dims][128 rows][128 B] f16
constexpr int kSmK = kSmQ + kPfTiles * 32768;   // K   [2 stages][2 col blocks of 64 dims][128 keys][128 B]
constexpr int kSmVt = kSmK + 2 * 32768;         // V^T [2 stages][2 col blocks of 64 keys][128 dims][128 B]
constexpr int kSmRaw = kSmVt + 2 * 32768;       // raw [2 halves][4 pool tiles, kRawPitch apart]
constexpr int kSmMisc = kSmRaw + 2 * kRawHalf;
// misc: Bars at +0, TMEM address at +160, staged-tile flags [2][4] at +168, abort word at +176
constexpr int kSmAlloc = kSmMisc + 256;
constexpr int kPfWarps = 14;
constexpr int kPfBlock = kPfWarps * 32;
constexpr int kCtlWarp = 12;
constexpr int kCopyWarp = 13;
static_assert(kSmAlloc <= 232448, "shared memory");

struct PrefillParams {
    const uint8_t* layer_base;
    int n_pages;
    int H;
    int G;
    int Hq;
    long long phb;
    int tpp;  // 16-token tiles per page
    const __half* q;
    const uint32_t* cu_q;
    const uint32_t* cu_k;
    const uint32_t* bt;
    int max_blocks;
    int max_seqlen_q;
    float scale_log2;
    __half* out;
    uint32_t* status;
    uint64_t wait_ns;  // bound of every wait
};

struct Bars {
    uint64_t raw_full[2], raw_free[2];  // staged 64-key halves of the pool (this CTA's halves)
    uint64_t k_full[2], v_full[2];      // K / V^T stage of a key tile written (own half + the peer's copy)
    uint64_t k_free[2], v_free[2];      // K / V^T stage read by its last MMA, here and in the peer
    uint64_t s_full[2], p_full[2];      // per query tile
    uint64_t o_done[2];                 // per query tile: last PV complete
    uint64_t drain;
};
static_assert(sizeof(Bars) <= 160, "barrier area");


template <int NB>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPfBlock, 1) prefill_tc_kernel(const PrefillParams p) {
    constexpr int kRawTileBytes = raw_tile_bytes<NB>();
    static_assert(kRawTileBytes <= kRawPitch && kRawTileBytes % 16 == 0, "staged tile");
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* base = smem_raw;
    const uint32_t sbase = smem_u32(smem_raw);
    Bars* bars = reinterpret_cast<Bars*>(base + kSmMisc);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + kSmMisc + 160);
    uint8_t* s_valid = base + kSmMisc + 168;  // [2][4] staged pool-tile flags
    volatile int* s_abort = reinterpret_cast<volatile int*>(base + kSmMisc + 176);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int b = blockIdx.z, h = blockIdx.y;
    const int ppb = kPfTiles * kPfRows / p.G;  // query positions per CTA

    // ---- geometry (same clamps as the split-KV kernels)
    const int cap = p.max_blocks * p.tpp * 16;
    const uint32_t tk_u = p.cu_k[b + 1] - p.cu_k[b];
    const int Tk = tk_u > (uint32_t)cap ? cap : (int)tk_u;
    const uint32_t tq_u = p.cu_q[b + 1] - p.cu_q[b];
    const int Tq = tq_u > (uint32_t)p.max_seqlen_q ? p.max_seqlen_q : (int)tq_u;
    if (tid == 0 && blockIdx.x == 0) {
        if (tk_u > (uint32_t)cap) atomicOr(p.status, YF_DEV_LEN_OVERFLOW);
        if (tq_u > (uint32_t)p.max_seqlen_q || Tq > Tk) atomicOr(p.status, YF_DEV_BAD_ROWS);
    }
    // the swizzled operand layouts need a 1024-aligned base (the whole map fits no slack)
    if (sbase & 1023u) {
        if (tid == 0) atomicOr(p.status, YF_DEV_SMEM_ALIGN);
        return;
    }
    const int qrow0 = (int)p.cu_q[b];
    const int rank = (int)(blockIdx.x & 1);  // rank in the cluster pair (x-adjacent CTAs)
    const uint32_t peer = (uint32_t)(rank ^ 1);
    const int pos0 = blockIdx.x * ppb, pair_pos0 = (blockIdx.x & ~1u) * ppb;
    if (pair_pos0 >= Tq) return;  // both CTAs of the pair: no rows
    const int npos = max(0, min(ppb, Tq - pos0));  // a pair's second CTA may have none
    const int rows = npos * p.G;
    const bool act1 = rows > kPfRows;  // query tile 1 holds rows (tile 0 always runs)
    const int kv0 = Tk - Tq;           // keys before the chunk
    // both CTAs stream the key tiles of the pair's last row
    const int kv_hi = max(0, min(Tk, kv0 + pair_pos0 + min(2 * ppb, Tq - pair_pos0)));
    const int n_kt = (kv_hi + kPfKeys - 1) / kPfKeys;
    const int pt_total = (Tk + 15) / 16;
    const int pt_need = (kv_hi + 15) / 16;  // pool tiles the pair reads
    const uint32_t* btrow = p.bt + (size_t)b * p.max_blocks;
    const uint8_t* head_base = p.layer_base + (size_t)h * p.phb;
    const long long page_stride = p.phb * p.H;

    // ---- set-up
    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bars->raw_full[i], 1);
            mbar_init(&bars->raw_free[i], 4);
            mbar_init(&bars->k_full[i], 4);  // the dequant warps; the peer's half comes as bytes
            mbar_init(&bars->v_full[i], 4);
            mbar_init(&bars->k_free[i], 2);  // this CTA's and the peer's last QK / PV of the tile
            mbar_init(&bars->v_free[i], 2);
            mbar_init(&bars->s_full[i], 1);
            mbar_init(&bars->p_full[i], 4);
            mbar_init(&bars->o_done[i], 1);
        }
        mbar_init(&bars->drain, 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == kCtlWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kPfTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    int bad = 0;
    if (warp < 8) {
        // Q row `row` (position pos0 + row/G, head h*G + row%G) into the SW128 Q tile
        const int qt = tid >> 7, r = tid & 127, row = tid;
        const bool live = row < rows;
        const uint4 zero = make_uint4(0, 0, 0, 0);
        const uint4* qp = nullptr;
        if (live)
            qp = reinterpret_cast<const uint4*>(
                p.q + ((size_t)(qrow0 + pos0 + row / p.G) * p.Hq + (size_t)h * p.G + row % p.G) * kPfD);
        const uint32_t qdst = sbase + kSmQ + qt * 32768;
#pragma unroll
        for (int c = 0; c < 16; ++c) sts128(qdst + sw128_off(r, c, kPfRows), live ? __ldg(qp + c) : zero);
        fence_proxy_async_smem();
        // every page this CTA reads exists (the common case skips per-tile page checks)
        for (int pt = tid; pt < pt_need; pt += 256)
            if (__ldg(btrow + pt / p.tpp) >= (uint32_t)p.n_pages) bad = 1;
    }
    tc_fence_before();
    const bool pages_ok = __syncthreads_or(bad) == 0;
    tc_fence_after();
    cluster_sync();  // the peer's barriers are initialised before any remote arrival
    const uint32_t tmem = *tmem_slot;

    if (warp == kCtlWarp) {
        // ================= control: bulk copies and MMAs =================
        if (lane == 0) {
            constexpr uint32_t IDESC = umma_idesc_f16(kPfRows, 128);  // S: N = 128 keys; O: N = 128 dims
            // Polling loop: issue whichever of {PV_i, QK_i} is ready.  S_i is
            // single-buffered: QK_i(j) follows PV_i(j-1), which read P_i from the same columns
            // (tcgen05.mma operations of one thread execute in issue order).
            int qk[2] = {0, 0}, pv[2] = {0, 0};
            uint32_t idle = 0;
            uint64_t idle_t0 = 0;
            while ((pv[0] < n_kt || (act1 && pv[1] < n_kt)) && !*s_abort) {
                bool prog = false;
#pragma unroll
                for (int i = 0; i < kPfTiles; ++i) {
                    if (i == 1 && !act1) break;
                    const uint32_t tS = tmem + 256 + i * 128;
                    if (pv[i] < qk[i] && mbar_test(&bars->p_full[i], pv[i]) &&
                        mbar_test(&bars->v_full[pv[i] & 1], pv[i] >> 1)) {
                        const int j = pv[i];
                        tc_fence_after();
#pragma unroll
                        for (int ks = 0; ks < kPfKeys / 16; ++ks) {
                            const uint64_t bd =
                                umma_desc_sw128(sbase + kSmVt + (j & 1) * 32768 + (ks >> 2) * 16384 + (ks & 3) * 32);
                            umma_ts(tmem + i * 128, tS + 64 + ks * 8, bd, IDESC, (j > 0 || ks > 0) ? 1u : 0u);
                        }
                        pv[i] = j + 1;
                        // the tile's last PV here: V^T may be rewritten once the peer's is done too
                        if (!act1 || pv[1 - i] > j) umma_commit_pair(&bars->v_free[j & 1]);
                        if (j == n_kt - 1) umma_commit(&bars->o_done[i]);
                        prog = true;
                    }
                    if (qk[i] < n_kt && qk[i] == pv[i] && mbar_test(&bars->k_full[qk[i] & 1], qk[i] >> 1)) {
                        const int j = qk[i];
                        tc_fence_after();
#pragma unroll
                        for (int ks = 0; ks < kPfD / 16; ++ks) {
                            const uint64_t a =
                                umma_desc_sw128(sbase + kSmQ + i * 32768 + (ks >> 2) * 16384 + (ks & 3) * 32);
                            const uint64_t bd =
                                umma_desc_sw128(sbase + kSmK + (j & 1) * 32768 + (ks >> 2) * 16384 + (ks & 3) * 32);
                            umma_ss(tS, a, bd, IDESC, ks > 0);
                        }
                        umma_commit(&bars->s_full[i]);
                        qk[i] = j + 1;
                        if (!act1 || qk[1 - i] > j) umma_commit_pair(&bars->k_free[j & 1]);  // last QK here
                        prog = true;
                    }
                }
                if (prog) {
                    idle = 0;
                } else if (++idle == 1) {
                    idle_t0 = globaltimer_ns();
                } else if ((idle & 63u) == 0 && globaltimer_ns() - idle_t0 > p.wait_ns) {
                    give_up(s_abort, p.status, wait_tag(1, kBarIdle, (qk[0] & 31) | ((pv[0] & 31) << 5)));
                }
            }
            // every MMA of this CTA has completed before TMEM is released
            umma_commit(&bars->drain);
            if (!mbar_wait(&bars->drain, 0u, p.wait_ns)) give_up(s_abort, p.status, wait_tag(1, kBarDrain, 0));
        }
        __syncwarp();
    } else if (warp == kCopyWarp) {
        // ================= copies: pool tiles of 64-key halves into the raw ring =================
        if (lane == 0) {
            uint32_t page[4];
            auto fetch_pages = [&](int hf) {  // page ids of pool tiles 4hf .. 4hf+3 (n_pages: skip)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int pt = hf * 4 + j;
                    page[j] = pt < pt_need ? __ldg(btrow + pt / p.tpp) : (uint32_t)p.n_pages;
                }
            };
            if (n_kt > 0) fetch_pages(rank);
            for (int kt = 0; kt < n_kt; ++kt) {
                const int hf = 2 * kt + rank, slot = kt & 1;  // this CTA's half of key tile kt
                uint32_t cur[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) cur[j] = page[j];
                if (kt + 1 < n_kt) fetch_pages(hf + 2);  // in flight while this half waits
                if (kt >= 2 &&
                    !wait_phase(&bars->raw_free[slot], (kt >> 1) - 1, s_abort, p.status, p.wait_ns, wait_tag(1, kBarRawFree, kt)))
                    break;
                uint8_t* dst = base + kSmRaw + slot * kRawHalf;
                uint32_t bytes = 0;
                const uint8_t* src[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int pt = hf * 4 + j;
                    src[j] = nullptr;
                    if (cur[j] < (uint32_t)p.n_pages)
                        src[j] = head_base + (size_t)cur[j] * page_stride + (pt % p.tpp) * kRawTileBytes;
                    else if (pt < pt_need)
                        atomicOr(p.status, YF_DEV_BAD_PAGE);
                    s_valid[slot * 4 + j] = src[j] != nullptr;
                    bytes += src[j] ? kRawTileBytes : 0;
                }
                mbar_arrive_expect_tx(&bars->raw_full[slot], bytes);
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (src[j]) bulk_g2s(dst + j * kRawPitch, src[j], kRawTileBytes, &bars->raw_full[slot]);
            }
        }
        __syncwarp();
    } else if (warp >= 8) {
        // ================= dequant: raw pool tiles -> f16 K and V^T =================
        const int t = tid - 256, dw = t >> 5;
        // K: lane -> (token g, dim octet tig) of a 512-byte block, paired so that each
        // quarter-warp's loads and swizzled stores hit eight distinct 16-byte bank groups
        const int qw = lane >> 3, k8 = lane & 7;
        const int kg = (k8 < 4) ? qw : (qw ^ 5), ktig = k8 & 3;
        // V: lane -> (dim bits 4, 3, 0; staged tile); warp and step give dim bits 5-6, 1-2
        const int vm1 = lane >> 4, vdh = (lane >> 3) & 1, vjt = (lane >> 1) & 3, vg1 = lane & 1;
        const uint32_t peer_sbase = peer_addr(sbase, peer);
        const uint32_t peer_k_full0 = peer_addr(smem_u32(&bars->k_full[0]), peer);
        const uint32_t peer_k_full1 = peer_addr(smem_u32(&bars->k_full[1]), peer);
        const uint32_t peer_v_full0 = peer_addr(smem_u32(&bars->v_full[0]), peer);
        const uint32_t peer_v_full1 = peer_addr(smem_u32(&bars->v_full[1]), peer);
        for (int j = 0; j < n_kt; ++j) {
            const int e = rank, slot = j & 1;  // half e of key tile j
            (void)wait_phase(&bars->raw_full[slot], j >> 1, s_abort, p.status, p.wait_ns, wait_tag(2, kBarRawFull, j));
            // stage j&1 was last read by QK(j-2) (K) and PV(j-2) (V^T), here and in the peer
            // K stage j&1 was last read by QK(j-2) here and in the peer
            if (j >= 2)
                (void)wait_phase(&bars->k_free[j & 1], (j >> 1) - 1, s_abort, p.status, p.wait_ns, wait_tag(2, kBarKFree, j));
            const uint8_t* raw = base + kSmRaw + slot * kRawHalf;
            const uint32_t kdst = sbase + kSmK + (j & 1) * 32768, vdst = sbase + kSmVt + (j & 1) * 32768 + e * 16384;
#pragma unroll
            for (int jt = 0; jt < 4; ++jt) {
                // K: tokens kg, kg+8 x dims 32dw + 8ktig .. +7 of pool tile jt
                const uint8_t* T = raw + jt * kRawPitch;
                uint4 o0 = make_uint4(0, 0, 0, 0), o1 = make_uint4(0, 0, 0, 0);
                if (s_valid[slot * 4 + jt]) {
                    const uint4 kw = lds128(T + dw * 512 + (kg * 4 + ktig) * 16);
                    // K scales [token%8][token/8][group]
                    // (the warp's 32 dims are scale group dw, or the row's one group)
                    const int sg = NB == 1 ? 0 : dw;
                    const uint16_t s0 = *reinterpret_cast<const uint16_t*>(T + 16 * kPfD + 2 * ((kg * 2) * NB + sg));
                    const uint16_t s1 =
                        *reinterpret_cast<const uint16_t*>(T + 16 * kPfD + 2 * ((kg * 2 + 1) * NB + sg));
                    const uint32_t d0 = (uint32_t)s0 | ((uint32_t)s0 << 16), d1 = (uint32_t)s1 | ((uint32_t)s1 << 16);
                    const uint32_t x0 = kw.x, x1 = kw.y, z0 = kw.z, z1 = kw.w;
                    o0 = make_uint4(dq2(x0, 0, d0), dq2(x0, 1, d0), dq2(x1, 0, d0), dq2(x1, 1, d0));
                    o1 = make_uint4(dq2(z0, 0, d1), dq2(z0, 1, d1), dq2(z1, 0, d1), dq2(z1, 1, d1));
                }
                const int key = e * 64 + jt * 16 + kg, c = dw * 4 + ktig;  // chunk c = dims 8c .. 8c+7
                sts128(kdst + sw128_off(key, c, kPfKeys), o0);
                sts128(kdst + sw128_off(key + 8, c, kPfKeys), o1);
            }
            fence_proxy_async_smem();
            asm volatile("bar.sync 2, 128;" ::: "memory");  // the four warps' K rows precede the copy
            if (t == 0) {
                // this half's K rows (64e .. 64e+63 of both column blocks) into the peer; its bytes
                // complete the peer's k_full, as the peer's do this CTA's (armed here)
                const uint32_t k0 = kdst + e * 64 * 128, k1 = kdst + 16384 + e * 64 * 128;
                const uint32_t pbar = (j & 1) ? peer_k_full1 : peer_k_full0;
                bulk_s2peer(peer_sbase + (k0 - sbase), k0, 8192, pbar);
                bulk_s2peer(peer_sbase + (k1 - sbase), k1, 8192, pbar);
                mbar_arrive_expect_tx(&bars->k_full[j & 1], 16384);
            } else if (lane == 0) {
                mbar_arrive(&bars->k_full[j & 1]);
            }
            // V^T stage j&1 was last read by PV(j-2) here and in the peer
            if (j >= 2)
                (void)wait_phase(&bars->v_free[j & 1], (j >> 1) - 1, s_abort, p.status, p.wait_ns, wait_tag(2, kBarVFree, j));
            // V: the thread's four dims share one scale group (dims 32dw .. 32dw+31) of tile vjt
            const uint8_t* TV = raw + vjt * kRawPitch;
            const bool vvalid = s_valid[slot * 4 + vjt] != 0;
            uint32_t sp[8];  // (token 2k, 2k+1) f16x2 for k = 0..7
            if (vvalid) {
                // V scales [tig][group][j]: pairs (2tig, 2tig+8), (2tig+1, 2tig+9)
                const uint8_t* vsc = TV + 32 * kPfD + 32 * NB + (NB == 1 ? 0 : dw) * 8;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint2 pr = lds64(vsc + q * 8 * NB);
                    sp[q] = __byte_perm(pr.x, pr.y, 0x5410);
                    sp[4 + q] = __byte_perm(pr.x, pr.y, 0x7632);
                }
            }
#pragma unroll
            for (int st = 0; st < 4; ++st) {
                // V^T row d, keys 16vjt .. +15 of this half: the four (token-pair) words of dim d
                // hold tokens {2tig, 2tig+8, 2tig+1, 2tig+9} for tig = 0..3
                const int d = 32 * dw + 16 * vm1 + 8 * vdh + 2 * st + vg1;
                const int m = d >> 4, gp = d & 7;
                uint4 lo = make_uint4(0, 0, 0, 0), hi = make_uint4(0, 0, 0, 0);
                if (vvalid) {
                    const uint8_t* vb = TV + 16 * kPfD + 32 * NB + (m >> 1) * 512 + ((m & 1) * 2 + vdh) * 4;
                    uint32_t wv[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q) wv[q] = lds32(vb + (gp * 4 + q) * 16);
                    // keys 0..7 = bytes 0,2 of wv[0..3]; keys 8..15 = bytes 1,3
                    const uint32_t k03 = __byte_perm(wv[0], wv[1], 0x6420), k47 = __byte_perm(wv[2], wv[3], 0x6420);
                    const uint32_t k8b = __byte_perm(wv[0], wv[1], 0x7531), kcf = __byte_perm(wv[2], wv[3], 0x7531);
                    const uint32_t a = k03, bq = k47, c8 = k8b, cf = kcf;
                    lo = make_uint4(dq2(a, 0, sp[0]), dq2(a, 1, sp[1]), dq2(bq, 0, sp[2]), dq2(bq, 1, sp[3]));
                    hi = make_uint4(dq2(c8, 0, sp[4]), dq2(c8, 1, sp[5]), dq2(cf, 0, sp[6]), dq2(cf, 1, sp[7]));
                }
                sts128(vdst + sw128_off(d, 2 * vjt, kPfD), lo);
                sts128(vdst + sw128_off(d, 2 * vjt + 1, kPfD), hi);
            }
            fence_proxy_async_smem();
            asm volatile("bar.sync 2, 128;" ::: "memory");  // the four warps' V^T columns precede the copy
            if (t == 0) {
                bulk_s2peer(peer_sbase + (vdst - sbase), vdst, 16384, (j & 1) ? peer_v_full1 : peer_v_full0);
                mbar_arrive_expect_tx(&bars->v_full[j & 1], 16384);
                mbar_arrive(&bars->raw_free[slot]);
            } else if (lane == 0) {
                mbar_arrive(&bars->v_full[j & 1]);
                mbar_arrive(&bars->raw_free[slot]);
            }
        }
    } else {
        // ================= softmax: thread = query row of tile qt =================
        const int qt = tid >> 7, row = tid;
        if (qt == 0 || act1) {
            const bool live = row < rows;
            const int kvlen = live ? max(0, min(Tk, kv0 + pos0 + row / p.G + 1)) : 0;
            const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
            const uint32_t tS = tmem + 256 + qt * 128 + lane_off, tP = tS + 64, tO = tmem + qt * 128 + lane_off;
            const float sl2 = p.scale_log2;
            float m_run = -INFINITY, l_run = 0.f;  // running max (scaled, base 2) and sum
            for (int it = 0; it < n_kt; ++it) {
                (void)wait_phase(&bars->s_full[qt], it, s_abort, p.status, p.wait_ns, wait_tag(3, kBarSFull, it));
                __syncwarp();
                tc_fence_after();
                const int key0 = it * kPfKeys, lim = kvlen - key0;
                uint32_t pm = 0xFFu;
                if (!pages_ok) {
#pragma unroll
                    for (int jt = 0; jt < 8; ++jt) {
                        const int pt = key0 / 16 + jt;
                        if (pt >= pt_total || __ldg(btrow + pt / p.tpp) >= (uint32_t)p.n_pages) pm &= ~(1u << jt);
                    }
                }
                // warp-uniform: both paths end in warp-collective TMEM accesses
                const bool full = __all_sync(0xffffffffu, pm == 0xFFu && lim >= kPfKeys);
                float v[64];
                tmem_ld64(tS, v);
                float mx = full ? row_max64<false>(v, 0, lim, pm) : row_max64<true>(v, 0, lim, pm);
                tmem_ld64(tS + 64, v);
                mx = fmaxf(mx, full ? row_max64<false>(v, 64, lim, pm) : row_max64<true>(v, 64, lim, pm));
                mx *= sl2;
                float alpha = 1.f;
                bool need = false;
                if (mx > m_run + kPfRescale) {
                    alpha = fast_exp2(m_run - mx);
                    m_run = mx;
                    l_run *= alpha;
                    need = it > 0;
                }
                if (__any_sync(0xffffffffu, need)) {
                    // PV(it-1) completed before QK(it) (committed in issue order): O_i is stable.
                    // Rare: S is reloaded afterwards rather than kept live across it.
#pragma unroll 1
                    for (int c0 = 0; c0 < kPfD; c0 += 32) {
                        float o[32];
                        uint32_t ob[32];
                        tmem_ld32(tO + c0, o);
#pragma unroll
                        for (int e = 0; e < 32; ++e) ob[e] = __float_as_uint(o[e] * alpha);
                        tmem_st32(tO + c0, ob);
                    }
                    tmem_ld64(tS + 64, v);
                }
                const float nm = m_run == -INFINITY ? 0.f : -m_run;
                // P over S columns 64..127: keys 64..127 first (their S columns are then free),
                // then keys 0..63
                float sum = full ? exp_store64<false>(v, 64, lim, pm, sl2, nm, tP + 32)
                                 : exp_store64<true>(v, 64, lim, pm, sl2, nm, tP + 32);
                tmem_ld64(tS, v);
                sum += full ? exp_store64<false>(v, 0, lim, pm, sl2, nm, tP) : exp_store64<true>(v, 0, lim, pm, sl2, nm, tP);
                l_run += sum;
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->p_full[qt]);
            }
            // ---- epilogue: thread r writes row r of O_i / l
            if (n_kt > 0) {
                (void)wait_phase(&bars->o_done[qt], 0, s_abort, p.status, p.wait_ns, wait_tag(3, kBarODone, 0));
                __syncwarp();
                tc_fence_after();
            }
            const float linv = l_run > 0.f ? 1.f / l_run : 0.f;
            uint4* orow = live ? reinterpret_cast<uint4*>(p.out + ((size_t)(qrow0 + pos0 + row / p.G) * p.Hq +
                                                                   (size_t)h * p.G + row % p.G) *
                                                                      kPfD)
                               : nullptr;
#pragma unroll
            for (int c0 = 0; c0 < kPfD; c0 += 32) {
                float o[32];
                if (n_kt > 0) {
                    tmem_ld32(tO + c0, o);
                } else {
#pragma unroll
                    for (int e = 0; e < 32; ++e) o[e] = 0.f;
                }
                if (live) {
#pragma unroll
                    for (int v = 0; v < 4; ++v)
                        orow[c0 / 8 + v] = make_uint4(pack_h2(o[8 * v] * linv, o[8 * v + 1] * linv),
                                                      pack_h2(o[8 * v + 2] * linv, o[8 * v + 3] * linv),
                                                      pack_h2(o[8 * v + 4] * linv, o[8 * v + 5] * linv),
                                                      pack_h2(o[8 * v + 6] * linv, o[8 * v + 7] * linv));
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kCtlWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPfTmemCols) : "memory");
    }
    cluster_sync();  // no CTA leaves while its peer may still address its shared memory
}

}  // namespace

// True when the tensor-core prefill kernel handles this call.
bool prefill_tc_applies(const yf_pool* pool, int n_q_heads, int max_seqlen_q) {
    if (pool->opts.prefill_kernel == YF_PREFILL_SPLITKV) return false;
    const yf_pool_desc& d = pool->desc;
    const int G = n_q_heads / d.n_kv_heads;
    return d.head_dim == kPfD && (d.group_size == 32 || d.group_size == d.head_dim) && kPfRows % G == 0 &&
           (long long)G * max_seqlen_q >= kPfRows;
}

int launch_prefill_tc(const AttnArgs& a) {
    const yf_pool_desc& d = a.pool->desc;
    PrefillParams p;
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
    p.scale_log2 = a.scale * 1.4426950408889634f;
    p.out = a.out;
    p.status = a.pool->d_status;
    p.wait_ns = wait_limit_ns(a.pool);
    const bool row_scale = d.group_size == d.head_dim;
    static LaunchCache cache4, cache1;
    const void* kern = row_scale ? (const void*)prefill_tc_kernel<1> : (const void*)prefill_tc_kernel<4>;
    const int rc = raise_smem_attr(kern, kSmAlloc, d.device, row_scale ? cache1 : cache4);
    if (rc) return rc;
    const int ppb = kPfTiles * kPfRows / p.G;
    const long long blocks = (a.max_seqlen_q + ppb - 1) / ppb;
    const dim3 grid((unsigned)((blocks + 1) / 2 * 2), d.n_kv_heads, a.batch);  // clusters of 2 along x
    if (grid.x > 0x7fffffffu) return fail(YF_E_UNSUPPORTED, "too many query rows");
    if (row_scale)
        prefill_tc_kernel<1><<<grid, kPfBlock, kSmAlloc, a.stream>>>(p);
    else
        prefill_tc_kernel<4><<<grid, kPfBlock, kSmAlloc, a.stream>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? YF_OK : cuda_fail(e, "prefill_tc launch");
}

}  // namespace yf
