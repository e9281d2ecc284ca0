// Causal chunked-prefill attention at head_dim 256 over the paged Q8_0 pool on the tcgen05
// tensor cores (the production model's attention shape: Hq 16, Hkv 2, D 256).
//
// Same call as the D=128 kernel (forward_attn_prefill_paged, docs/plans/2026-08-27-mtp-cuda-graphs.md:132,244-248):
// query row i of an entry sees keys 0 .. Tk - Tq + i.  At D=256 an O accumulator of 128 rows
// takes 256 TMEM columns, so a CTA holds one query tile (128 rows = 128/G query positions x the
// G q heads of a kv head), and Q itself lives in TMEM as the A operand of QK:
//   TMEM (512 columns): O [0,256) f32, Q [256,384) f16 pairs, S0 [384,448), S1 [448,512).
// Keys advance in tiles of 64.  Per key tile j:
//   S_{j&1} = Q K_j^T      tcgen05.mma kind::f16, A = Q from TMEM, B = K_j from shared memory
//                          (K-major, 128-byte swizzle, 4 column blocks of 64 dims), M = 128,
//                          N = 64 keys, K = 256;
//   P_j = softmax part     written as f16 pairs over the upper half of S_{j&1};
//   O += P_j V_j           A = P_j from TMEM, B = V_j^T from shared memory (256 dims x 64 keys),
//                          M = 128, N = 256, K = 64.
// S is double-buffered: QK(j+1) runs while the softmax of tile j does.  CTAs come in clusters
// of kCln covering adjacent row blocks of the same (entry, kv head); CTA e of a cluster copies
// and dequantizes dims [e 256/kCln, (e+1) 256/kCln) of every key (its share of each pool tile's
// K and V bytes, plus the tile's scales) and writes the f16 result into every CTA's shared
// memory, so each pool byte is dequantized once for kCln x 128 query rows (a CTA holds one query
// tile at D=256, so clusters of 4 bring the dequant per MMA flop down to the D=128 kernel's with
// its pairs of two-tile CTAs).
//
// Warp roles (14 warps):
//   * warps 0-3, softmax: thread r owns row r (TMEM lane r): Q row into TMEM at the start, then
//     per tile the row max, a lazy base-2 rescale of the running max (O rescaled in TMEM, after
//     the previous PV has completed), exponentials, f16 P into TMEM; the output row at the end;
//   * warps 4-7 / 8-11, dequant: this CTA's dims of each key tile -> f16 K [key][dim] / V^T
//     [dim][key], the two groups in parallel;
//   * warp 12, control (one lane): every MMA and commit;
//   * warp 13, copies: page ids a chunk ahead in its lanes; one lane bulk-copies the 4 pool tiles
//     of a key tile.
#include <cstdint>

#include "yf_device.cuh"
#include "yf_internal.h"
#include "yf_pfcommon.cuh"
#include "yf_tc.cuh"

namespace yf {
namespace {

constexpr int kQRows = 128;   // query rows per CTA (M of both MMAs)
constexpr int kKeys = 64;     // keys per key tile (N of S, K of PV)
constexpr int kD = 256;       // head dim (K of S, N of PV)
constexpr int kTmemCols = 512;
constexpr int kTmO = 0, kTmQ = 256, kTmS = 384;  // S_b at kTmS + 64 b
constexpr float kRescale = 8.0f;

constexpr int kCln = 2;              // CTAs per cluster
constexpr int kDpc = kD / kCln;       // dims each CTA dequantizes
static_assert(kDpc % 64 == 0 && kDpc >= 64, "whole K column blocks per CTA");
// Every CTA stages whole 16-token pool tiles (one bulk copy each: a copy costs ~50 ns to issue,
// so four per key tile rather than one per piece of a tile); staged tiles 16 B apart modulo 128 B.
template <int NB>
constexpr int tile_bytes() { return 32 * kD + 64 * NB; }
template <int NB>
constexpr int raw_pitch() { return (tile_bytes<NB>() - 16 + 127) / 128 * 128 + 16; }

constexpr int kSmK = 0;                    // K   [2 stages][4 col blocks of 64 dims][64 keys][128 B]
constexpr int kSmVt = kSmK + 2 * 32768;    // V^T [2 stages][256 dims][128 B]
constexpr int kSmRaw = kSmVt + 2 * 32768;  // raw [2 slots][4 pool tiles][pitch] (whole tiles)
template <int NB>
constexpr int sm_misc() { return kSmRaw + 2 * 4 * raw_pitch<NB>(); }
template <int NB>
constexpr int sm_alloc() { return sm_misc<NB>() + 256; }
constexpr int kWarps = 14;
constexpr int kBlock = kWarps * 32;
constexpr int kCtlWarp = 12;
constexpr int kCopyWarp = 13;

struct Params {
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
    uint64_t wait_ns;
};

struct Bars {
    uint64_t raw_full[2], raw_free[2];  // the 4 staged pool tiles of a key tile
    uint64_t k_full[2], v_full[2];      // K / V^T stage written (own share + the peers' copies)
    uint64_t k_free[2], v_free[2];      // K / V^T stage read by its MMA in every CTA of the cluster
    uint64_t s_full[2], p_full[2];      // per S buffer
    uint64_t q_ready;                   // Q rows in TMEM
    uint64_t pv_done;                   // every PV completion (the rescale waits for the last)
    uint64_t o_done;                    // last PV complete
    uint64_t drain;
};
static_assert(sizeof(Bars) <= 160, "barrier area");

template <int NB>
__global__ void __cluster_dims__(kCln, 1, 1) __launch_bounds__(kBlock, 1) prefill_tc256_kernel(const Params p) {
    constexpr int TB = tile_bytes<NB>(), PITCH = raw_pitch<NB>();
    static_assert(TB % 16 == 0 && PITCH >= TB, "staged tile");
    constexpr int SMISC = sm_misc<NB>();
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* base = smem_raw;
    const uint32_t sbase = smem_u32(smem_raw);
    Bars* bars = reinterpret_cast<Bars*>(base + SMISC);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + SMISC + 160);
    uint8_t* s_valid = base + SMISC + 168;  // [2][4] staged pool-tile flags
    volatile int* s_abort = reinterpret_cast<volatile int*>(base + SMISC + 176);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int b = blockIdx.z, h = blockIdx.y;
    const int ppb = kQRows / p.G;  // query positions per CTA

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
    if (sbase & 1023u) {  // the swizzled operand layouts need a 1024-aligned base
        if (tid == 0) atomicOr(p.status, YF_DEV_SMEM_ALIGN);
        return;
    }
    const int qrow0 = (int)p.cu_q[b];
    const int rank = (int)(blockIdx.x % kCln);  // rank in the cluster; dims [kDpc rank, +kDpc)
    const int pos0 = blockIdx.x * ppb, cl_pos0 = (blockIdx.x / kCln) * kCln * ppb;
    if (cl_pos0 >= Tq) return;  // every CTA of the cluster: no rows
    const int npos = max(0, min(ppb, Tq - pos0));  // a cluster's later CTAs may have none
    const int rows = npos * p.G;
    const int kv0 = Tk - Tq;  // keys before the chunk
    // every CTA streams the key tiles of the cluster's last row
    const int kv_hi = max(0, min(Tk, kv0 + cl_pos0 + min(kCln * ppb, Tq - cl_pos0)));
    const int n_kt = (kv_hi + kKeys - 1) / kKeys;
    const int pt_total = (Tk + 15) / 16;
    const int pt_need = (kv_hi + 15) / 16;  // pool tiles the cluster reads
    const uint32_t* btrow = p.bt + (size_t)b * p.max_blocks;
    const uint8_t* head_base = p.layer_base + (size_t)h * p.phb;
    const long long page_stride = p.phb * p.H;

    // ---- set-up
    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bars->raw_full[i], 1);
            mbar_init(&bars->raw_free[i], 8);  // the K and the V dequant warps
            mbar_init(&bars->k_full[i], 4);  // the dequant warps; the peers' shares come as bytes
            mbar_init(&bars->v_full[i], 4);
            mbar_init(&bars->k_free[i], kCln);  // every CTA's QK / PV of the stage
            mbar_init(&bars->v_free[i], kCln);
            mbar_init(&bars->s_full[i], 1);
            mbar_init(&bars->p_full[i], 4);
        }
        mbar_init(&bars->q_ready, 4);
        mbar_init(&bars->pv_done, 1);
        mbar_init(&bars->o_done, 1);
        mbar_init(&bars->drain, 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == kCtlWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    int bad = 0;
    if (warp >= 4 && warp < 8) {  // every page this CTA reads exists (the common case skips per-tile checks)
        for (int pt = tid - 128; pt < pt_need; pt += 128)
            if (__ldg(btrow + pt / p.tpp) >= (uint32_t)p.n_pages) bad = 1;
    }
    tc_fence_before();
    const bool pages_ok = __syncthreads_or(bad) == 0;
    tc_fence_after();
    cluster_sync();  // the peers' barriers are initialised before any remote arrival
    const uint32_t tmem = *tmem_slot;

    if (warp == kCtlWarp) {
        // ================= control: every MMA and commit =================
        if (lane == 0) {
            constexpr uint32_t IDESC_S = umma_idesc_f16(kQRows, kKeys);  // N = 64 keys
            constexpr uint32_t IDESC_O = umma_idesc_f16(kQRows, kD);     // N = 256 dims
            int qk = 0, pv = 0;
            uint32_t idle = 0;
            uint64_t idle_t0 = 0;
            const bool q_ok = n_kt == 0 || wait_phase(&bars->q_ready, 0, s_abort, p.status, p.wait_ns, wait_tag(1, kBarSFull, 0));
            while (q_ok && pv < n_kt && !*s_abort) {
                bool prog = false;
                // PV(pv): P in S buffer pv&1, V^T stage pv&1
                if (pv < qk && mbar_test(&bars->p_full[pv & 1], pv >> 1) && mbar_test(&bars->v_full[pv & 1], pv >> 1)) {
                    const int j = pv;
                    tc_fence_after();
                    const uint32_t tP = tmem + kTmS + (j & 1) * 64 + 32;
#pragma unroll
                    for (int ks = 0; ks < kKeys / 16; ++ks) {
                        const uint64_t bd = umma_desc_sw128(sbase + kSmVt + (j & 1) * 32768 + ks * 32);
                        umma_ts(tmem + kTmO, tP + ks * 8, bd, IDESC_O, (j > 0 || ks > 0) ? 1u : 0u);
                    }
                    umma_commit_mc(&bars->v_free[j & 1], (1u << kCln) - 1u);
                    umma_commit(&bars->pv_done);
                    if (j == n_kt - 1) umma_commit(&bars->o_done);
                    pv = j + 1;
                    prog = true;
                }
                // QK(qk) into S buffer qk&1, once PV(qk-2) (the buffer's last reader) is issued
                if (qk < n_kt && qk <= pv + 1 && mbar_test(&bars->k_full[qk & 1], qk >> 1)) {
                    const int j = qk;
                    tc_fence_after();
                    const uint32_t tS = tmem + kTmS + (j & 1) * 64;
#pragma unroll
                    for (int ks = 0; ks < kD / 16; ++ks) {
                        const uint64_t bd =
                            umma_desc_sw128(sbase + kSmK + (j & 1) * 32768 + (ks >> 2) * 8192 + (ks & 3) * 32);
                        umma_ts(tS, tmem + kTmQ + ks * 8, bd, IDESC_S, ks > 0 ? 1u : 0u);
                    }
                    umma_commit(&bars->s_full[j & 1]);
                    umma_commit_mc(&bars->k_free[j & 1], (1u << kCln) - 1u);
                    qk = j + 1;
                    prog = true;
                }
                if (prog) {
                    idle = 0;
                } else if (++idle == 1) {
                    idle_t0 = globaltimer_ns();
                } else if ((idle & 63u) == 0 && globaltimer_ns() - idle_t0 > p.wait_ns) {
                    give_up(s_abort, p.status, wait_tag(1, kBarIdle, (qk & 31) | ((pv & 31) << 5)));
                }
            }
            // every MMA of this CTA has completed before TMEM is released
            umma_commit(&bars->drain);
            if (!mbar_wait(&bars->drain, 0u, p.wait_ns)) give_up(s_abort, p.status, wait_tag(1, kBarDrain, 0));
        }
        __syncwarp();
    } else if (warp == kCopyWarp) {
        // ================= copies: the 4 pool tiles of each key tile =================
        // page ids of pool tiles [32c, 32c + 32) sit in the lanes' registers, the next chunk's
        // loads in flight one chunk ahead; lane 0 issues the copies
        auto load_chunk = [&](int c) -> uint32_t {
            const int pt = c * 32 + lane;
            return pt < pt_need ? __ldg(btrow + pt / p.tpp) : (uint32_t)p.n_pages;
        };
        uint32_t pg_cur = load_chunk(0), pg_next = load_chunk(1);
        for (int kt = 0; kt < n_kt; ++kt) {
            const int slot = kt & 1;
            if (kt > 0 && (kt & 7) == 0) {
                pg_cur = pg_next;
                pg_next = load_chunk((kt >> 3) + 1);
            }
            uint32_t cur[4];
#pragma unroll
            for (int jt = 0; jt < 4; ++jt) cur[jt] = __shfl_sync(0xffffffffu, pg_cur, ((kt & 7) << 2) + jt);
            bool ok = true;
            if (lane == 0 && kt >= 2)
                ok = wait_phase(&bars->raw_free[slot], (kt >> 1) - 1, s_abort, p.status, p.wait_ns, wait_tag(1, kBarRawFree, kt));
            if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
            if (lane == 0) {
                uint8_t* dst = base + kSmRaw + slot * 4 * PITCH;
                uint32_t bytes = 0;
                const uint8_t* src[4];
#pragma unroll
                for (int jt = 0; jt < 4; ++jt) {
                    const int pt = kt * 4 + jt;
                    src[jt] = nullptr;
                    if (cur[jt] < (uint32_t)p.n_pages)
                        src[jt] = head_base + (size_t)cur[jt] * page_stride + (pt % p.tpp) * TB;
                    else if (pt < pt_need)
                        atomicOr(p.status, YF_DEV_BAD_PAGE);
                    s_valid[slot * 4 + jt] = src[jt] != nullptr;
                    bytes += src[jt] ? TB : 0;
                }
                mbar_arrive_expect_tx(&bars->raw_full[slot], bytes);
#pragma unroll
                for (int jt = 0; jt < 4; ++jt)
                    if (src[jt]) bulk_g2s(dst + jt * PITCH, src[jt], TB, &bars->raw_full[slot]);
            }
        }
        __syncwarp();
    } else if (warp >= 4) {
        // ================= dequant: staged tiles -> f16 K (warps 4-7) and V^T (warps 8-11) =================
        // The two groups convert the same staged tiles in parallel.  kDpc / 32 blocks of 32 dims;
        // warp dw of a group takes block db = dw / WPB and, when two warps share a block, half of
        // its pool tiles (K) or half of its dim steps (V)
        constexpr int NBLK = kDpc / 32, WPB = 4 / NBLK, JT = 4 / WPB;
        const bool kgrp = warp < 8;
        const int t = tid - (kgrp ? 128 : 256), dw = t >> 5, db = dw / WPB, part = dw % WPB;
        const int sg = NB == 1 ? 0 : kDpc / 32 * rank + db;  // the scale group of the block
        // K: lane -> (token g, dim octet tig) of a 512-byte block, paired so that each
        // quarter-warp's loads and swizzled stores hit eight distinct 16-byte bank groups
        const int qw = lane >> 3, k8 = lane & 7;
        const int kg = (k8 < 4) ? qw : (qw ^ 5), ktig = k8 & 3;
        // V: lane -> (dim bits 4, 3, 0; staged tile); block and step give dim bits 5-6, 1-2
        const int vm1 = lane >> 4, vdh = (lane >> 3) & 1, vjt = (lane >> 1) & 3, vg1 = lane & 1;
        // K column: global dims kDpc rank + 32 db + 8 ktig .. +7 -> column block and chunk
        const int kdim = kDpc * rank + 32 * db + 8 * ktig;
        const int kc = (kdim >> 6) * 8 + ((kdim & 63) >> 3);
        constexpr uint32_t SHARE = kDpc * 128;  // bytes of this CTA's K columns, and of its V^T rows
        for (int j = 0; j < n_kt; ++j) {
            const int slot = j & 1;
            (void)wait_phase(&bars->raw_full[slot], j >> 1, s_abort, p.status, p.wait_ns, wait_tag(2, kBarRawFull, j));
            const uint8_t* raw = base + kSmRaw + slot * 4 * PITCH;
            const uint32_t kdst = sbase + kSmK + slot * 32768, vdst = sbase + kSmVt + slot * 32768;
            if (kgrp) {
            // K stage j&1 was last read by QK(j-2), in every CTA of the cluster
            if (j >= 2)
                (void)wait_phase(&bars->k_free[slot], (j >> 1) - 1, s_abort, p.status, p.wait_ns, wait_tag(2, kBarKFree, j));
#pragma unroll
            for (int i = 0; i < JT; ++i) {
                // K: tokens kg, kg+8 x dims 32db + 8ktig .. +7 (of this share) of pool tile jt
                const int jt = part * JT + i;
                const uint8_t* T = raw + jt * PITCH;
                uint4 o0 = make_uint4(0, 0, 0, 0), o1 = make_uint4(0, 0, 0, 0);
                if (s_valid[slot * 4 + jt]) {
                    const uint4 kw = lds128(T + (kDpc / 32 * rank + db) * 512 + (kg * 4 + ktig) * 16);
                    // K scales [token%8][token/8][group]
                    const uint8_t* ks = T + 16 * kD;
                    const uint16_t s0 = *reinterpret_cast<const uint16_t*>(ks + 2 * ((kg * 2) * NB + sg));
                    const uint16_t s1 = *reinterpret_cast<const uint16_t*>(ks + 2 * ((kg * 2 + 1) * NB + sg));
                    const uint32_t d0 = (uint32_t)s0 | ((uint32_t)s0 << 16), d1 = (uint32_t)s1 | ((uint32_t)s1 << 16);
                    o0 = make_uint4(dq2(kw.x, 0, d0), dq2(kw.x, 1, d0), dq2(kw.y, 0, d0), dq2(kw.y, 1, d0));
                    o1 = make_uint4(dq2(kw.z, 0, d1), dq2(kw.z, 1, d1), dq2(kw.w, 0, d1), dq2(kw.w, 1, d1));
                }
                const int key = jt * 16 + kg;
                sts128(kdst + sw128_off(key, kc, kKeys), o0);
                sts128(kdst + sw128_off(key + 8, kc, kKeys), o1);
            }
            fence_proxy_async_smem();
            asm volatile("bar.sync 2, 128;" ::: "memory");  // the four warps' K columns precede the copies
            if (t == 0) {
                // this CTA's K columns into every other CTA of the cluster; their bytes complete
                // those CTAs' k_full, as theirs do this CTA's (armed here)
                const uint32_t k0 = kdst + (kDpc * rank / 64) * 8192;
#pragma unroll
                for (int q = 1; q < kCln; ++q) {
                    const uint32_t peer = (uint32_t)((rank + q) % kCln);
                    bulk_s2peer(peer_addr(k0, peer), k0, SHARE, peer_addr(smem_u32(&bars->k_full[slot]), peer));
                }
                mbar_arrive_expect_tx(&bars->k_full[slot], (kCln - 1) * SHARE);
                mbar_arrive(&bars->raw_free[slot]);
            } else if (lane == 0) {
                mbar_arrive(&bars->k_full[slot]);
                mbar_arrive(&bars->raw_free[slot]);
            }
            } else {
            // V^T stage j&1 was last read by PV(j-2), in every CTA of the cluster
            if (j >= 2)
                (void)wait_phase(&bars->v_free[slot], (j >> 1) - 1, s_abort, p.status, p.wait_ns, wait_tag(2, kBarVFree, j));
            // V: the block's dims share one scale group; tile vjt
            const uint8_t* TV = raw + vjt * PITCH;
            const bool vvalid = s_valid[slot * 4 + vjt] != 0;
            uint32_t sp[8];  // (token 2k, 2k+1) f16x2 for k = 0..7
            if (vvalid) {
                // V scales [tig][group][j]: pairs (2tig, 2tig+8), (2tig+1, 2tig+9)
                const uint8_t* vsc = TV + 32 * kD + 32 * NB + sg * 8;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint2 pr = lds64(vsc + q * 8 * NB);
                    sp[q] = __byte_perm(pr.x, pr.y, 0x5410);
                    sp[4 + q] = __byte_perm(pr.x, pr.y, 0x7632);
                }
            }
#pragma unroll
            for (int i = 0; i < 4 / WPB; ++i) {
                // V^T row kDpc rank + d, keys 16vjt .. +15 of the tile
                const int st = part * (4 / WPB) + i;
                const int d = 32 * db + 16 * vm1 + 8 * vdh + 2 * st + vg1;
                const int m = d >> 4, gp = d & 7;
                uint4 lo = make_uint4(0, 0, 0, 0), hi = make_uint4(0, 0, 0, 0);
                if (vvalid) {
                    // V of global dim kDpc rank + d: 512-byte block (kDpc rank + d) / 32
                    const uint8_t* vb = TV + 16 * kD + 32 * NB + (kDpc / 32 * rank + (m >> 1)) * 512 + ((m & 1) * 2 + vdh) * 4;
                    uint32_t wv[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q) wv[q] = lds32(vb + (gp * 4 + q) * 16);
                    // keys 0..7 = bytes 0,2 of wv[0..3]; keys 8..15 = bytes 1,3
                    const uint32_t k03 = __byte_perm(wv[0], wv[1], 0x6420), k47 = __byte_perm(wv[2], wv[3], 0x6420);
                    const uint32_t k8b = __byte_perm(wv[0], wv[1], 0x7531), kcf = __byte_perm(wv[2], wv[3], 0x7531);
                    lo = make_uint4(dq2(k03, 0, sp[0]), dq2(k03, 1, sp[1]), dq2(k47, 0, sp[2]), dq2(k47, 1, sp[3]));
                    hi = make_uint4(dq2(k8b, 0, sp[4]), dq2(k8b, 1, sp[5]), dq2(kcf, 0, sp[6]), dq2(kcf, 1, sp[7]));
                }
                sts128(vdst + sw128_off(kDpc * rank + d, 2 * vjt, kD), lo);
                sts128(vdst + sw128_off(kDpc * rank + d, 2 * vjt + 1, kD), hi);
            }
            fence_proxy_async_smem();
            asm volatile("bar.sync 3, 128;" ::: "memory");  // the four warps' V^T rows precede the copies
            if (t == 0) {
                const uint32_t v0 = vdst + kDpc * rank * 128;  // rows kDpc rank .. +kDpc-1
#pragma unroll
                for (int q = 1; q < kCln; ++q) {
                    const uint32_t peer = (uint32_t)((rank + q) % kCln);
                    bulk_s2peer(peer_addr(v0, peer), v0, SHARE, peer_addr(smem_u32(&bars->v_full[slot]), peer));
                }
                mbar_arrive_expect_tx(&bars->v_full[slot], (kCln - 1) * SHARE);
                mbar_arrive(&bars->raw_free[slot]);
            } else if (lane == 0) {
                mbar_arrive(&bars->v_full[slot]);
                mbar_arrive(&bars->raw_free[slot]);
            }
            }
        }
    } else {
        // ================= softmax: thread = query row =================
        const int row = tid;
        const bool live = row < rows;
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        // Q row (position pos0 + row/G, head h*G + row%G) into TMEM columns kTmQ .. +127
        {
            const uint4* qp = live ? reinterpret_cast<const uint4*>(
                                         p.q + ((size_t)(qrow0 + pos0 + row / p.G) * p.Hq + (size_t)h * p.G + row % p.G) * kD)
                                   : nullptr;
#pragma unroll
            for (int c0 = 0; c0 < 4; ++c0) {
                uint32_t w[32];
#pragma unroll
                for (int v = 0; v < 8; ++v) {
                    const uint4 x = live ? __ldg(qp + c0 * 8 + v) : make_uint4(0, 0, 0, 0);
                    w[4 * v] = x.x;
                    w[4 * v + 1] = x.y;
                    w[4 * v + 2] = x.z;
                    w[4 * v + 3] = x.w;
                }
                tmem_st32(tmem + kTmQ + lane_off + c0 * 32, w);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->q_ready);
        }
        const int kvlen = live ? max(0, min(Tk, kv0 + pos0 + row / p.G + 1)) : 0;
        const uint32_t tO = tmem + kTmO + lane_off;
        const float sl2 = p.scale_log2;
        float m_run = -INFINITY, l_run = 0.f;  // running max (scaled, base 2) and sum
        for (int it = 0; it < n_kt; ++it) {
            const int sb = it & 1;
            (void)wait_phase(&bars->s_full[sb], it >> 1, s_abort, p.status, p.wait_ns, wait_tag(3, kBarSFull, it));
            __syncwarp();
            tc_fence_after();
            const uint32_t tS = tmem + kTmS + sb * 64 + lane_off;
            const int key0 = it * kKeys, lim = kvlen - key0;
            uint32_t pm = 0xFu;
            if (!pages_ok) {
#pragma unroll
                for (int jt = 0; jt < 4; ++jt) {
                    const int pt = key0 / 16 + jt;
                    if (pt >= pt_total || __ldg(btrow + pt / p.tpp) >= (uint32_t)p.n_pages) pm &= ~(1u << jt);
                }
            }
            // warp-uniform: both paths end in warp-collective TMEM accesses
            const bool full = __all_sync(0xffffffffu, pm == 0xFu && lim >= kKeys);
            float v[64];
            tmem_ld64(tS, v);
            float mx = full ? row_max64<false>(v, 0, lim, pm) : row_max64<true>(v, 0, lim, pm);
            mx *= sl2;
            float alpha = 1.f;
            bool need = false;
            if (mx > m_run + kRescale) {
                alpha = fast_exp2(m_run - mx);
                m_run = mx;
                l_run *= alpha;
                need = it > 0;
            }
            if (__any_sync(0xffffffffu, need)) {
                // O is stable once PV(it-1) has completed (QK(it) may have run ahead of it)
                (void)wait_phase(&bars->pv_done, it - 1, s_abort, p.status, p.wait_ns, wait_tag(3, kBarODone, it));
                __syncwarp();
                tc_fence_after();
#pragma unroll 1
                for (int c0 = 0; c0 < kD; c0 += 32) {
                    float o[32];
                    uint32_t ob[32];
                    tmem_ld32(tO + c0, o);
#pragma unroll
                    for (int e = 0; e < 32; ++e) ob[e] = __float_as_uint(o[e] * alpha);
                    tmem_st32(tO + c0, ob);
                }
            }
            const float nm = m_run == -INFINITY ? 0.f : -m_run;
            // P of the 64 keys over S columns 32..63 (every S value is in registers)
            const float sum = full ? exp_store64<false>(v, 0, lim, pm, sl2, nm, tS + 32)
                                   : exp_store64<true>(v, 0, lim, pm, sl2, nm, tS + 32);
            l_run += sum;
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->p_full[sb]);
        }
        // ---- epilogue: thread r writes row r of O / l
        if (n_kt > 0) {
            (void)wait_phase(&bars->o_done, 0, s_abort, p.status, p.wait_ns, wait_tag(3, kBarODone, 0));
            __syncwarp();
            tc_fence_after();
        }
        const float linv = l_run > 0.f ? 1.f / l_run : 0.f;
        uint4* orow = live ? reinterpret_cast<uint4*>(p.out + ((size_t)(qrow0 + pos0 + row / p.G) * p.Hq +
                                                               (size_t)h * p.G + row % p.G) *
                                                                  kD)
                           : nullptr;
#pragma unroll 1
        for (int c0 = 0; c0 < kD; c0 += 32) {
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
    tc_fence_before();
    __syncthreads();
    if (warp == kCtlWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
    cluster_sync();  // no CTA leaves while a peer may still address its shared memory
}

}  // namespace

// True when the D=256 tensor-core prefill kernel handles this call.
bool prefill_tc256_applies(const yf_pool* pool, int n_q_heads, int max_seqlen_q) {
    if (pool->opts.prefill_kernel == YF_PREFILL_SPLITKV) return false;
    const yf_pool_desc& d = pool->desc;
    const int G = n_q_heads / d.n_kv_heads;
    return d.head_dim == kD && (d.group_size == 32 || d.group_size == d.head_dim) && kQRows % G == 0 &&
           (long long)G * max_seqlen_q >= kQRows;
}

int launch_prefill_tc256(const AttnArgs& a) {
    const yf_pool_desc& d = a.pool->desc;
    Params p;
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
    static LaunchCache cache8, cache1;
    const void* kern = row_scale ? (const void*)prefill_tc256_kernel<1> : (const void*)prefill_tc256_kernel<8>;
    const int smem = row_scale ? sm_alloc<1>() : sm_alloc<8>();
    const int rc = raise_smem_attr(kern, smem, d.device, row_scale ? cache1 : cache8);
    if (rc) return rc;
    const int ppb = kQRows / p.G;
    const long long blocks = (a.max_seqlen_q + ppb - 1) / ppb;
    const dim3 grid((unsigned)((blocks + kCln - 1) / kCln * kCln), d.n_kv_heads, a.batch);  // clusters along x
    if (grid.x > 0x7fffffffu) return fail(YF_E_UNSUPPORTED, "too many query rows");
    if (row_scale)
        prefill_tc256_kernel<1><<<grid, kBlock, smem, a.stream>>>(p);
    else
        prefill_tc256_kernel<8><<<grid, kBlock, smem, a.stream>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? YF_OK : cuda_fail(e, "prefill_tc256 launch");
}

}  // namespace yf
