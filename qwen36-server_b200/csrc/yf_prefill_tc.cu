// Causal chunked-prefill attention over the paged Q8_0 pool on the 5th-generation
// tensor cores (tcgen05, TMEM accumulators).
//
// Replaces the prefill branch of the engine's FA2 varlen split-KV call from
// forward_attn_prefill_paged (docs/plans/2026-08-27-mtp-cuda-graphs.md:132,244-248;
// QK_INT8_PREFILL described at docs/research/2026-09-16-head-to-head-llamacpp-and-phase-profile.md:3627-3634):
// query row i of an entry sees keys 0 .. Tk - Tq + i.
//
// One CTA = one entry, one kv head, 128 query rows = 128/G query positions x the G q heads
// of the kv head (GQA folded into M, so every key tile is dequantized once for all of them).
// The CTA's nine warps are specialised and hand 64-key tiles to each other through
// mbarriers, double-buffered so that the stages of consecutive tiles overlap:
//   * control warp (lane 0): bulk-copies the four 16-token pool tiles of a key tile (K+V int8
//     + scales, one contiguous block each) into a raw staging buffer two tiles ahead, and
//     issues the MMAs: S = Q K^T (M=128 rows, N=64 keys, K=128 dims: 8 x tcgen05.mma
//     kind::f16, f32 in TMEM) and O^T += V^T P^T (M=128 dims, N=128 rows, K=64 keys: 4 MMAs);
//   * 4 dequant warps: int8 K -> f16 [key][dim], int8 V -> f16 V^T [dim][key], both in the
//     K-major 128-byte-swizzled layout the MMA descriptors describe;
//   * 4 softmax warps: thread r owns query row r (TMEM lane r of S): scale, causal mask,
//     online base-2 softmax with lazy rescale, P (f16) to shared memory; when a row's max
//     moved they rescale O^T in TMEM (thread d owns lane d) before the next PV.
// At the end thread d reads lane d of O^T (all 128 rows) and writes out[row][d] / l[row].
#include <cstdint>
#include <cstdlib>

#include "yf_device.cuh"
#include "yf_internal.h"

namespace yf {
namespace {

constexpr int kPfRows = 128;     // query rows per CTA (M of S, N of O^T)
constexpr int kPfKeys = 64;      // keys per tile (N of S, K of O^T)
constexpr int kPfD = 128;        // head dim (K of S, M of O^T)
constexpr int kPfTmemCols = 256; // S[2]: cols [0,128), O^T: cols [128,256)
constexpr float kPfRescale = 8.0f;  // lazy rescale threshold (base 2), as in the decode kernels

// shared-memory map (bytes from a 1024-aligned base); [n] = ring of n buffers
constexpr int kSmQ = 0;                         // Q   [128 rows][128 d] f16: 2 column blocks x 16 KB
constexpr int kSmK = kSmQ + 32768;              // K   [2][64 keys][128 d] f16 (2 column blocks x 8 KB)
constexpr int kSmVt = kSmK + 2 * 16384;         // V^T [3][128 d][64 keys] f16
constexpr int kSmP = kSmVt + 3 * 16384;         // P   [2][128 rows][64 keys] f16
constexpr int kSmRaw = kSmP + 2 * 16384;        // raw [3][4 pool tiles x 4352 B]
constexpr int kRawTileBytes = 4352;             // D=128, group 32
constexpr int kRawBytes = 4 * kRawTileBytes;    // one 64-key tile
constexpr int kSmMisc = kSmRaw + 3 * kRawBytes;
// misc: Bars at +0 (< 256 B), TMEM address at +256, alpha[2][128] at +512, 1/l[128] at +1536,
// pool-tile flags [3][4] at +2048, abort word at +2064
constexpr int kSmBytes = kSmMisc + 4096;
constexpr int kSmAlloc = kSmBytes + 1024;       // + alignment slack
constexpr int kPfWarps = 9;                     // 4 softmax, 4 dequant, 1 control
constexpr int kPfBlock = kPfWarps * 32;

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
};

// ---- tcgen05 / UMMA helpers ----------------------------------------------------------

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    const uint64_t start = (saddr >> 4) & 0x3FFFu;
    const uint64_t lbo = 1;           // (16 B) >> 4: unused by swizzled K-major layouts
    const uint64_t sbo = 1024 >> 4;   // next 8-row group
    return start | (lbo << 16) | (sbo << 32) | (1ull << 46) /* sm100 version */ | (2ull << 61) /* SWIZZLE_128B */;
}

// Instruction descriptor of kind::f16: f16 A and B, f32 accumulator, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N) {
    return (1u << 4)                         // D format f32
           | (0u << 7) | (0u << 10)          // A, B f16
           | ((uint32_t)(N >> 3) << 17)      // N / 8
           | ((uint32_t)(M >> 4) << 24);     // M / 16
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accum)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive TMEM columns of this thread's lane (warp w reads lanes 32w..32w+31).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])),
        "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
        "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])),
        "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}

__device__ __forceinline__ void sts128(uint32_t saddr, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(saddr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

// Byte offset of 16-byte chunk `c` (8 f16) of row `r` in a K-major SW128 tile whose rows are
// 128 B (64 f16) wide; column blocks of `rows` rows follow each other.
__device__ __forceinline__ uint32_t sw128_off(int r, int c, int rows) {
    const int kb = c >> 3, cc = c & 7;
    return (uint32_t)(kb * rows * 128 + (r >> 3) * 1024 + (r & 7) * 128 + ((cc ^ (r & 7)) << 4));
}

// f16x2 of bytes (lo, hi) of a biased word, times an f16x2 scale pair.
__device__ __forceinline__ uint32_t dq2(uint32_t biased, int sel, uint32_t scale2) {
    const uint32_t h = sel ? s8hi_to_h2(biased) : s8lo_to_h2(biased);
    return h2mul(h, scale2);
}

// True for every thread of the 4 softmax warps when any of them passes true.
__device__ __forceinline__ bool softmax_any(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\t"
        "bar.red.or.pred po, 1, 128, pi;\n\tselp.u32 %0, 1, 0, po;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ void softmax_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

struct Bars {
    uint64_t raw_full[3], raw_free[3], vt_free[3], kv_full[2], s_full[2], s_free[2], p_full[2], pv_done[2], drain;
};
static_assert(sizeof(Bars) <= 256, "barrier area");

__device__ __forceinline__ bool mbar_test(uint64_t* bar, int use) {  // non-blocking: use-th completion done?
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"((uint32_t)use & 1u)
        : "memory");
    return ok != 0;
}

// Bounded wait for the use-th completion (0-based) of `bar`.  A wait that gives up raises the
// CTA's abort flag, after which every role skips its remaining waits and drains quickly.
__device__ __forceinline__ bool wait_phase(uint64_t* bar, int use, volatile int* abort) {
    if (*abort) return false;
    for (uint32_t i = 0; i < kMaxWaitIters; ++i) {
        if (mbar_try_wait(bar, (uint32_t)use & 1u)) return true;
        if ((i & 255u) == 255u && *abort) return false;
    }
    *abort = 1;
    return false;
}

__global__ void __launch_bounds__(kPfBlock, 1) prefill_tc_kernel(const PrefillParams p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t sraw = smem_u32(smem_raw);
    const uint32_t sbase = (sraw + 1023u) & ~1023u;
    uint8_t* base = smem_raw + (sbase - sraw);
    Bars* bars = reinterpret_cast<Bars*>(base + kSmMisc);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + kSmMisc + 256);
    float* s_alpha = reinterpret_cast<float*>(base + kSmMisc + 512);     // [2][128]
    float* s_linv = s_alpha + 2 * kPfRows;                                  // [128]
    uint8_t* s_valid = reinterpret_cast<uint8_t*>(s_linv + kPfRows);      // [3][4] pool-tile flags
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_valid + 16);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int b = blockIdx.z, h = blockIdx.y;
    const int ppb = kPfRows / p.G;  // query positions per CTA

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
    const int qrow0 = (int)p.cu_q[b];
    const int pos0 = blockIdx.x * ppb;
    if (pos0 >= Tq) return;
    const int npos = min(ppb, Tq - pos0);
    const int rows = npos * p.G;
    const int kv0 = Tk - Tq;  // keys before the chunk
    const int kv_hi = max(0, min(Tk, kv0 + pos0 + npos));
    const int kv_lo = max(0, min(Tk, kv0 + pos0 + 1));  // every row sees keys [0, kv_lo)
    const int n_kt = (kv_hi + kPfKeys - 1) / kPfKeys;
    const int pt_total = (Tk + 15) / 16;
    const uint32_t* btrow = p.bt + (size_t)b * p.max_blocks;
    const uint8_t* head_base = p.layer_base + (size_t)h * p.phb;
    const long long page_stride = p.phb * p.H;

    // ---- set-up
    if (tid == 0) {
        for (int i = 0; i < 3; ++i) {
            mbar_init(&bars->raw_full[i], 1);
            mbar_init(&bars->raw_free[i], 4);
            mbar_init(&bars->vt_free[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bars->kv_full[i], 4);
            mbar_init(&bars->s_full[i], 1);
            mbar_init(&bars->s_free[i], 4);
            mbar_init(&bars->p_full[i], 4);
            mbar_init(&bars->pv_done[i], 1);
        }
        mbar_init(&bars->drain, 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 8) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kPfTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (warp < 4) {
        // Q row `tid` (position pos0 + tid/G, head h*G + tid%G) into the SW128 Q tile
        const bool live = tid < rows;
        const uint4 zero = make_uint4(0, 0, 0, 0);
        const uint4* qp = nullptr;
        if (live)
            qp = reinterpret_cast<const uint4*>(
                p.q + ((size_t)(qrow0 + pos0 + tid / p.G) * p.Hq + (size_t)h * p.G + tid % p.G) * kPfD);
#pragma unroll
        for (int c = 0; c < 16; ++c) sts128(sbase + kSmQ + sw128_off(tid, c, kPfRows), live ? __ldg(qp + c) : zero);
        fence_proxy_async_smem();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool timed_out = false;

    if (warp == 8) {
        // ================= control: bulk copies and MMAs =================
        if (lane == 0) {
            auto issue_raw = [&](int kt, int buf) {
                uint8_t* dst = base + kSmRaw + buf * kRawBytes;
                uint32_t bytes = 0;
                const uint8_t* src[4];
                for (int j = 0; j < 4; ++j) {
                    const int pt = kt * 4 + j;
                    src[j] = nullptr;
                    if (pt < pt_total) {
                        const uint32_t page = __ldg(btrow + pt / p.tpp);
                        if (page < (uint32_t)p.n_pages)
                            src[j] = head_base + (size_t)page * page_stride + (pt % p.tpp) * kRawTileBytes;
                        else
                            atomicOr(p.status, YF_DEV_BAD_PAGE);
                    }
                    s_valid[buf * 4 + j] = src[j] != nullptr;
                    bytes += src[j] ? kRawTileBytes : 0;
                }
                mbar_arrive_expect_tx(&bars->raw_full[buf], bytes);
                for (int j = 0; j < 4; ++j)
                    if (src[j]) bulk_g2s(dst + j * kRawTileBytes, src[j], kRawTileBytes, &bars->raw_full[buf]);
            };
            constexpr uint32_t IDESC_S = umma_idesc_f16(kPfRows, kPfKeys);
            constexpr uint32_t IDESC_O = umma_idesc_f16(kPfD, kPfRows);
            // Polling loop: issue whichever of {next raw copy, next QK, next PV} is ready.
            // QK runs at most 2 tiles ahead of PV (two S buffers; keeps every parity wait
            // within one phase of its barrier).
            int qk = 0, pv = 0, rw = 0;
            uint32_t idle = 0;
            while (pv < n_kt && !*s_abort) {
                bool prog = false;
                if (rw < n_kt && (rw < 3 || mbar_test(&bars->raw_free[rw % 3], rw / 3 - 1))) {
                    issue_raw(rw, rw % 3);
                    ++rw;
                    prog = true;
                }
                if (qk < n_kt && qk < pv + 2 && mbar_test(&bars->kv_full[qk & 1], qk >> 1) &&
                    (qk < 2 || mbar_test(&bars->s_free[qk & 1], (qk - 2) >> 1))) {
                    const int b2 = qk & 1;
                    tc_fence_after();
#pragma unroll
                    for (int ks = 0; ks < kPfD / 16; ++ks) {
                        const uint64_t a = umma_desc_sw128(sbase + kSmQ + (ks >> 2) * (kPfRows * 128) + (ks & 3) * 32);
                        const uint64_t bd =
                            umma_desc_sw128(sbase + kSmK + b2 * 16384 + (ks >> 2) * (kPfKeys * 128) + (ks & 3) * 32);
                        umma_f16(tmem + b2 * 64, a, bd, IDESC_S, ks > 0);
                    }
                    umma_commit(&bars->s_full[b2]);
                    ++qk;
                    prog = true;
                }
                if (pv < qk && mbar_test(&bars->p_full[pv & 1], pv >> 1)) {
                    const int bp = pv & 1, bv = pv % 3;
                    tc_fence_after();
#pragma unroll
                    for (int ks = 0; ks < kPfKeys / 16; ++ks) {
                        const uint64_t a = umma_desc_sw128(sbase + kSmVt + bv * 16384 + ks * 32);
                        const uint64_t bd = umma_desc_sw128(sbase + kSmP + bp * 16384 + ks * 32);
                        umma_f16(tmem + 128, a, bd, IDESC_O, (pv > 0 || ks > 0) ? 1u : 0u);
                    }
                    umma_commit(&bars->pv_done[bp]);
                    umma_commit(&bars->vt_free[bv]);
                    ++pv;
                    prog = true;
                }
                if (prog) {
                    idle = 0;
                } else if (++idle > 4u * kMaxWaitIters) {
                    *s_abort = 1;
                    timed_out = true;
                }
            }
            // every MMA of this CTA has completed before TMEM is released
            umma_commit(&bars->drain);
            (void)mbar_wait(&bars->drain, 0u);
        }
        __syncwarp();
    } else if (warp >= 4) {
        // ================= dequant: raw pool tiles -> f16 K and V^T =================
        const int t = tid - 128;
        for (int it = 0; it < n_kt; ++it) {
            const int b2 = it & 1, b3 = it % 3;
            if (!wait_phase(&bars->raw_full[b3], it / 3, s_abort)) timed_out = true;
            // K[b2] was read by QK(it-2), V^T[b3] by PV(it-3)
            if (it >= 2 && !wait_phase(&bars->s_full[b2], (it - 2) >> 1, s_abort)) timed_out = true;
            if (it >= 3 && !wait_phase(&bars->vt_free[b3], it / 3 - 1, s_abort)) timed_out = true;
            const uint8_t* raw = base + kSmRaw + b3 * kRawBytes;
            const uint32_t kdst = sbase + kSmK + b2 * 16384, vdst = sbase + kSmVt + b3 * 16384;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                // K: 16-byte word w of pool tile j = tokens g, g+8 x dims 32cb+8tig .. +7
                const int w = t + i * 128;
                const int j = w >> 7, cb = (w & 127) >> 5, ln = w & 31, g = ln >> 2, tig = ln & 3;
                const uint8_t* T = raw + j * kRawTileBytes;
                uint4 o0 = make_uint4(0, 0, 0, 0), o1 = make_uint4(0, 0, 0, 0);
                if (s_valid[b3 * 4 + j]) {
                    const uint4 kw = lds128(T + cb * 512 + ln * 16);
                    // K scales [g][half][group]: token g is half 0, token g+8 half 1
                    const uint16_t s0 = *reinterpret_cast<const uint16_t*>(T + 16 * kPfD + 2 * ((g * 2) * 4 + cb));
                    const uint16_t s1 = *reinterpret_cast<const uint16_t*>(T + 16 * kPfD + 2 * ((g * 2 + 1) * 4 + cb));
                    const uint32_t d0 = (uint32_t)s0 | ((uint32_t)s0 << 16), d1 = (uint32_t)s1 | ((uint32_t)s1 << 16);
                    const uint32_t x0 = bias8(kw.x), x1 = bias8(kw.y), z0 = bias8(kw.z), z1 = bias8(kw.w);
                    o0 = make_uint4(dq2(x0, 0, d0), dq2(x0, 1, d0), dq2(x1, 0, d0), dq2(x1, 1, d0));
                    o1 = make_uint4(dq2(z0, 0, d1), dq2(z0, 1, d1), dq2(z1, 0, d1), dq2(z1, 1, d1));
                }
                const int t0 = j * 16 + g, c = cb * 4 + tig;  // 16-byte chunk = dims 8c .. 8c+7
                sts128(kdst + sw128_off(t0, c, kPfKeys), o0);
                sts128(kdst + sw128_off(t0 + 8, c, kPfKeys), o1);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                // V^T row d, keys 16j .. 16j+15: the four lanes (g', tig=0..3) of dim d hold
                // tokens {2tig, 2tig+8, 2tig+1, 2tig+9} in one 32-bit word each
                const int item = t + i * 128;
                const int j = item >> 7, d = item & 127;
                const int m = d >> 4, gp = d & 7, dh = (d >> 3) & 1;
                const uint8_t* T = raw + j * kRawTileBytes;
                uint4 lo = make_uint4(0, 0, 0, 0), hi = make_uint4(0, 0, 0, 0);
                if (s_valid[b3 * 4 + j]) {
                    const uint8_t* vb = T + 16 * kPfD + 128 + (m >> 1) * 512 + ((m & 1) * 2 + dh) * 4;
                    uint32_t wv[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q) wv[q] = lds32(vb + (gp * 4 + q) * 16);
                    // keys 0..7 = bytes 0,2 of wv[0..3]; keys 8..15 = bytes 1,3
                    const uint32_t k03 = __byte_perm(wv[0], wv[1], 0x6420), k47 = __byte_perm(wv[2], wv[3], 0x6420);
                    const uint32_t k8b = __byte_perm(wv[0], wv[1], 0x7531), kcf = __byte_perm(wv[2], wv[3], 0x7531);
                    // V scales [tig][group][j]: pairs (2tig, 2tig+8), (2tig+1, 2tig+9)
                    const int sg = d >> 5;
                    uint32_t sp[8];  // (token 2k, 2k+1) f16x2 for k = 0..7
                    const uint8_t* vs = T + 32 * kPfD + 128 + sg * 8;
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const uint2 pr = lds64(vs + q * 32);
                        sp[q] = __byte_perm(pr.x, pr.y, 0x5410);
                        sp[4 + q] = __byte_perm(pr.x, pr.y, 0x7632);
                    }
                    const uint32_t a = bias8(k03), bq = bias8(k47), c8 = bias8(k8b), cf = bias8(kcf);
                    lo = make_uint4(dq2(a, 0, sp[0]), dq2(a, 1, sp[1]), dq2(bq, 0, sp[2]), dq2(bq, 1, sp[3]));
                    hi = make_uint4(dq2(c8, 0, sp[4]), dq2(c8, 1, sp[5]), dq2(cf, 0, sp[6]), dq2(cf, 1, sp[7]));
                }
                sts128(vdst + sw128_off(d, 2 * j, kPfD), lo);
                sts128(vdst + sw128_off(d, 2 * j + 1, kPfD), hi);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&bars->kv_full[b2]);
                mbar_arrive(&bars->raw_free[b3]);
            }
        }
    } else {
        // ================= softmax: thread = query row =================
        const int row = tid;
        const int kvlen = row < rows ? max(0, min(Tk, kv0 + pos0 + row / p.G + 1)) : 0;
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        float m_run = -INFINITY, l_run = 0.f;
        for (int it = 0; it < n_kt; ++it) {
            const int b2 = it & 1;
            if (!wait_phase(&bars->s_full[b2], it >> 1, s_abort)) timed_out = true;
            tc_fence_after();
            float s[64];
            tmem_ld32(tmem + b2 * 64 + lane_off, *reinterpret_cast<float(*)[32]>(s));
            tmem_ld32(tmem + b2 * 64 + 32 + lane_off, *reinterpret_cast<float(*)[32]>(s + 32));
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->s_free[b2]);

            const int key0 = it * kPfKeys;
            // pool tiles of this key tile that hold keys (read from the block table: the control
            // warp already reuses its flags for the tile two ahead)
            bool pv[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int pt = it * 4 + j;
                pv[j] = pt < pt_total && __ldg(btrow + pt / p.tpp) < (uint32_t)p.n_pages;
            }
            const bool full = key0 + kPfKeys <= kv_lo && pv[0] && pv[1] && pv[2] && pv[3];
            float mx = -INFINITY;
            if (full) {
#pragma unroll
                for (int c = 0; c < 64; ++c) {
                    s[c] *= p.scale_log2;
                    mx = fmaxf(mx, s[c]);
                }
            } else {
#pragma unroll
                for (int c = 0; c < 64; ++c) {
                    const bool ok = key0 + c < kvlen && pv[c >> 4];
                    s[c] = ok ? s[c] * p.scale_log2 : -INFINITY;
                    mx = fmaxf(mx, s[c]);
                }
            }
            float alpha = 1.f;
            bool need = false;
            if (mx > m_run + kPfRescale) {
                alpha = fast_exp2(m_run - mx);
                m_run = mx;
                l_run *= alpha;
                need = it > 0;
            }
            const float muse = m_run == -INFINITY ? 0.f : m_run;
            if (it >= 2 && !wait_phase(&bars->pv_done[b2], (it - 2) >> 1, s_abort)) timed_out = true;  // P[b2] free
            const uint32_t pdst = sbase + kSmP + b2 * 16384;
            float sum = 0.f;
#pragma unroll
            for (int c8 = 0; c8 < 8; ++c8) {
                uint32_t pk[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float p0 = fast_exp2(s[c8 * 8 + 2 * e] - muse), p1 = fast_exp2(s[c8 * 8 + 2 * e + 1] - muse);
                    sum += p0 + p1;
                    pk[e] = pack_h2(p0, p1);
                }
                sts128(pdst + sw128_off(row, c8, kPfRows), make_uint4(pk[0], pk[1], pk[2], pk[3]));
            }
            l_run += sum;
            s_alpha[b2 * kPfRows + row] = alpha;
            if (softmax_any(need)) {
                // PV(it-1) must have landed before O^T is rescaled; thread d owns lane d
                if (!wait_phase(&bars->pv_done[(it - 1) & 1], (it - 1) >> 1, s_abort)) timed_out = true;
                tc_fence_after();
#pragma unroll
                for (int c0 = 0; c0 < kPfRows; c0 += 32) {
                    float o[32];
                    tmem_ld32(tmem + 128 + c0 + lane_off, o);
#pragma unroll
                    for (int e = 0; e < 32; ++e) o[e] *= s_alpha[b2 * kPfRows + c0 + e];
                    tmem_st32(tmem + 128 + c0 + lane_off, o);
                }
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->p_full[b2]);
        }
        // ---- epilogue: thread d writes dim d of every row
        s_linv[row] = l_run > 0.f ? 1.f / l_run : 0.f;
        if (n_kt > 0 && !wait_phase(&bars->pv_done[(n_kt - 1) & 1], (n_kt - 1) >> 1, s_abort)) timed_out = true;
        tc_fence_after();
        softmax_sync();
        const int d = tid;
        if (n_kt > 0) {
#pragma unroll
            for (int c0 = 0; c0 < kPfRows; c0 += 32) {
                float o[32];
                tmem_ld32(tmem + 128 + c0 + lane_off, o);
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    const int r = c0 + e;
                    if (r < rows)
                        p.out[((size_t)(qrow0 + pos0 + r / p.G) * p.Hq + (size_t)h * p.G + r % p.G) * kPfD + d] =
                            __float2half_rn(o[e] * s_linv[r]);
                }
            }
        } else {
            for (int r = 0; r < rows; ++r)
                p.out[((size_t)(qrow0 + pos0 + r / p.G) * p.Hq + (size_t)h * p.G + r % p.G) * kPfD + d] =
                    __float2half_rn(0.f);
        }
    }
    if (timed_out) atomicOr(p.status, YF_DEV_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    if (warp == 8) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPfTmemCols) : "memory");
    }
}

}  // namespace

// True when the tensor-core prefill kernel handles this call.
bool prefill_tc_applies(const yf_pool* pool, int n_q_heads, int max_seqlen_q) {
    const char* env = getenv("YF_PREFILL_TC");  // host-side switch for A/B runs
    if (env && atoi(env) == 0) return false;
    const yf_pool_desc& d = pool->desc;
    const int G = n_q_heads / d.n_kv_heads;
    return d.head_dim == kPfD && d.group_size == 32 && kPfRows % G == 0 && (long long)G * max_seqlen_q >= kPfRows;
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
    static int attr_dev[64] = {};
    const int dev = d.device;
    if (dev < 0 || dev >= 64 || !attr_dev[dev]) {
        const cudaError_t e =
            cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmAlloc);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(prefill_tc)");
        if (dev >= 0 && dev < 64) attr_dev[dev] = 1;
    }
    const int ppb = kPfRows / p.G;
    const dim3 grid((a.max_seqlen_q + ppb - 1) / ppb, d.n_kv_heads, a.batch);
    if (grid.x > 0x7fffffffu) return fail(YF_E_UNSUPPORTED, "too many query rows");
    prefill_tc_kernel<<<grid, kPfBlock, kSmAlloc, a.stream>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? YF_OK : cuda_fail(e, "prefill_tc launch");
}

}  // namespace yf
