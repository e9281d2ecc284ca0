// Causal chunked-prefill attention over the paged Q8_0 pool on the 5th-generation
// tensor cores (tcgen05, TMEM accumulators).
//
// Replaces the prefill branch of the engine's FA2 varlen split-KV call from
// forward_attn_prefill_paged (docs/plans/2026-08-27-mtp-cuda-graphs.md:132,244-248;
// QK_INT8_PREFILL described at docs/research/2026-09-16-head-to-head-llamacpp-and-phase-profile.md:3627-3634):
// query row i of an entry sees keys 0 .. Tk - Tq + i.
//
// One CTA (128 threads) = one entry, one kv head, 128 query rows = 128/G query positions x
// the G q heads of the kv head (GQA folded into M, so every key tile is dequantized once for
// all of them).  Per 64-key tile:
//   1. lane 0 of warp 0 bulk-copies the four 16-token pool tiles (K+V int8 + scales, one
//      contiguous block each) into a raw staging buffer, double-buffered one tile ahead;
//   2. all threads dequantize K into f16 [key][dim] and V into f16 V^T [dim][key], both in
//      the K-major 128-byte-swizzled shared-memory layout the MMA descriptors describe;
//   3. one thread issues S = Q K^T (M=128 rows, N=64 keys, K=128 dims: 8 x tcgen05.mma
//      kind::f16, f32 accumulator in TMEM) and commits to an mbarrier;
//   4. thread r (TMEM lane r) loads its row of S, applies the scale, the causal mask and
//      an online base-2 softmax with lazy rescale, and writes its row of P (f16) over K;
//      when a row's max moved, every thread rescales its TMEM lane of O^T;
//   5. one thread issues O^T += V^T P^T (M=128 dims, N=128 rows, K=64 keys: 4 MMAs).
// At the end thread d reads lane d of O^T (all 128 rows) and writes out[row][d] / l[row].
#include <cstdint>
#include <cstdlib>

#include "yf_device.cuh"
#include "yf_internal.h"

namespace yf {
namespace {

constexpr int kPfThreads = 128;
constexpr int kPfRows = 128;     // query rows per CTA (M of S, N of O^T)
constexpr int kPfKeys = 64;      // keys per tile (N of S, K of O^T)
constexpr int kPfD = 128;        // head dim (K of S, M of O^T)
constexpr int kPfTmemCols = 256; // S: cols [0,64), O^T: cols [64,192)
constexpr float kPfRescale = 8.0f;  // lazy rescale threshold (base 2), as in the decode kernels

// shared-memory map (bytes from a 1024-aligned base)
constexpr int kSmQ = 0;                        // Q  [128 rows][128 d] f16, 2 column blocks x 16 KB
constexpr int kSmKP = kSmQ + 32768;            // K  [64 keys][128 d] f16 (2 x 8 KB); later P [128 rows][64 keys]
constexpr int kSmVt = kSmKP + 16384;           // V^T [128 d][64 keys] f16
constexpr int kSmRaw = kSmVt + 16384;          // 2 x 4 raw pool tiles (4352 B each)
constexpr int kRawTileBytes = 4352;            // D=128, group 32
constexpr int kRawBytes = 4 * kRawTileBytes;   // one 64-key tile
constexpr int kSmMisc = kSmRaw + 2 * kRawBytes;
constexpr int kSmBytes = kSmMisc + 2048;       // misc: barriers, tmem address, alpha, 1/l, flags
constexpr int kSmAlloc = kSmBytes + 1024;      // + alignment slack

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

__global__ void __launch_bounds__(kPfThreads, 1) prefill_tc_kernel(const PrefillParams p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t sraw = smem_u32(smem_raw);
    const uint32_t sbase = (sraw + 1023u) & ~1023u;
    uint8_t* base = smem_raw + (sbase - sraw);
    uint64_t* bar_mma = reinterpret_cast<uint64_t*>(base + kSmMisc);
    uint64_t* bar_raw = bar_mma + 1;  // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + kSmMisc + 64);
    float* s_alpha = reinterpret_cast<float*>(base + kSmMisc + 128);   // [128]
    float* s_linv = s_alpha + kPfRows;                                    // [128]
    uint8_t* s_valid = reinterpret_cast<uint8_t*>(s_linv + kPfRows);    // [2][4] pool-tile flags

    const int tid = threadIdx.x, warp = tid >> 5;
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
    const int kv0 = Tk - Tq;                     // keys before the chunk
    const int kv_hi = max(0, min(Tk, kv0 + pos0 + npos));
    const int n_kt = (kv_hi + kPfKeys - 1) / kPfKeys;
    const int pt_total = (Tk + 15) / 16;         // pool tiles that hold keys
    const uint32_t* btrow = p.bt + (size_t)b * p.max_blocks;
    const uint8_t* head_base = p.layer_base + (size_t)h * p.phb;
    const long long page_stride = p.phb * p.H;

    // this thread's softmax row
    const int my_row = tid;
    const bool row_live = my_row < rows;
    const int my_kvlen = row_live ? max(0, min(Tk, kv0 + pos0 + my_row / p.G + 1)) : 0;

    // ---- set-up: barriers, TMEM, Q tile
    if (tid == 0) {
        mbar_init(bar_mma, 1);
        mbar_init(&bar_raw[0], 1);
        mbar_init(&bar_raw[1], 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kPfTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    {
        // Q row `tid` (position pos0 + tid/G, head h*G + tid%G) into the SW128 Q tile
        uint4 zero = make_uint4(0, 0, 0, 0);
        const uint4* qp = nullptr;
        if (row_live)
            qp = reinterpret_cast<const uint4*>(
                p.q + ((size_t)(qrow0 + pos0 + my_row / p.G) * p.Hq + (size_t)h * p.G + my_row % p.G) * kPfD);
#pragma unroll
        for (int c = 0; c < 16; ++c) sts128(sbase + kSmQ + sw128_off(my_row, c, kPfRows), row_live ? __ldg(qp + c) : zero);
    }

    // lane 0 of warp 0: copy the four pool tiles of key tile `kt` into raw buffer `buf`
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
        mbar_arrive_expect_tx(&bar_raw[buf], bytes);
        for (int j = 0; j < 4; ++j)
            if (src[j]) bulk_g2s(dst + j * kRawTileBytes, src[j], kRawTileBytes, &bar_raw[buf]);
    };

    fence_proxy_async_smem();  // Q tile (generic writes) before the MMAs read it
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tmem_S = tmem;
    const uint32_t tmem_O = tmem + 64;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    if (tid == 0 && n_kt > 0) issue_raw(0, 0);

    constexpr uint32_t IDESC_S = umma_idesc_f16(kPfRows, kPfKeys);
    constexpr uint32_t IDESC_O = umma_idesc_f16(kPfD, kPfRows);
    float m_run = -INFINITY, l_run = 0.f;
    bool timed_out = false;

    for (int it = 0; it < n_kt; ++it) {
        const int buf = it & 1;
        if (tid == 0 && it + 1 < n_kt) issue_raw(it + 1, buf ^ 1);
        if (!mbar_wait(&bar_raw[buf], (uint32_t)(it >> 1) & 1u)) timed_out = true;
        const uint8_t* raw = base + kSmRaw + buf * kRawBytes;

        // ---- 2. dequantize K -> [key][d] and V -> V^T [d][key] (f16, SW128)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            // K: 16-byte word w of the tile = tokens g, g+8 x dims 32cb+8tig .. +7
            const int w = tid + i * kPfThreads;
            const int j = w >> 7, cb = (w & 127) >> 5, ln = w & 31, g = ln >> 2, tig = ln & 3;
            const uint8_t* T = raw + j * kRawTileBytes;
            uint4 o0 = make_uint4(0, 0, 0, 0), o1 = make_uint4(0, 0, 0, 0);
            if (s_valid[buf * 4 + j]) {
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
            sts128(sbase + kSmKP + sw128_off(t0, c, kPfKeys), o0);
            sts128(sbase + kSmKP + sw128_off(t0 + 8, c, kPfKeys), o1);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            // V^T row d, keys 16j .. 16j+15: the four lanes (g', tig=0..3) of dim d hold
            // tokens {2tig, 2tig+8, 2tig+1, 2tig+9} in one 32-bit word each
            const int item = tid + i * kPfThreads;
            const int j = item >> 7, d = item & 127;
            const int m = d >> 4, gp = d & 7, dh = (d >> 3) & 1;
            const uint8_t* T = raw + j * kRawTileBytes;
            uint4 lo = make_uint4(0, 0, 0, 0), hi = make_uint4(0, 0, 0, 0);
            if (s_valid[buf * 4 + j]) {
                const uint8_t* vb = T + 16 * kPfD + 128 + (m >> 1) * 512 + ((m & 1) * 2 + dh) * 4;
                uint32_t wv[4];
#pragma unroll
                for (int t = 0; t < 4; ++t) wv[t] = lds32(vb + (gp * 4 + t) * 16);
                // keys 0..7 = bytes 0,2 of wv[0..3]; keys 8..15 = bytes 1,3
                const uint32_t k03 = __byte_perm(wv[0], wv[1], 0x6420), k47 = __byte_perm(wv[2], wv[3], 0x6420);
                const uint32_t k8b = __byte_perm(wv[0], wv[1], 0x7531), kcf = __byte_perm(wv[2], wv[3], 0x7531);
                // V scales of group s = d/32 for tokens 0..15: [tig][s][j] pairs (2tig, 2tig+8), (2tig+1, 2tig+9)
                const int s = d >> 5;
                uint32_t sp[8];  // (token 2k, 2k+1) f16x2 for k = 0..7
                const uint8_t* vs = T + 32 * kPfD + 128 + s * 8;
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const uint2 q = lds64(vs + t * 4 * 8);  // .x = (2t, 2t+8), .y = (2t+1, 2t+9)
                    sp[t] = __byte_perm(q.x, q.y, 0x5410);       // (2t, 2t+1)
                    sp[4 + t] = __byte_perm(q.x, q.y, 0x7632);   // (2t+8, 2t+9)
                }
                const uint32_t a = bias8(k03), bq = bias8(k47), c8 = bias8(k8b), cf = bias8(kcf);
                lo = make_uint4(dq2(a, 0, sp[0]), dq2(a, 1, sp[1]), dq2(bq, 0, sp[2]), dq2(bq, 1, sp[3]));
                hi = make_uint4(dq2(c8, 0, sp[4]), dq2(c8, 1, sp[5]), dq2(cf, 0, sp[6]), dq2(cf, 1, sp[7]));
            }
            sts128(sbase + kSmVt + sw128_off(d, 2 * j, kPfD), lo);
            sts128(sbase + kSmVt + sw128_off(d, 2 * j + 1, kPfD), hi);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();

        // ---- 3. S = Q K^T
        if (tid == 0) {
            tc_fence_after();
#pragma unroll
            for (int ks = 0; ks < kPfD / 16; ++ks) {
                const uint64_t a = umma_desc_sw128(sbase + kSmQ + (ks >> 2) * (kPfRows * 128) + (ks & 3) * 32);
                const uint64_t bd = umma_desc_sw128(sbase + kSmKP + (ks >> 2) * (kPfKeys * 128) + (ks & 3) * 32);
                umma_f16(tmem_S, a, bd, IDESC_S, ks > 0);
            }
            umma_commit(bar_mma);
        }
        if (!mbar_wait(bar_mma, 0u)) timed_out = true;
        tc_fence_after();

        // ---- 4. softmax of row tid; P over K
        bool need = false;
        float alpha = 1.f;
        {
            float s[64];
            float* s0 = s;
            tmem_ld32(tmem_S + lane_off + 0, *reinterpret_cast<float(*)[32]>(s0));
            tmem_ld32(tmem_S + lane_off + 32, *reinterpret_cast<float(*)[32]>(s0 + 32));
            const int key0 = it * kPfKeys;
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < 64; ++c) {
                const int key = key0 + c;
                const bool ok = key < my_kvlen && s_valid[buf * 4 + (c >> 4)];
                s[c] = ok ? s[c] * p.scale_log2 : -INFINITY;
                mx = fmaxf(mx, s[c]);
            }
            if (mx > m_run + kPfRescale) {
                alpha = fast_exp2(m_run - mx);
                m_run = mx;
                l_run *= alpha;
                need = true;
            }
            const float muse = m_run == -INFINITY ? 0.f : m_run;
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
                sts128(sbase + kSmKP + sw128_off(my_row, c8, kPfRows), make_uint4(pk[0], pk[1], pk[2], pk[3]));
            }
            l_run += sum;
        }
        s_alpha[tid] = alpha;
        const bool any_need = __syncthreads_or(need && it > 0);
        if (any_need) {
            // thread d rescales lane d of O^T: column r is query row r
#pragma unroll
            for (int c0 = 0; c0 < kPfRows; c0 += 32) {
                float o[32];
                tmem_ld32(tmem_O + lane_off + c0, o);
#pragma unroll
                for (int e = 0; e < 32; ++e) o[e] *= s_alpha[c0 + e];
                tmem_st32(tmem_O + lane_off + c0, o);
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();

        // ---- 5. O^T += V^T P^T
        if (tid == 0) {
            tc_fence_after();
#pragma unroll
            for (int ks = 0; ks < kPfKeys / 16; ++ks) {
                const uint64_t a = umma_desc_sw128(sbase + kSmVt + ks * 32);
                const uint64_t bd = umma_desc_sw128(sbase + kSmKP + ks * 32);
                umma_f16(tmem_O, a, bd, IDESC_O, (it > 0 || ks > 0) ? 1u : 0u);
            }
            umma_commit(bar_mma);
        }
        if (!mbar_wait(bar_mma, 1u)) timed_out = true;
        tc_fence_after();
    }
    if (timed_out) atomicOr(p.status, YF_DEV_TIMEOUT);

    // ---- epilogue: thread d writes dim d of every row
    s_linv[tid] = l_run > 0.f ? 1.f / l_run : 0.f;
    __syncthreads();
    if (n_kt > 0) {
        const int d = tid;
#pragma unroll
        for (int c0 = 0; c0 < kPfRows; c0 += 32) {
            float o[32];
            tmem_ld32(tmem_O + lane_off + c0, o);
#pragma unroll
            for (int e = 0; e < 32; ++e) {
                const int r = c0 + e;
                if (r < rows) {
                    __half* op = p.out + ((size_t)(qrow0 + pos0 + r / p.G) * p.Hq + (size_t)h * p.G + r % p.G) * kPfD + d;
                    *op = __float2half_rn(o[e] * s_linv[r]);
                }
            }
        }
    } else {
        for (int r = 0; r < rows; ++r)
            p.out[((size_t)(qrow0 + pos0 + r / p.G) * p.Hq + (size_t)h * p.G + r % p.G) * kPfD + tid] = __float2half_rn(0.f);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
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
    prefill_tc_kernel<<<grid, kPfThreads, kSmAlloc, a.stream>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? YF_OK : cuda_fail(e, "prefill_tc launch");
}

}  // namespace yf
