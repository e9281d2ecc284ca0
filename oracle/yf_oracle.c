/*
 * yf_oracle.c — CPU oracle for the paged Q8_0 KV attention path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py load this library, and only as
 * the checker or the timed CPU baseline.  The product path (the CUDA library
 * in qwen36-server_b200/csrc) never links, loads or calls it.
 *
 * What it restates, and from where:
 *  - Q8_0 quantization: GGML's published reference quantizer for Q8_0, which
 *    candle-core's BlockQ8_0::from_float restates (candle-core is the
 *    reference's path dependency, Cargo.toml:40, an un-vendored checkout with
 *    no pinned version).  Per group of G values x (f16 inputs widened to
 *    f32):  amax = max|x|;  d = amax / 127;  id = d ? 1/d : 0;
 *    q = roundf(x * id) (half away from zero);  d stored as f16 (RNE).
 *    The reference's own pool keeps one scale per (token, kv-head) row
 *    (docs/plans/2026-08-24-qwen35-4b-benchmark.md:586-588; formula at
 *    docs/research/2026-09-16-head-to-head-llamacpp-and-phase-profile.md:3079-3080);
 *    that is the same rule with G = head_dim.
 *  - Paged addressing: token pos of entry b lives in page
 *    block_table[b*max_blocks + pos/P], slot pos%P
 *    (docs/plans/2026-08-27-tiered-kv-cache.md:52-58, src/bin/decode_gqa_probe.rs:40-46).
 *  - Attention: o = softmax(q k^T * scale) v per query head over the
 *    dequantized cache, GQA group = Hq/Hkv (kv head of q head h = h/(Hq/Hkv)),
 *    causal rows "row i sees 0..kv0+i" (docs/plans/2026-08-27-mtp-cuda-graphs.md:244-246),
 *    the F32 matmul-softmax reference of src/bin/fa_probe.rs:54-82.
 *  - The byte layout of a 16-token tile is this library's own format
 *    (include/yfattn.h); the oracle computes offsets independently of the
 *    CUDA code so that a layout bug shows up as a byte mismatch.
 *
 * Parity status: the quantizer is pinned to gguf-py's Q8_0 implementation
 * (tests/golden); the attention path is pinned only to the reference's
 * documented semantics and probe shapes, since the reference kernels are not
 * in the mounted tree and cannot be run here ("parity unpinned" for attention).
 */
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    int32_t n_layers, n_pages, n_kv_heads, head_dim, page_size, group_size;
} yfo_desc;

/* ---- f16 <-> f32, written from the IEEE 754 binary16 definition ---------- */
float yfo_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: man * 2^-24 */
            float v = (float)man * 5.9604644775390625e-08f;
            memcpy(&bits, &v, 4);
            bits |= sign;
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t yfo_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) { /* inf or nan */
        return (uint16_t)(sign | 0x7c00u | (absx > 0x7f800000u ? 0x200u : 0u));
    }
    int32_t e = (int32_t)(absx >> 23) - 127; /* unbiased exponent */
    uint32_t m = (absx & 0x7fffffu) | 0x800000u;
    if (absx < 0x00800000u) return (uint16_t)sign; /* f32 subnormal -> 0 in f16 */
    if (e > 15) return (uint16_t)(sign | 0x7c00u);
    int32_t shift; /* right shift of the 24-bit significand */
    uint32_t hexp;
    if (e >= -14) {
        shift = 13;
        hexp = (uint32_t)(e + 15);
    } else {
        shift = 13 + (-14 - e);
        hexp = 0;
        if (shift > 24) return (uint16_t)sign;
    }
    uint32_t kept = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (kept & 1u))) kept += 1u;
    uint32_t out;
    if (hexp == 0) {
        out = kept; /* subnormal; a carry into 0x400 is the smallest normal */
    } else {
        out = (hexp << 10) + (kept - 0x400u); /* carry may bump the exponent */
    }
    if (out >= 0x7c00u) out = 0x7c00u;
    return (uint16_t)(sign | out);
}

/* ---- format ---------------------------------------------------------------- */
static int nb_of(const yfo_desc* d) { return d->head_dim / d->group_size; }

size_t yfo_tile_bytes(const yfo_desc* d) {
    return (size_t)2 * (16 * (size_t)d->head_dim + 32 * (size_t)nb_of(d));
}
size_t yfo_page_head_bytes(const yfo_desc* d) { return (size_t)(d->page_size / 16) * yfo_tile_bytes(d); }
size_t yfo_pool_bytes(const yfo_desc* d) {
    return (size_t)d->n_layers * d->n_pages * d->n_kv_heads * yfo_page_head_bytes(d);
}

/* Offset of the value byte (t, dim) inside a tile; the byte holds the Q8_0 value q as the
 * excess-128 byte q + 128.  K: lane (g = t%8, tig)
 * holds dims 32b+8tig..+7 of tokens g and g+8 in one 16-byte word.  V: lane
 * (g = dim%8, tig = (t%8)/2) holds tokens {2tig, 2tig+8, 2tig+1, 2tig+9} of
 * dims 16m+g and 16m+g+8 for two adjacent 16-dim tiles m. */
int64_t yfo_tile_offset(const yfo_desc* d, int is_v, int t, int dim) {
    int D = d->head_dim, NB = nb_of(d);
    if (!is_v) {
        int b = dim / 32, r = dim % 32, tig = r / 8, e = r % 8, g = t % 8, half = t / 8;
        return (int64_t)b * 512 + (g * 4 + tig) * 16 + half * 8 + e;
    }
    int base = 16 * D + 32 * NB;
    int m = dim / 16, i = dim % 16, gg = i % 8, dhalf = i / 8;
    int tig = (t % 8) / 2, j = (t & 1) * 2 + t / 8;
    int lane = gg * 4 + tig;
    return (int64_t)base + (m / 2) * 512 + lane * 16 + (m % 2) * 8 + dhalf * 4 + j;
}

int64_t yfo_scale_offset(const yfo_desc* d, int is_v, int t, int grp) {
    int D = d->head_dim, NB = nb_of(d);
    if (!is_v) {
        int g = t % 8, half = t / 8;
        return (int64_t)16 * D + 2 * ((g * 2 + half) * NB + grp);
    }
    int base = 16 * D + 32 * NB + 16 * D;
    int tig = (t % 8) / 2, j = (t & 1) * 2 + t / 8;
    return (int64_t)base + 2 * ((tig * NB + grp) * 4 + j);
}

/* ---- quantizer --------------------------------------------------------------- */
void yfo_quantize_group(const uint16_t* x, int n, int8_t* q, uint16_t* d_out) {
    float amax = 0.0f;
    for (int i = 0; i < n; ++i) {
        float a = fabsf(yfo_f16_to_f32(x[i]));
        if (a > amax) amax = a;
    }
    volatile float d = amax / 127.0f; /* volatile: keep the f32 division exact */
    float id = (d != 0.0f) ? 1.0f / d : 0.0f;
    for (int i = 0; i < n; ++i) {
        volatile float v = yfo_f16_to_f32(x[i]) * id;
        q[i] = (int8_t)roundf(v);
    }
    *d_out = yfo_f32_to_f16(d);
}

/* Quantizes one head row of D values into q[D] and d[D/G]. */
void yfo_quantize_row(const uint16_t* x, int D, int G, int8_t* q, uint16_t* d) {
    for (int s = 0; s < D / G; ++s) yfo_quantize_group(x + s * G, G, q + s * G, d + s);
}

static uint8_t* tile_ptr(const yfo_desc* d, uint8_t* pool, int layer, int page, int head, int pos_in_page) {
    size_t blk = ((size_t)layer * d->n_pages + page) * d->n_kv_heads + head;
    return pool + blk * yfo_page_head_bytes(d) + (size_t)(pos_in_page / 16) * yfo_tile_bytes(d);
}

/* Quantizes and scatters n_rows rows.  Row r (K and V f16 [n_rows, Hkv, D])
 * goes to entry row_entry[r] at position row_pos[r].  Rows whose position is
 * outside the entry's table, or whose page id is >= n_pages, are skipped.
 * Returns the number of skipped rows. */
int yfo_kv_write_rows(const yfo_desc* d, uint8_t* pool, int layer, const uint16_t* k, const uint16_t* v,
                      int n_rows, const int32_t* row_entry, const int32_t* row_pos,
                      const uint32_t* block_table, int max_blocks) {
    int D = d->head_dim, G = d->group_size, NB = nb_of(d), P = d->page_size, H = d->n_kv_heads;
    int skipped = 0;
    int8_t* q = (int8_t*)malloc((size_t)D);
    uint16_t* sc = (uint16_t*)malloc((size_t)NB * 2);
    for (int r = 0; r < n_rows; ++r) {
        int b = row_entry[r], pos = row_pos[r];
        if (pos < 0 || pos >= max_blocks * P) { ++skipped; continue; }
        uint32_t page = block_table[(size_t)b * max_blocks + pos / P];
        if (page >= (uint32_t)d->n_pages) { ++skipped; continue; }
        int t = pos % 16;
        for (int h = 0; h < H; ++h) {
            uint8_t* tile = tile_ptr(d, pool, layer, (int)page, h, pos % P);
            for (int kv = 0; kv < 2; ++kv) {
                const uint16_t* src = (kv ? v : k) + ((size_t)r * H + h) * D;
                yfo_quantize_row(src, D, G, q, sc);
                for (int dim = 0; dim < D; ++dim)
                    tile[yfo_tile_offset(d, kv, t, dim)] = (uint8_t)((uint8_t)q[dim] ^ 0x80u);
                for (int s = 0; s < NB; ++s) memcpy(tile + yfo_scale_offset(d, kv, t, s), &sc[s], 2);
            }
        }
    }
    free(q);
    free(sc);
    return skipped;
}

/* Dequantized K and V of (layer, page, head, pos_in_page) into k_out[D], v_out[D]. */
void yfo_read_kv(const yfo_desc* d, const uint8_t* pool, int layer, int page, int head, int pos_in_page,
                 float* k_out, float* v_out) {
    int D = d->head_dim, G = d->group_size;
    const uint8_t* tile = tile_ptr(d, (uint8_t*)pool, layer, page, head, pos_in_page);
    int t = pos_in_page % 16;
    for (int kv = 0; kv < 2; ++kv) {
        float* o = kv ? v_out : k_out;
        for (int dim = 0; dim < D; ++dim) {
            uint16_t sb;
            memcpy(&sb, tile + yfo_scale_offset(d, kv, t, dim / G), 2);
            int8_t qv = (int8_t)(tile[yfo_tile_offset(d, kv, t, dim)] ^ 0x80u);
            o[dim] = (float)qv * yfo_f16_to_f32(sb);
        }
    }
}

typedef struct {
    const yfo_desc* d;
    const uint8_t* pool;
    int layer;
    const uint16_t* q;
    int Hq;
    const uint32_t *cu_q, *cu_k, *block_table;
    int max_blocks, B;
    float scale;
    float* out;
    atomic_long next;
    atomic_int bad;
} attn_job;

/* One (entry b, kv head h) unit: every query row of b and every q head of h. */
static void attn_unit(attn_job* J, int b, int h) {
    const yfo_desc* d = J->d;
    int D = d->head_dim, P = d->page_size, H = d->n_kv_heads, Hq = J->Hq;
    int grp = Hq / H;
    int Tq = (int)(J->cu_q[b + 1] - J->cu_q[b]);
    int Tk = (int)(J->cu_k[b + 1] - J->cu_k[b]);
    if (Tk > J->max_blocks * P) Tk = J->max_blocks * P;
    size_t nk_alloc = (size_t)(Tk > 0 ? Tk : 1);
    float* kbuf = (float*)malloc(sizeof(float) * nk_alloc * D);
    float* vbuf = (float*)malloc(sizeof(float) * nk_alloc * D);
    char* ok = (char*)malloc(nk_alloc);
    double* s = (double*)malloc(sizeof(double) * nk_alloc);
    double* acc = (double*)malloc(sizeof(double) * (size_t)D);
    float* qf = (float*)malloc(sizeof(float) * (size_t)D);
    for (int pos = 0; pos < Tk; ++pos) {
        uint32_t page = J->block_table[(size_t)b * J->max_blocks + pos / P];
        ok[pos] = page < (uint32_t)d->n_pages;
        if (!ok[pos]) { atomic_fetch_add(&J->bad, 1); continue; }
        yfo_read_kv(d, J->pool, J->layer, (int)page, h, pos % P, kbuf + (size_t)pos * D, vbuf + (size_t)pos * D);
    }
    for (int i = 0; i < Tq; ++i) {
        long row = (long)J->cu_q[b] + i;
        int nk = Tk - Tq + i + 1;
        if (nk > Tk) nk = Tk;
        for (int hh = h * grp; hh < (h + 1) * grp; ++hh) {
            const uint16_t* qrow = J->q + ((size_t)row * Hq + hh) * D;
            float* orow = J->out + ((size_t)row * Hq + hh) * D;
            for (int dim = 0; dim < D; ++dim) qf[dim] = yfo_f16_to_f32(qrow[dim]);
            double mx = -INFINITY;
            for (int j = 0; j < nk; ++j) {
                if (!ok[j]) { s[j] = -INFINITY; continue; }
                double dot = 0.0;
                const float* kr = kbuf + (size_t)j * D;
                for (int dim = 0; dim < D; ++dim) dot += (double)qf[dim] * (double)kr[dim];
                s[j] = dot * (double)J->scale;
                if (s[j] > mx) mx = s[j];
            }
            for (int dim = 0; dim < D; ++dim) acc[dim] = 0.0;
            double l = 0.0;
            if (nk > 0 && mx > -INFINITY) {
                for (int j = 0; j < nk; ++j) {
                    if (!ok[j]) continue;
                    double p = exp(s[j] - mx);
                    l += p;
                    const float* vr = vbuf + (size_t)j * D;
                    for (int dim = 0; dim < D; ++dim) acc[dim] += p * (double)vr[dim];
                }
            }
            for (int dim = 0; dim < D; ++dim) orow[dim] = (l > 0.0) ? (float)(acc[dim] / l) : 0.0f;
        }
    }
    free(s);
    free(acc);
    free(qf);
    free(kbuf);
    free(vbuf);
    free(ok);
}

static void* attn_worker(void* arg) {
    attn_job* J = (attn_job*)arg;
    long units = (long)J->B * J->d->n_kv_heads;
    for (;;) {
        long w = atomic_fetch_add(&J->next, 1);
        if (w >= units) break;
        attn_unit(J, (int)(w / J->d->n_kv_heads), (int)(w % J->d->n_kv_heads));
    }
    return NULL;
}

/* Causal paged attention over the dequantized cache, in double precision.
 * q: f16 [total_q, Hq, D]; out: f32 [total_q, Hq, D].
 * Entry b: query rows cu_q[b]..cu_q[b+1]-1, Tk = cu_k[b+1]-cu_k[b] keys;
 * row i sees keys 0..Tk-Tq+i.  A row that sees no key gets zeros; a key whose
 * page id is >= n_pages is skipped.  Returns the number of bad pages met.
 * n_threads <= 1 runs on the calling thread. */
int yfo_attn(const yfo_desc* d, const uint8_t* pool, int layer, const uint16_t* q, int Hq,
             const uint32_t* cu_q, const uint32_t* cu_k, const uint32_t* block_table, int max_blocks,
             int B, float scale, float* out, int n_threads) {
    attn_job J;
    J.d = d; J.pool = pool; J.layer = layer; J.q = q; J.Hq = Hq;
    J.cu_q = cu_q; J.cu_k = cu_k; J.block_table = block_table;
    J.max_blocks = max_blocks; J.B = B; J.scale = scale; J.out = out;
    atomic_init(&J.next, 0);
    atomic_init(&J.bad, 0);
    if (n_threads <= 1) {
        attn_worker(&J);
    } else {
        pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)n_threads);
        for (int i = 0; i < n_threads; ++i) pthread_create(&th[i], NULL, attn_worker, &J);
        for (int i = 0; i < n_threads; ++i) pthread_join(th[i], NULL);
        free(th);
    }
    return atomic_load(&J.bad);
}

/* xorshift32 Fisher-Yates shuffle of 0..count-1 with the seed and step order of
 * the reference's decode probe (src/bin/decode_gqa_probe.rs:13-23). */
void yfo_shuffled_pages(uint32_t count, uint32_t seed, uint32_t* out) {
    for (uint32_t i = 0; i < count; ++i) out[i] = i;
    uint32_t state = seed;
    for (uint32_t i = count ? count - 1 : 0; i >= 1; --i) {
        state ^= state << 13;
        state ^= state >> 17;
        state ^= state << 5;
        uint32_t j = state % (i + 1);
        uint32_t tmp = out[i];
        out[i] = out[j];
        out[j] = tmp;
    }
}

/* CRC-32C by its definition: the Castagnoli polynomial, bit-reflected (0x82F63B78), one input
 * bit at a time, register preset and final xor 0xFFFFFFFF.  The check value of the ASCII digits
 * "123456789" is 0xE3069283.  Used for the prefix cache's page records
 * (docs/plans/2026-08-27-tiered-kv-cache.md:237-251: a CRC32C per page record). */
uint32_t yfo_crc32c(const uint8_t* p, size_t n) {
    uint32_t c = 0xFFFFFFFFu;
    for (size_t i = 0; i < n; ++i) {
        c ^= p[i];
        for (int b = 0; b < 8; ++b) c = (c & 1u) ? (c >> 1) ^ 0x82F63B78u : c >> 1;
    }
    return c ^ 0xFFFFFFFFu;
}
