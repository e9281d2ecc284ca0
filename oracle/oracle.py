"""CPU oracle for the paged Q8_0 KV attention path (test infrastructure).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline and
reference legs import this module, and only as the checker or the timed CPU
baseline.  The product (qwen36-server_b200) never imports it.

Two restatements live here:
  * ``yf_oracle.c`` (ctypes): the Q8_0 quantizer, the pool scatter and a
    double-precision causal paged attention, multi-threaded with pthreads;
  * numpy mirrors of the quantizer and of the pool byte layout, vectorised for
    the large seeded workloads.
Both follow GGML's Q8_0 rule (restated by candle-core's BlockQ8_0::from_float,
the reference's path dependency at Cargo.toml:40) and the reference's paged
addressing ``pool[block_table[b][pos/P]][pos%P]``
(docs/plans/2026-08-27-tiered-kv-cache.md:52-58).  The quantizer is pinned to
gguf-py's Q8_0 implementation by tests/golden; the attention semantics follow
src/bin/fa_probe.rs:54-82 and docs/plans/2026-08-27-mtp-cuda-graphs.md:244-246.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "build", "libyforacle.so")
_lib = None


def build() -> str:
    """Compiles yf_oracle.c with the Makefile beside it; returns the .so path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(
            os.path.join(_HERE, "yf_oracle.c")
        ):
            build()
        L = ctypes.CDLL(_SO)
        vp, ci = ctypes.c_void_p, ctypes.c_int
        L.yfo_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.yfo_f16_to_f32.restype = ctypes.c_float
        L.yfo_f32_to_f16.argtypes = [ctypes.c_float]
        L.yfo_f32_to_f16.restype = ctypes.c_uint16
        L.yfo_quantize_row.argtypes = [vp, ci, ci, vp, vp]
        L.yfo_quantize_row.restype = None
        for name in ("yfo_tile_bytes", "yfo_page_head_bytes", "yfo_pool_bytes"):
            getattr(L, name).argtypes = [vp]
            getattr(L, name).restype = ctypes.c_size_t
        for name in ("yfo_tile_offset", "yfo_scale_offset"):
            getattr(L, name).argtypes = [vp, ci, ci, ci]
            getattr(L, name).restype = ctypes.c_int64
        L.yfo_kv_write_rows.argtypes = [vp, vp, ci, vp, vp, ci, vp, vp, vp, ci]
        L.yfo_kv_write_rows.restype = ci
        L.yfo_read_kv.argtypes = [vp, vp, ci, ci, ci, ci, vp, vp]
        L.yfo_read_kv.restype = None
        L.yfo_attn.argtypes = [vp, vp, ci, vp, ci, vp, vp, vp, ci, ci, ctypes.c_float, vp, ci]
        L.yfo_attn.restype = ci
        L.yfo_shuffled_pages.argtypes = [ctypes.c_uint32, ctypes.c_uint32, vp]
        L.yfo_shuffled_pages.restype = None
        L.yfo_crc32c.argtypes = [vp, ctypes.c_size_t]
        L.yfo_crc32c.restype = ctypes.c_uint32
        _lib = L
    return _lib


class _CDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in
                ("n_layers", "n_pages", "n_kv_heads", "head_dim", "page_size", "group_size")]


@dataclass(frozen=True)
class PoolDesc:
    """Pool shape; mirrors yf_pool_desc without the device fields."""
    n_layers: int
    n_pages: int
    n_kv_heads: int
    head_dim: int
    page_size: int = 16
    group_size: int = 32

    def c(self) -> _CDesc:
        return _CDesc(self.n_layers, self.n_pages, self.n_kv_heads, self.head_dim, self.page_size,
                      self.group_size)

    @property
    def n_groups(self) -> int:
        return self.head_dim // self.group_size

    @property
    def tile_bytes(self) -> int:
        return 2 * (16 * self.head_dim + 32 * self.n_groups)

    @property
    def page_head_bytes(self) -> int:
        return (self.page_size // 16) * self.tile_bytes

    @property
    def pool_bytes(self) -> int:
        return self.n_layers * self.n_pages * self.n_kv_heads * self.page_head_bytes


def _ptr(a: np.ndarray) -> ctypes.c_void_p:
    assert a.flags["C_CONTIGUOUS"]
    return ctypes.c_void_p(a.ctypes.data)


# ---- the C restatement ---------------------------------------------------------------

def c_quantize_rows(x: np.ndarray, group: int):
    """Q8_0 of f16 rows [..., D] -> (int8 [..., D], f16 [..., D/group]) through yf_oracle.c."""
    x = np.ascontiguousarray(x, dtype=np.float16)
    D = x.shape[-1]
    flat = x.reshape(-1, D)
    q = np.empty(flat.shape, np.int8)
    d = np.empty((flat.shape[0], D // group), np.float16)
    L = lib()
    for r in range(flat.shape[0]):
        L.yfo_quantize_row(ctypes.c_void_p(flat[r].ctypes.data), D, group,
                           ctypes.c_void_p(q[r].ctypes.data), ctypes.c_void_p(d[r].ctypes.data))
    return q.reshape(x.shape), d.reshape(x.shape[:-1] + (D // group,))


def c_kv_write_rows(desc: PoolDesc, pool: np.ndarray, layer: int, k: np.ndarray, v: np.ndarray,
                    row_entry: np.ndarray, row_pos: np.ndarray, block_table: np.ndarray) -> int:
    """Quantize-and-scatter rows into the pool image ``pool`` (uint8, pool_bytes) in place."""
    cd = desc.c()
    k = np.ascontiguousarray(k, np.float16)
    v = np.ascontiguousarray(v, np.float16)
    re_ = np.ascontiguousarray(row_entry, np.int32)
    rp = np.ascontiguousarray(row_pos, np.int32)
    bt = np.ascontiguousarray(block_table, np.uint32)
    return lib().yfo_kv_write_rows(ctypes.byref(cd), _ptr(pool), layer, _ptr(k), _ptr(v), k.shape[0],
                                   _ptr(re_), _ptr(rp), _ptr(bt), bt.shape[1])


def c_attn(desc: PoolDesc, pool: np.ndarray, layer: int, q: np.ndarray, cu_q: np.ndarray, cu_k: np.ndarray,
           block_table: np.ndarray, scale: float, n_threads: int = 0) -> np.ndarray:
    """Causal paged attention over the dequantized pool (double precision), f32 [total_q, Hq, D]."""
    cd = desc.c()
    q = np.ascontiguousarray(q, np.float16)
    cu_q = np.ascontiguousarray(cu_q, np.uint32)
    cu_k = np.ascontiguousarray(cu_k, np.uint32)
    bt = np.ascontiguousarray(block_table, np.uint32)
    out = np.zeros(q.shape, np.float32)
    if n_threads <= 0:
        n_threads = os.cpu_count() or 1
    lib().yfo_attn(ctypes.byref(cd), _ptr(pool), layer, _ptr(q), q.shape[1], _ptr(cu_q), _ptr(cu_k), _ptr(bt),
                   bt.shape[1], len(cu_q) - 1, ctypes.c_float(scale), _ptr(out), n_threads)
    return out


def c_read_kv(desc: PoolDesc, pool: np.ndarray, layer: int, page: int, head: int, pos_in_page: int):
    cd = desc.c()
    k = np.empty(desc.head_dim, np.float32)
    v = np.empty(desc.head_dim, np.float32)
    lib().yfo_read_kv(ctypes.byref(cd), _ptr(pool), layer, page, head, pos_in_page, _ptr(k), _ptr(v))
    return k, v


def crc32c(data) -> int:
    """CRC-32C (Castagnoli, reflected 0x82F63B78, preset and final xor 0xFFFFFFFF) through the
    bitwise definition in yf_oracle.c."""
    a = np.ascontiguousarray(np.frombuffer(bytes(data), np.uint8) if not isinstance(data, np.ndarray) else data,
                             np.uint8)
    return int(lib().yfo_crc32c(_ptr(a) if a.size else None, a.size))


def page_records(desc: "PoolDesc", pool: np.ndarray, pages, chain_hashes, page_indices, prev_hashes=None,
                 tokens=None) -> np.ndarray:
    """The prefix cache's page records (pages.kv, docs/plans/2026-08-27-tiered-kv-cache.md:141-145,
    237-251) of pool-image pages: [u64 chain_hash][u64 prev_hash][u32 page_index][u32 n_tokens]
    [u32 payload_len][u32 crc32c][u32 tokens[page_size]][payload], little-endian, packed; payload =
    the page in every layer, layer 0 first; the CRC-32C covers the token ids, then the payload."""
    page_bytes = desc.page_head_bytes * desc.n_kv_heads
    layer_bytes = desc.n_pages * page_bytes
    P = desc.page_size
    n = len(pages)
    prev_hashes = [0] * n if prev_hashes is None else list(prev_hashes)
    tokens = np.zeros((n, P), np.uint32) if tokens is None else np.asarray(tokens, np.int64).astype(np.uint32)
    out = []
    for i, (pg, hsh, idx) in enumerate(zip(pages, chain_hashes, page_indices)):
        payload = np.concatenate([pool[l * layer_bytes + int(pg) * page_bytes:
                                       l * layer_bytes + (int(pg) + 1) * page_bytes] for l in range(desc.n_layers)])
        tok = tokens[i].reshape(P).view(np.uint8)
        crc = crc32c(np.concatenate([tok, payload]))
        h, pv = int(hsh) & (2 ** 64 - 1), int(prev_hashes[i]) & (2 ** 64 - 1)
        head = np.array([h & 0xFFFFFFFF, h >> 32, pv & 0xFFFFFFFF, pv >> 32, int(idx), P, payload.size, crc],
                        np.uint32)
        out.append(np.concatenate([head.view(np.uint8), tok, payload]))
    return np.concatenate(out) if out else np.zeros(0, np.uint8)


def shuffled_pages(count: int, seed: int = 0x9E3779B9) -> np.ndarray:
    """The decode probe's xorshift32 Fisher-Yates page order (src/bin/decode_gqa_probe.rs:13-23)."""
    out = np.empty(count, np.uint32)
    lib().yfo_shuffled_pages(count, seed, _ptr(out))
    return out


# ---- numpy mirrors -------------------------------------------------------------------

def np_roundf(x: np.ndarray) -> np.ndarray:
    """roundf (half away from zero) in exact float arithmetic."""
    a = np.abs(x)
    f = np.floor(a)
    return np.sign(x) * (f + np.floor(2 * (a - f)))


def np_quantize_q8(x: np.ndarray, group: int):
    """Vectorised Q8_0 of f16 values [..., D] with the oracle's f32 arithmetic."""
    x = np.asarray(x, dtype=np.float16).astype(np.float32)
    shp = x.shape
    D = shp[-1]
    blk = x.reshape(-1, group)
    amax = np.abs(blk).max(axis=1, keepdims=True)
    d = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        idv = np.where(d == 0, np.float32(0), np.float32(1.0) / d).astype(np.float32)
    q = np_roundf((blk * idv).astype(np.float32)).astype(np.int8)
    return q.reshape(shp), d.astype(np.float16).reshape(shp[:-1] + (D // group,))


def excess128(q: np.ndarray) -> np.ndarray:
    """Pool bytes of Q8_0 values: q + 128 (the top bit of the two's-complement byte flipped)."""
    return q.view(np.uint8) ^ np.uint8(0x80)


def from_excess128(b: np.ndarray) -> np.ndarray:
    """Q8_0 values of pool bytes."""
    return (b ^ np.uint8(0x80)).view(np.int8)


def layout_maps(desc: PoolDesc):
    """Offset tables of the 16-token tile: K/V value offsets [16, D] and scale offsets [16, NB]."""
    D, NB = desc.head_dim, desc.n_groups
    t = np.arange(16)[:, None]
    dim = np.arange(D)[None, :]
    b, r = dim // 32, dim % 32
    koff = b * 512 + ((t % 8) * 4 + r // 8) * 16 + (t // 8) * 8 + r % 8
    m, i = dim // 16, dim % 16
    tig, j = (t % 8) // 2, (t & 1) * 2 + t // 8
    vbase = 16 * D + 32 * NB
    voff = vbase + (m // 2) * 512 + ((i % 8) * 4 + tig) * 16 + (m % 2) * 8 + (i // 8) * 4 + j
    s = np.arange(NB)[None, :]
    ksoff = 16 * D + 2 * (((t % 8) * 2 + t // 8) * NB + s)
    vsoff = vbase + 16 * D + 2 * ((tig * NB + s) * 4 + j)
    return koff.astype(np.int64), voff.astype(np.int64), ksoff.astype(np.int64), vsoff.astype(np.int64)


def np_tile_base(desc: PoolDesc, layer: int, page: np.ndarray, head: np.ndarray, pos_in_page: np.ndarray):
    blk = (layer * desc.n_pages + page.astype(np.int64)) * desc.n_kv_heads + head.astype(np.int64)
    return blk * desc.page_head_bytes + (pos_in_page.astype(np.int64) // 16) * desc.tile_bytes


def np_kv_write_rows(desc: PoolDesc, pool: np.ndarray, layer: int, k: np.ndarray, v: np.ndarray,
                     row_entry: np.ndarray, row_pos: np.ndarray, block_table: np.ndarray) -> int:
    """Vectorised twin of c_kv_write_rows (same skip rules); returns the skipped row count."""
    P, H, NB = desc.page_size, desc.n_kv_heads, desc.n_groups
    max_blocks = block_table.shape[1]
    row_entry = np.asarray(row_entry, np.int64)
    row_pos = np.asarray(row_pos, np.int64)
    ok = (row_pos >= 0) & (row_pos < max_blocks * P)
    page = np.zeros_like(row_pos)
    page[ok] = block_table[row_entry[ok], row_pos[ok] // P]
    ok &= (page >= 0) & (page < desc.n_pages)
    idx = np.nonzero(ok)[0]
    if idx.size == 0:
        return int(len(row_pos))
    koff, voff, ksoff, vsoff = layout_maps(desc)
    kq, kd = np_quantize_q8(k[idx], desc.group_size)
    vq, vd = np_quantize_q8(v[idx], desc.group_size)
    t = row_pos[idx] % 16
    for h in range(H):
        base = np_tile_base(desc, layer, page[idx], np.full(idx.size, h), row_pos[idx] % P)
        pool[base[:, None] + koff[t]] = excess128(kq[:, h, :])
        pool[base[:, None] + voff[t]] = excess128(vq[:, h, :])
        kdb = np.ascontiguousarray(kd[:, h, :]).view(np.uint8).reshape(-1, NB, 2)
        vdb = np.ascontiguousarray(vd[:, h, :]).view(np.uint8).reshape(-1, NB, 2)
        for byte in range(2):
            pool[base[:, None] + ksoff[t] + byte] = kdb[:, :, byte]
            pool[base[:, None] + vsoff[t] + byte] = vdb[:, :, byte]
    return int(len(row_pos) - idx.size)


def np_dequant_entry(desc: PoolDesc, pool: np.ndarray, layer: int, block_row: np.ndarray, n_tokens: int,
                     head: int):
    """Dequantized K, V f32 [n_tokens, D] of one entry and kv head (pages from one block-table row)."""
    P, G = desc.page_size, desc.group_size
    pos = np.arange(n_tokens)
    page = np.asarray(block_row, np.int64)[pos // P]
    base = np_tile_base(desc, layer, page, np.full(n_tokens, head), pos % P)
    koff, voff, ksoff, vsoff = layout_maps(desc)
    t = pos % 16
    kq = from_excess128(pool[base[:, None] + koff[t]]).astype(np.float32)
    vq = from_excess128(pool[base[:, None] + voff[t]]).astype(np.float32)

    def scales(off):
        lo = pool[base[:, None] + off[t]].astype(np.uint16)
        hi = pool[base[:, None] + off[t] + 1].astype(np.uint16)
        return (lo | (hi << 8)).view(np.float16).astype(np.float32)

    ks = np.repeat(scales(ksoff), G, axis=1)
    vs = np.repeat(scales(vsoff), G, axis=1)
    return kq * ks, vq * vs


def np_attn(desc: PoolDesc, pool: np.ndarray, layer: int, q: np.ndarray, cu_q, cu_k, block_table,
            scale: float) -> np.ndarray:
    """numpy twin of c_attn (float64 softmax) for small cases."""
    q = np.asarray(q, np.float16).astype(np.float64)
    Hq = q.shape[1]
    H = desc.n_kv_heads
    grp = Hq // H
    out = np.zeros(q.shape, np.float32)
    for b in range(len(cu_q) - 1):
        Tq = int(cu_q[b + 1] - cu_q[b])
        Tk = int(cu_k[b + 1] - cu_k[b])
        for h in range(H):
            K, V = np_dequant_entry(desc, pool, layer, block_table[b], Tk, h)
            for i in range(Tq):
                nk = min(Tk, Tk - Tq + i + 1)
                if nk <= 0:
                    continue
                row = int(cu_q[b]) + i
                qs = q[row, h * grp:(h + 1) * grp]
                s = qs @ K[:nk].astype(np.float64).T * scale
                s -= s.max(axis=1, keepdims=True)
                p = np.exp(s)
                out[row, h * grp:(h + 1) * grp] = (p @ V[:nk].astype(np.float64)) / p.sum(axis=1, keepdims=True)
    return out


def np_norm_rope(x: np.ndarray, w: np.ndarray, eps: float, w_offset: int, cos: np.ndarray, sin: np.ndarray,
                 rope_dim: int, pos: np.ndarray) -> np.ndarray:
    """The attention prep of attn_prepare_decode
    (docs/research/2026-09-16-head-to-head-llamacpp-and-phase-profile.md:181-216) for rows
    x f16 [rows, heads, D] at positions pos [rows]: RMSNorm with weights (w + w_offset), then the
    rotate-half RoPE on dims [0, rope_dim) from the cos/sin tables [*, rope_dim/2].  float32,
    every step rounded like the kernel's IEEE operations, the sum of squares in the kernel's order
    (32 lanes of D/32 consecutive dims, each summed in dim order, then an xor butterfly over the
    lanes with offsets 16, 8, 4, 2, 1)."""
    f32 = np.float32
    x = np.asarray(x, np.float16).astype(f32)
    R, Hh, D = x.shape
    E = D // 32
    lanes = x.reshape(R, Hh, 32, E)
    ss = np.zeros((R, Hh, 32), f32)
    for e in range(E):
        ss = (ss + lanes[..., e] * lanes[..., e]).astype(f32)
    idx = np.arange(32)
    for off in (16, 8, 4, 2, 1):
        ss = (ss + ss[..., idx ^ off]).astype(f32)
    mean = (ss[..., 0] * f32(1.0 / D)).astype(f32)
    r = (f32(1.0) / np.sqrt((mean + f32(eps)).astype(f32))).astype(f32)
    wf = (np.asarray(w, f32) + f32(w_offset)).astype(f32)
    y = ((x * r[..., None]).astype(f32) * wf).astype(f32)
    if rope_dim:
        h = rope_dim // 2
        c = np.asarray(cos, f32)[pos][:, None, :]
        s = np.asarray(sin, f32)[pos][:, None, :]
        x1, x2 = y[..., :h].copy(), y[..., h:rope_dim].copy()
        y[..., :h] = ((x1 * c).astype(f32) - (x2 * s).astype(f32)).astype(f32)
        y[..., h:rope_dim] = ((x2 * c).astype(f32) + (x1 * s).astype(f32)).astype(f32)
    return y


def np_attn_prep(qg: np.ndarray, k: np.ndarray, wq, wk, eps: float, w_offset: int, cos, sin, rope_dim: int,
                 pos: np.ndarray):
    """q f16, gate f16 [rows, Hq, D] and the normed, rotated K rounded to f16 [rows, Hkv, D] (the
    tensor the unfused path would hand to the KV append) of the fused attention prep."""
    qg = np.asarray(qg, np.float16)
    D = qg.shape[2] // 2
    q = np_norm_rope(qg[..., :D], wq, eps, w_offset, cos, sin, rope_dim, pos).astype(np.float16)
    kk = np_norm_rope(k, wk, eps, w_offset, cos, sin, rope_dim, pos).astype(np.float16)
    return q, qg[..., D:].copy(), kk


def tree_visible(ranges: np.ndarray, i: int) -> np.ndarray:
    """Draft nodes row i of a trie verify sees: node j with j <= i and start_j <= i <= end_j,
    ranges int [Tq, 2] of inclusive depth-first subtree ranges (the reference's trie mask
    "committed prefix plus the current node's subtree ranges",
    docs/plans/2026-10-09-tree-speculative-decoding.md:26-38)."""
    j = np.arange(len(ranges))
    return (j <= i) & (ranges[:, 0] <= i) & (i <= ranges[:, 1])


def np_attn_tree(desc: PoolDesc, pool: np.ndarray, layer: int, q: np.ndarray, cu_q, cu_k, block_table,
                 scale: float, trie_ranges: np.ndarray) -> np.ndarray:
    """Tree speculative verify over the dequantized pool (float64 softmax): entry b's draft rows
    are trie nodes at keys Tk-Tq .. Tk-1; row i sees keys 0 .. Tk-Tq-1 and the draft keys of the
    nodes tree_visible(ranges of b, i).  trie_ranges int [total_q, 2]."""
    q = np.asarray(q, np.float16).astype(np.float64)
    Hq = q.shape[1]
    H = desc.n_kv_heads
    grp = Hq // H
    out = np.zeros(q.shape, np.float32)
    for b in range(len(cu_q) - 1):
        q0, Tq = int(cu_q[b]), int(cu_q[b + 1] - cu_q[b])
        Tk = int(cu_k[b + 1] - cu_k[b])
        kv0 = Tk - Tq
        rng = np.asarray(trie_ranges[q0:q0 + Tq], np.int64)
        for h in range(H):
            K, V = np_dequant_entry(desc, pool, layer, block_table[b], Tk, h)
            for i in range(Tq):
                keys = np.concatenate([np.arange(kv0), kv0 + np.nonzero(tree_visible(rng, i))[0]])
                qs = q[q0 + i, h * grp:(h + 1) * grp]
                s = qs @ K[keys].astype(np.float64).T * scale
                s -= s.max(axis=1, keepdims=True)
                p = np.exp(s)
                out[q0 + i, h * grp:(h + 1) * grp] = (p @ V[keys].astype(np.float64)) / p.sum(axis=1, keepdims=True)
    return out


def np_partial_decode(q: np.ndarray, K: np.ndarray, V: np.ndarray, scale: float):
    """One decode row over one key range, as the split-KV partial the reference's combine
    consumes: q [hq, D] (f16 values), K/V [n_keys, D] dequantized.  Returns (O [hq, D]
    normalised over the range, lse [hq] = ln sum exp(q.k * scale)); a range without keys gives
    (0, -inf).  Float64."""
    q = np.asarray(q, np.float16).astype(np.float64)
    hq, D = q.shape
    if K.shape[0] == 0:
        return np.zeros((hq, D)), np.full(hq, -np.inf)
    s = q @ K.astype(np.float64).T * scale
    m = s.max(axis=1, keepdims=True)
    p = np.exp(s - m)
    l = p.sum(axis=1, keepdims=True)
    return (p @ V.astype(np.float64)) / l, (m + np.log(l))[:, 0]


def np_combine(o_parts: np.ndarray, lse_parts: np.ndarray) -> np.ndarray:
    """LSE merge of partials (flash_fwd_splitkv_combine_kernel's formula,
    docs/plans/2026-09-16-prefil-parity-fa2-and-mmq.md:104-107): o_parts [n, rows, D],
    lse_parts [n, rows] -> [rows, D]; rows whose every lse is -inf give zeros."""
    o = np.asarray(o_parts, np.float64)
    lse = np.asarray(lse_parts, np.float64)
    M = lse.max(axis=0)
    finite = np.isfinite(M)
    w = np.where(np.isfinite(lse), np.exp(lse - np.where(finite, M, 0.0)), 0.0)
    L = w.sum(axis=0)
    out = np.einsum("nr,nrd->rd", w, o)
    return np.where(L[:, None] > 0, out / np.where(L > 0, L, 1.0)[:, None], 0.0)


def error_profile(err: np.ndarray):
    """Per-head and per-row max |error| of an error tensor [1, seq, heads, dim]
    (the helper of src/bin/fa_probe.rs:107-112)."""
    a = np.abs(err)
    per_head = a.max(axis=3).max(axis=1)[0]
    per_row = a.max(axis=3).max(axis=2)[0]
    return per_head, per_row
