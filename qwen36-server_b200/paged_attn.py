"""Host-side mirror of the engine's paged-KV attention operator surface.

The names follow the reference's call sites so that engine-side code and the
parity tests read like the reference's own:

  * ``PagedKvPool``                 -- real::paged_kv_cuda's PagedKvPool
                                       (docs/plans/2026-08-27-tiered-kv-cache.md:352-353),
                                       plus a free-list page allocator with refcounts
  * ``kv_append_paged``             -- kv_append_paged_f16, one row per slot (fork quantized.cu:6996)
  * ``launch_append_multi``         -- T contiguous rows per slot (fork quantized.cu:7040)
  * ``dispatch_flash_decode_paged`` -- src/bin/decode_gqa_probe.rs:26,40-46 (q, pool, lens, table, scale)
  * ``forward_attn_prefill_paged``  -- causal chunk "row i sees 0..kv0+i"
                                       (docs/plans/2026-08-27-mtp-cuda-graphs.md:132,244-248)
  * ``forward_verify_paged``        -- MTP verify of k draft rows (same doc, :279-284, :537-541)
  * ``PagedKvPool.export_pages`` / ``restore_pages`` -- StateSnapshot::to_host / to_device
                                       of int8 pages + scales (src/prefix_cache.rs:71-91, :361)

Tensors are torch tensors on the pool's device; torch only supplies device
memory and the current stream.  Every call goes through libyfattn.so; errors
raise ``YfError`` (the reference's calls return candle_core::Error).
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional, Sequence

import torch

from . import _abi
from ._abi import YfError, call, lib


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _i32(t, device) -> torch.Tensor:
    """Block tables, lengths and positions travel as int32 (read as uint32 where the ABI says so)."""
    if not torch.is_tensor(t):
        t = torch.as_tensor(t)
    if t.dtype != torch.int32:
        t = t.to(torch.int32)
    return t.to(device).contiguous()


class PagedKvPool:
    """The persistent Q8_0 KV pool of one model: ``n_layers`` planes of ``n_pages`` pages.

    ``device=None`` builds a host-only pool that carries only the page allocator.
    """

    def __init__(self, n_layers: int, n_pages: int, n_kv_heads: int, head_dim: int, page_size: int = 16,
                 group_size: int = 32, device: Optional[int] = 0):
        self.desc = _abi.PoolDesc(n_layers, n_pages, n_kv_heads, head_dim, page_size, group_size,
                                  -1 if device is None else int(device), 0, None)
        self.device = None if device is None else torch.device("cuda", int(device))
        h = ctypes.c_void_p()
        call("yf_pool_create", ctypes.byref(self.desc), ctypes.byref(h))
        self._h = h
        self._ws = None

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    n_layers = property(lambda self: self.desc.n_layers)
    n_pages = property(lambda self: self.desc.n_pages)
    n_kv_heads = property(lambda self: self.desc.n_kv_heads)
    head_dim = property(lambda self: self.desc.head_dim)
    page_size = property(lambda self: self.desc.page_size)
    group_size = property(lambda self: self.desc.group_size)

    @property
    def page_head_bytes(self) -> int:
        return lib().yf_pool_page_head_bytes(ctypes.byref(self.desc))

    @property
    def page_bytes(self) -> int:
        return self.page_head_bytes * self.n_kv_heads

    @property
    def bytes(self) -> int:
        return lib().yf_pool_bytes(ctypes.byref(self.desc))

    def layer_ptr(self, layer: int) -> int:
        p = ctypes.c_void_p()
        call("yf_pool_layer_ptr", self._h, layer, ctypes.byref(p))
        return p.value or 0

    def layer_bytes_view(self, layer: int) -> torch.Tensor:
        """A uint8 tensor aliasing one layer plane (device memory owned by the pool)."""
        return _alias_u8(self.layer_ptr(layer), self.n_pages * self.page_bytes, self.device)

    # -- allocator ------------------------------------------------------------------
    def alloc_pages(self, n: int) -> list:
        out = (ctypes.c_int32 * max(n, 1))()
        call("yf_pool_alloc_pages", self._h, n, out)
        return list(out[:n])

    def retain_pages(self, pages: Sequence[int]) -> None:
        arr = (ctypes.c_int32 * max(len(pages), 1))(*pages)
        call("yf_pool_retain_pages", self._h, len(pages), arr)

    def free_pages(self, pages: Sequence[int]) -> None:
        arr = (ctypes.c_int32 * max(len(pages), 1))(*pages)
        call("yf_pool_free_pages", self._h, len(pages), arr)

    def free_count(self) -> int:
        v = ctypes.c_int32()
        call("yf_pool_free_count", self._h, ctypes.byref(v))
        return v.value

    def refcount(self, page: int) -> int:
        v = ctypes.c_int32()
        call("yf_pool_refcount", self._h, page, ctypes.byref(v))
        return v.value

    # -- options (yf_attn_options) ----------------------------------------------------
    def options(self) -> dict:
        """The pool's attention options as a dict of field -> value."""
        o = _abi.AttnOptions()
        call("yf_pool_get_options", self._h, ctypes.byref(o))
        return {f: getattr(o, f) for f, _ in o._fields_ if f != "reserved"}

    def set_options(self, **fields) -> None:
        """Replaces the named options (others keep their values): schedule, chunk_tiles,
        copy_stages, merge, prefill_kernel, wait_limit_us."""
        cur = self.options()
        cur.update(fields)
        o = _abi.AttnOptions(**cur)
        call("yf_pool_set_options", self._h, ctypes.byref(o))

    def plant_counter(self, index: int, value: int) -> None:
        """Fault-injection hook for the bounded waits: stores ``value`` into merge counter ``index``."""
        call("yf_pool_plant_counter", self._h, index, value, _stream(self.device))

    def status(self, clear: bool = True) -> int:
        """Device status bits (YF_DEV_*); synchronizes the device."""
        v = ctypes.c_uint32()
        call("yf_pool_status", self._h, ctypes.byref(v), 1 if clear else 0)
        return v.value

    # -- snapshots ------------------------------------------------------------------
    def export_pages(self, layer: int, pages: Sequence[int], out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Bytes of ``pages`` (one layer, all kv heads) back to back; pinned host memory by default."""
        n = len(pages)
        if out is None:
            out = torch.empty(n * self.page_bytes, dtype=torch.uint8, pin_memory=True)
        arr = (ctypes.c_int32 * max(n, 1))(*pages)
        call("yf_pool_export_pages", self._h, layer, n, arr, ctypes.c_void_p(out.data_ptr()), _stream(self.device))
        return out

    def restore_pages(self, layer: int, pages: Sequence[int], snapshot: torch.Tensor) -> None:
        """Copies a snapshot made by export_pages into ``pages`` (no requantization)."""
        n = len(pages)
        if snapshot.numel() * snapshot.element_size() < n * self.page_bytes:
            raise YfError(_abi.YF_E_INVALID, "restore_pages", "snapshot smaller than the page list")
        arr = (ctypes.c_int32 * max(n, 1))(*pages)
        call("yf_pool_restore_pages", self._h, layer, n, arr, ctypes.c_void_p(snapshot.data_ptr()),
             _stream(self.device))

    # -- snapshot wire records (pages.kv, docs/plans/2026-08-27-tiered-kv-cache.md:141-145,237-251) --
    @property
    def record_bytes(self) -> int:
        """Bytes of one record: 32 + 4 * page_size header bytes + the page in every layer."""
        return lib().yf_pool_record_bytes(ctypes.byref(self.desc))

    def export_records(self, pages, chain_hashes=None, page_indices=None, prev_hashes=None, tokens=None,
                       out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Records [u64 chain_hash][u64 prev_hash][u32 page_index][u32 n_tokens][u32 payload_len]
        [u32 crc32c][u32 tokens[page_size]][payload] of ``pages`` back to back in a device uint8
        tensor, the CRC-32C (over token ids and payload) computed on the GPU.  ``tokens``: the
        pages' token ids, [n, page_size]."""
        pg = _i32(pages, self.device)
        n = pg.numel()
        if out is None:
            out = torch.empty(n * self.record_bytes, dtype=torch.uint8, device=self.device)
        u64 = lambda a: None if a is None else torch.as_tensor(a, dtype=torch.int64).to(self.device)  # noqa: E731
        pi = None if page_indices is None else _i32(page_indices, self.device)
        tk = None if tokens is None else _i32(tokens, self.device).reshape(n, self.page_size).contiguous()
        hs, pv = u64(chain_hashes), u64(prev_hashes)   # held until the launch is queued
        call("yf_pool_export_records", self._h, n, _ptr(pg), _ptr(hs), _ptr(pv), _ptr(pi), _ptr(tk), _ptr(out),
             _stream(self.device))
        return out

    def import_records(self, pages, records: torch.Tensor, expect_hashes=None, expect_tokens=None) -> torch.Tensor:
        """Restores the intact records of ``records`` (device) into ``pages``; with expected chain
        hashes and/or token ids, only records that carry them.  Returns per-record verdicts
        (int32 YF_REC_REJECTED 0 / YF_REC_RESTORED 1 / YF_REC_MISMATCH 2)."""
        pg = _i32(pages, self.device)
        n = pg.numel()
        if records.numel() * records.element_size() < n * self.record_bytes:
            raise YfError(_abi.YF_E_INVALID, "import_records", "records smaller than the page list")
        ok = torch.zeros(n, dtype=torch.int32, device=self.device)
        eh = None if expect_hashes is None else torch.as_tensor(expect_hashes, dtype=torch.int64).to(self.device)
        et = None if expect_tokens is None else _i32(expect_tokens, self.device).reshape(n, self.page_size).contiguous()
        call("yf_pool_import_records", self._h, n, _ptr(pg), _ptr(records), _ptr(eh), _ptr(et), _ptr(ok),
             _stream(self.device))
        return ok

    # -- workspace ------------------------------------------------------------------
    def workspace_size(self, n_q_heads: int, batch: int, max_seqlen_q: int, max_seqlen_k: int) -> int:
        return lib().yf_attn_workspace_size(self._h, n_q_heads, batch, max_seqlen_q, max_seqlen_k)

    def workspace(self, nbytes: int) -> Optional[torch.Tensor]:
        """A cached device buffer of at least ``nbytes`` (grown, never shrunk)."""
        if nbytes <= 0:
            return None
        if self._ws is None or self._ws.numel() < nbytes:
            self._ws = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        return self._ws

    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            lib().yf_pool_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _alias_u8(ptr: int, n: int, device: torch.device) -> torch.Tensor:
    """Wraps foreign device memory as a uint8 tensor without copying (lifetime: the owner's)."""

    class _Holder:
        __cuda_array_interface__ = {"shape": (n,), "typestr": "|u1", "data": (ptr, False), "version": 2,
                                    "strides": None}

    return torch.as_tensor(_Holder(), device=device)


# ---- KV write ------------------------------------------------------------------------

def _check_rows(pool: PagedKvPool, k: torch.Tensor, v: torch.Tensor) -> None:
    if k.dtype != torch.float16 or v.dtype != torch.float16:
        raise YfError(_abi.YF_E_INVALID, "kv write", "k and v must be float16")
    if k.shape != v.shape or k.dim() != 3 or k.shape[1] != pool.n_kv_heads or k.shape[2] != pool.head_dim:
        raise YfError(_abi.YF_E_INVALID, "kv write", f"k/v must be [rows, {pool.n_kv_heads}, {pool.head_dim}]")
    if not (k.is_contiguous() and v.is_contiguous()):
        raise YfError(_abi.YF_E_INVALID, "kv write", "k and v must be contiguous")


def kv_append_paged(pool: PagedKvPool, layer: int, k: torch.Tensor, v: torch.Tensor, pos, block_table) -> None:
    """Quantize one new K/V row per batch entry into its page: k, v f16 [B, Hkv, D]; pos int [B]."""
    _check_rows(pool, k, v)
    pos = _i32(pos, pool.device)
    bt = _i32(block_table, pool.device)
    call("yf_kv_append_paged", pool.handle, layer, _ptr(k), _ptr(v), _ptr(pos), _ptr(bt), bt.shape[1], k.shape[0],
         _stream(pool.device))


def launch_append_multi(pool: PagedKvPool, layer: int, k: torch.Tensor, v: torch.Tensor, cu_rows, start_pos,
                        block_table, max_rows: Optional[int] = None) -> None:
    """Quantize T contiguous rows per entry: k, v f16 [total_rows, Hkv, D]; entry b's rows
    cu_rows[b]..cu_rows[b+1]-1 go to positions start_pos[b]+i."""
    _check_rows(pool, k, v)
    if max_rows is None:
        max_rows = _max_len(cu_rows)
    cu = _i32(cu_rows, pool.device)
    sp = _i32(start_pos, pool.device)
    bt = _i32(block_table, pool.device)
    call("yf_kv_append_paged_multi", pool.handle, layer, _ptr(k), _ptr(v), _ptr(cu), _ptr(sp), _ptr(bt),
         bt.shape[1], cu.numel() - 1, max_rows, _stream(pool.device))


# ---- attention -----------------------------------------------------------------------

def attn_prepare_append(pool: PagedKvPool, layer: int, qg: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                        q_norm_w: torch.Tensor, k_norm_w: torch.Tensor, eps: float, rope_cos: Optional[torch.Tensor],
                        rope_sin: Optional[torch.Tensor], rope_dim: int, cu_rows, start_pos, block_table,
                        norm_weight_offset: int = 1, max_rows: Optional[int] = None,
                        q_out: Optional[torch.Tensor] = None, gate_out: Optional[torch.Tensor] = None):
    """The engine's attn_prepare_decode fused with the KV append
    (docs/research/2026-09-16-head-to-head-llamacpp-and-phase-profile.md:181-216): q and k RMSNorm
    (weights w + norm_weight_offset), rotate-half RoPE on the first rope_dim dims from the cos/sin
    tables [rows, rope_dim/2], the gate half split out, and K/V written into the pool as Q8_0.
    qg f16 [T, Hq, 2D] (q then gate per head), k/v f16 [T, Hkv, D]; returns (q, gate) f16
    [T, Hq, D]."""
    T, Hq, D2 = qg.shape
    D = pool.head_dim
    if qg.dtype != torch.float16 or D2 != 2 * D or not qg.is_contiguous():
        raise YfError(_abi.YF_E_INVALID, "attn_prepare_append", "qg must be contiguous f16 [T, Hq, 2*head_dim]")
    _check_rows(pool, k, v)
    cu = _i32(cu_rows, pool.device)
    start = _i32(start_pos, pool.device)
    table = _i32(block_table, pool.device)
    if max_rows is None:
        max_rows = _max_len(cu_rows)
    wq = q_norm_w.to(device=pool.device, dtype=torch.float32).contiguous()
    wk = k_norm_w.to(device=pool.device, dtype=torch.float32).contiguous()
    if rope_dim:
        rc = rope_cos.to(device=pool.device, dtype=torch.float32).contiguous()
        rs = rope_sin.to(device=pool.device, dtype=torch.float32).contiguous()
        rows = rc.shape[0]
    else:
        rc = rs = None
        rows = 0
    if q_out is None:
        q_out = torch.empty((T, Hq, D), dtype=torch.float16, device=qg.device)
    if gate_out is None:
        gate_out = torch.empty((T, Hq, D), dtype=torch.float16, device=qg.device)
    call("yf_attn_prepare_append", pool.handle, layer, Hq, _ptr(qg), _ptr(k), _ptr(v), _ptr(wq), _ptr(wk),
         ctypes.c_float(eps), int(norm_weight_offset), _ptr(rc), _ptr(rs), int(rope_dim), int(rows), _ptr(cu),
         _ptr(start), _ptr(table), table.shape[1], cu.numel() - 1, int(max_rows), _ptr(q_out), _ptr(gate_out),
         _stream(pool.device))
    return q_out, gate_out


def _max_len(cu) -> int:
    c = torch.as_tensor(cu).to("cpu", torch.int64)
    return int((c[1:] - c[:-1]).max()) if c.numel() > 1 else 0


def _ws_args(pool: PagedKvPool, workspace: Optional[torch.Tensor], nbytes: int):
    if workspace is None:
        workspace = pool.workspace(nbytes)
    size = 0 if workspace is None else workspace.numel() * workspace.element_size()
    return _ptr(workspace), size


def dispatch_flash_decode_paged(q: torch.Tensor, pool: PagedKvPool, layer: int, lens, table, scale: float,
                                max_seqlen_k: Optional[int] = None, out: Optional[torch.Tensor] = None,
                                workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Batched paged decode attention.  q f16 [B, Hq, D]; lens = cu_seqlens_k [B+1] (as the
    probe's ``lens``); table [B, max_blocks].  Returns f16 [B, Hq, D]."""
    B, Hq, D = q.shape
    if q.dtype != torch.float16 or D != pool.head_dim or not q.is_contiguous():
        raise YfError(_abi.YF_E_INVALID, "dispatch_flash_decode_paged", "q must be contiguous f16 [B, Hq, D]")
    if max_seqlen_k is None:
        max_seqlen_k = _max_len(lens)
    lens = _i32(lens, pool.device)
    table = _i32(table, pool.device)
    if out is None:
        out = torch.empty_like(q)
    ws, ws_bytes = _ws_args(pool, workspace, pool.workspace_size(Hq, B, 1, max_seqlen_k))
    call("yf_attn_decode", pool.handle, layer, _ptr(q), Hq, _ptr(lens), _ptr(table), table.shape[1], B,
         max_seqlen_k, ctypes.c_float(scale), _ptr(out), ws, ws_bytes, _stream(pool.device))
    return out


def dispatch_flash_decode_partial(q: torch.Tensor, pool: PagedKvPool, layer: int, lens, table, scale: float,
                                  max_seqlen_k: Optional[int] = None, o_part: Optional[torch.Tensor] = None,
                                  lse_part: Optional[torch.Tensor] = None,
                                  workspace: Optional[torch.Tensor] = None):
    """Decode over the keys this pool holds (one shard), as partials: returns (o f32 [B, Hq, D]
    normalised over the shard, lse f32 [B, Hq] natural-log log-sum-exp of the scaled logits)."""
    B, Hq, D = q.shape
    if q.dtype != torch.float16 or D != pool.head_dim or not q.is_contiguous():
        raise YfError(_abi.YF_E_INVALID, "dispatch_flash_decode_partial", "q must be contiguous f16 [B, Hq, D]")
    if max_seqlen_k is None:
        max_seqlen_k = _max_len(lens)
    lens = _i32(lens, pool.device)
    table = _i32(table, pool.device)
    if o_part is None:
        o_part = torch.empty((B, Hq, D), dtype=torch.float32, device=q.device)
    if lse_part is None:
        lse_part = torch.empty((B, Hq), dtype=torch.float32, device=q.device)
    ws, ws_bytes = _ws_args(pool, workspace, pool.workspace_size(Hq, B, 1, max_seqlen_k))
    call("yf_attn_decode_partial", pool.handle, layer, _ptr(q), Hq, _ptr(lens), _ptr(table), table.shape[1], B,
         max_seqlen_k, ctypes.c_float(scale), _ptr(o_part), _ptr(lse_part), ws, ws_bytes, _stream(pool.device))
    return o_part, lse_part


def combine_partials(o_parts: torch.Tensor, lse_parts: torch.Tensor, out: Optional[torch.Tensor] = None, *,
                     n_parts: Optional[int] = None, rows: Optional[int] = None, head_dim: Optional[int] = None,
                     o_part_stride: Optional[int] = None, lse_part_stride: Optional[int] = None):
    """LSE merge of n partials into f16 [rows, D] (or ``out``).  By default o_parts is f32
    [n, rows, D] and lse_parts f32 [n, rows]; with explicit counts and strides (in floats) both
    may be views into one buffer that packs each part's O and lse together."""
    if n_parts is None:
        n_parts = int(o_parts.shape[0])
    if head_dim is None:
        head_dim = int(o_parts.shape[-1])
    if rows is None:
        rows = int(lse_parts[0].numel())
    if o_part_stride is None:
        o_part_stride = rows * head_dim
    if lse_part_stride is None:
        lse_part_stride = rows
    if o_parts.dtype != torch.float32 or lse_parts.dtype != torch.float32:
        raise YfError(_abi.YF_E_INVALID, "combine_partials", "partials must be f32")
    need_o = (n_parts - 1) * o_part_stride + rows * head_dim
    need_l = (n_parts - 1) * lse_part_stride + rows
    if o_parts.numel() < need_o or lse_parts.numel() < need_l:
        raise YfError(_abi.YF_E_INVALID, "combine_partials", "partials smaller than n_parts x strides")
    if out is None:
        out = torch.empty((rows, head_dim), dtype=torch.float16, device=o_parts.device)
    call("yf_attn_combine", _ptr(o_parts), int(o_part_stride), _ptr(lse_parts), int(lse_part_stride), n_parts,
         rows, head_dim, _ptr(out), _stream(o_parts.device))
    return out


def forward_attn_prefill_paged(q: torch.Tensor, pool: PagedKvPool, layer: int, cu_seqlens_q, cu_seqlens_k, table,
                               scale: float, max_seqlen_q: Optional[int] = None,
                               max_seqlen_k: Optional[int] = None, out: Optional[torch.Tensor] = None,
                               workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Causal attention of query blocks against the pool.  q f16 [total_q, Hq, D]; entry b's
    rows cu_seqlens_q[b].. see keys 0..Tk_b-Tq_b+i (its new K/V rows must already be written)."""
    T, Hq, D = q.shape
    if q.dtype != torch.float16 or D != pool.head_dim or not q.is_contiguous():
        raise YfError(_abi.YF_E_INVALID, "forward_attn_prefill_paged", "q must be contiguous f16 [T, Hq, D]")
    if max_seqlen_q is None:
        max_seqlen_q = _max_len(cu_seqlens_q)
    if max_seqlen_k is None:
        max_seqlen_k = _max_len(cu_seqlens_k)
    max_seqlen_q = max(int(max_seqlen_q), 1)
    cq = _i32(cu_seqlens_q, pool.device)
    ck = _i32(cu_seqlens_k, pool.device)
    table = _i32(table, pool.device)
    B = ck.numel() - 1
    if out is None:
        out = torch.empty_like(q)
    ws, ws_bytes = _ws_args(pool, workspace, pool.workspace_size(Hq, B, max_seqlen_q, max_seqlen_k))
    call("yf_attn_prefill", pool.handle, layer, _ptr(q), Hq, _ptr(cq), _ptr(ck), _ptr(table), table.shape[1], B,
         max_seqlen_q, max_seqlen_k, ctypes.c_float(scale), _ptr(out), ws, ws_bytes, _stream(pool.device))
    return out


def forward_verify_paged(q: torch.Tensor, pool: PagedKvPool, layer: int, cu_seqlens_q, cu_seqlens_k, table,
                         scale: float, **kw) -> torch.Tensor:
    """MTP verify: k draft rows per slot, row j sees ctx+j+1 keys (the draft rows are in the pool).
    The same causal call as prefill; with k*G <= 16 rows per kv head it runs the split-KV kernel
    with GQA folded into the MMA N dimension (the reference's per_row_gqa decode mode)."""
    return forward_attn_prefill_paged(q, pool, layer, cu_seqlens_q, cu_seqlens_k, table, scale, **kw)


def forward_verify_tree_paged(q: torch.Tensor, pool: PagedKvPool, layer: int, cu_seqlens_q, cu_seqlens_k, table,
                              scale: float, trie_ranges, max_seqlen_q: Optional[int] = None,
                              max_seqlen_k: Optional[int] = None, out: Optional[torch.Tensor] = None,
                              workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Tree speculative verify (the reference's forward_verify_tree_graphed with trie_ranges,
    docs/plans/2026-10-09-tree-speculative-decoding.md:26-38): each entry's <= 64 draft rows are
    trie nodes in depth-first order and trie_ranges (int32 [total_q, 2]) holds every node's
    inclusive subtree range [start, end] within its entry; row i sees the committed keys and the
    draft keys of i and its ancestors (node j with j <= i and start_j <= i <= end_j)."""
    T, Hq, D = q.shape
    if q.dtype != torch.float16 or D != pool.head_dim or not q.is_contiguous():
        raise YfError(_abi.YF_E_INVALID, "forward_verify_tree_paged", "q must be contiguous f16 [T, Hq, D]")
    if max_seqlen_q is None:
        max_seqlen_q = _max_len(cu_seqlens_q)
    if max_seqlen_k is None:
        max_seqlen_k = _max_len(cu_seqlens_k)
    max_seqlen_q = max(int(max_seqlen_q), 1)
    cq = _i32(cu_seqlens_q, pool.device)
    ck = _i32(cu_seqlens_k, pool.device)
    table = _i32(table, pool.device)
    tr = _i32(trie_ranges, pool.device).reshape(-1, 2).contiguous()
    if tr.shape[0] != T:
        raise YfError(_abi.YF_E_INVALID, "forward_verify_tree_paged", "trie_ranges must be int32 [total_q, 2]")
    B = ck.numel() - 1
    if out is None:
        out = torch.empty_like(q)
    ws, ws_bytes = _ws_args(pool, workspace, pool.workspace_size(Hq, B, max_seqlen_q, max_seqlen_k))
    call("yf_attn_verify_tree", pool.handle, layer, _ptr(q), Hq, _ptr(cq), _ptr(ck), _ptr(table), table.shape[1], B,
         max_seqlen_q, max_seqlen_k, ctypes.c_float(scale), _ptr(tr), _ptr(out), ws, ws_bytes, _stream(pool.device))
    return out


def default_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
