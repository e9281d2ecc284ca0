"""Multi-GPU partitions of the attention path.

Independent slots (continuous-batched decode, MTP verify) go to GPUs by longest-processing-time
bin packing on their context (lpt_partition): each GPU holds its slots' pages in its own pool and
nothing crosses NVLink on the data path.

Long-context decode is split across GPUs: kv heads first, then contiguous key ranges.

A sequence too long for one GPU to read quickly (the 131072-key, 2-kv-head decode) is
split into world = n_head_groups x n_seq shards.  Rank r owns kv-head group r % n_head_groups
and key range r // n_head_groups of the sequence, holds only those pages in its own pool,
and runs yf_attn_decode_partial over them.  Every rank's packed partial
([O f32 B*hq*D | lse f32 B*hq]) reaches every rank through one all-gather (NCCL over
NVLink), and yf_attn_combine merges the key ranges of each head group in place in the
gathered buffer.  This replaces the reference's single-GPU split-KV + combine
(flash_fwd_splitkv_combine_kernel, docs/plans/2026-09-16-prefil-parity-fa2-and-mmq.md:104-107)
for a sequence spread over GPUs; partitions with independent slots need no such exchange.

The "p2p" transport (PeerExchange) replaces that all-gather and combine with two kernels of
libyfattn.so over NVLink peer memory: a push that stores this rank's partial straight into
every rank's exchange area and raises a release flag there, and a combine that waits (bounded)
for every rank's flag in its own area and merges in place.  No collective library call remains
on the data path; the areas are mapped once with CUDA IPC when the decode is built.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import List

import torch

from . import _abi
from . import paged_attn as pa
from ._abi import call, lib


def lpt_partition(costs, n_bins: int) -> List[List[int]]:
    """Longest-processing-time-first assignment of independent slots to ``n_bins`` GPUs: slots
    in order of falling cost (ties by index), each to the bin with the least cost so far (ties by
    bin index).  A slot's cost is the KV bytes its attention reads, proportional to its context.
    Returns each bin's slot indices in ascending order; deterministic for a given input."""
    if n_bins < 1:
        raise ValueError("n_bins must be >= 1")
    c = [int(x) for x in costs]
    order = sorted(range(len(c)), key=lambda i: (-c[i], i))
    load = [0] * n_bins
    bins: List[List[int]] = [[] for _ in range(n_bins)]
    for i in order:
        j = min(range(n_bins), key=lambda b: (load[b], b))
        bins[j].append(i)
        load[j] += c[i]
    return [sorted(b) for b in bins]


@dataclass(frozen=True)
class LongShard:
    """What rank `rank` of `world` holds."""
    rank: int
    world: int
    n_head_groups: int
    head_group: int
    kv_head0: int       # first kv head of the group
    kv_heads: int       # kv heads per group
    n_seq: int
    seq: int
    k0: int             # first key of the range
    k1: int             # one past the last key


def long_context_plan(world: int, n_kv_heads: int, ctx: int, page_size: int = 16) -> List[LongShard]:
    """Shards of one sequence of `ctx` keys: world divides n_kv_heads (heads split, whole
    sequence per rank) or n_kv_heads divides world (one head group of one kv head, and
    world / n_kv_heads page-aligned key ranges).  Rank order is seq-major:
    rank = seq * n_head_groups + head_group."""
    if world < 1 or n_kv_heads < 1:
        raise ValueError("world and n_kv_heads must be >= 1")
    if world <= n_kv_heads:
        if n_kv_heads % world:
            raise ValueError(f"world {world} does not divide n_kv_heads {n_kv_heads}")
        n_hg, n_seq = world, 1
    else:
        if world % n_kv_heads:
            raise ValueError(f"n_kv_heads {n_kv_heads} does not divide world {world}")
        n_hg, n_seq = n_kv_heads, world // n_kv_heads
    hpg = n_kv_heads // n_hg
    per = -(-(-(-ctx // n_seq)) // page_size) * page_size
    out = []
    for r in range(world):
        hg, s = r % n_hg, r // n_hg
        out.append(LongShard(r, world, n_hg, hg, hg * hpg, hpg, n_seq, s, min(ctx, s * per), min(ctx, (s + 1) * per)))
    return out


def packed_floats(batch: int, q_heads: int, head_dim: int) -> int:
    """Floats of one rank's packed partial: O [batch, q_heads, head_dim] then lse [batch, q_heads],
    padded so that every rank's O starts 16-byte aligned in the gathered buffer."""
    n = batch * q_heads * (head_dim + 1)
    return -(-n // 4) * 4


def combine_views(shard: LongShard, batch: int, q_heads: int, head_dim: int):
    """For each head group g: (o_offset, lse_offset, part_stride, n_parts, rows) of its parts
    in the gathered buffer [world][packed_floats], in floats."""
    blk = packed_floats(batch, q_heads, head_dim)
    rows = batch * q_heads
    return [(g * blk, g * blk + rows * head_dim, shard.n_head_groups * blk, shard.n_seq, rows)
            for g in range(shard.n_head_groups)]


def gather_packed(local: torch.Tensor, gathered: torch.Tensor, world: int, group=None) -> None:
    """Every rank's packed partial into `gathered` [world * len(local)], in rank order."""
    if world > 1:
        torch.distributed.all_gather_into_tensor(gathered, local, group=group)
    else:
        gathered.copy_(local)


class PeerExchange:
    """One rank's end of the NVLink partial exchange (yf_exchange_* of libyfattn.so).

    Every rank's partial is ``slot_floats`` f32 (packed_floats: O then lse).  ``connect`` maps
    all ranks' areas into each other over a process group (their IPC handles travel through
    one all-gather at set-up); ``emulated`` builds ``world`` exchanges on one GPU attached to
    each other, for tests that run every rank's push and then every rank's combine."""

    def __init__(self, rank: int, world: int, slot_floats: int, device: int = 0, wait_limit_us: int = 0):
        if slot_floats % 4:
            raise ValueError("slot_floats must be a multiple of 4")
        self.rank, self.world, self.slot_floats = rank, world, slot_floats
        self.device = torch.device("cuda", device)
        h = ctypes.c_void_p()
        call("yf_exchange_create", device, rank, world, slot_floats, ctypes.byref(h))
        self._h = h
        if wait_limit_us:
            call("yf_exchange_set_wait_limit", self._h, wait_limit_us)

    def handle(self) -> bytes:
        buf = (ctypes.c_uint8 * _abi.YF_EXCHANGE_HANDLE_BYTES)()
        call("yf_exchange_handle", self._h, buf)
        return bytes(buf)

    def open_peer(self, peer: int, handle: bytes) -> None:
        buf = (ctypes.c_uint8 * _abi.YF_EXCHANGE_HANDLE_BYTES).from_buffer_copy(handle)
        call("yf_exchange_open_peer", self._h, peer, buf)

    def attach(self, peer: int, other: "PeerExchange") -> None:
        call("yf_exchange_attach", self._h, peer, other._h)

    def set_wait_limit(self, wait_limit_us: int) -> None:
        call("yf_exchange_set_wait_limit", self._h, wait_limit_us)

    def push(self, local: torch.Tensor) -> None:
        if local.dtype != torch.float32 or local.numel() < self.slot_floats or not local.is_contiguous():
            raise ValueError("local partial must be contiguous f32 of at least slot_floats")
        call("yf_exchange_push", self._h, ctypes.c_void_p(local.data_ptr()), pa._stream(self.device))

    def combine(self, out: torch.Tensor, n_head_groups: int, n_seq: int, rows: int, hq: int, n_q_heads: int,
                head_dim: int, lse_offset: int) -> torch.Tensor:
        if out.dtype != torch.float16 or out.numel() < rows // hq * n_q_heads * head_dim:
            raise ValueError("out must be f16 [rows / hq, n_q_heads, head_dim]")
        call("yf_exchange_combine", self._h, n_head_groups, n_seq, rows, hq, n_q_heads, head_dim, lse_offset,
             ctypes.c_void_p(out.data_ptr()), pa._stream(self.device))
        return out

    def decode(self, pool, q: torch.Tensor, cu_k, table, scale: float, max_seqlen_k: int, n_head_groups: int,
               n_seq: int, n_q_heads: int, out: torch.Tensor, workspace: torch.Tensor, layer: int = 0) -> torch.Tensor:
        """The whole sharded step (yf_exchange_decode): this rank's partial over `pool` stored into
        every rank's area, then every rank's partial merged into ``out`` [B, n_q_heads, D] f16 --
        one launch where the cluster decode schedule applies.  Ranks on separate GPUs only."""
        batch, hq = int(q.shape[0]), int(q.shape[1])
        if out.dtype != torch.float16 or out.numel() < batch * n_q_heads * q.shape[-1]:
            raise ValueError("out must be f16 [B, n_q_heads, D]")
        cu = pa._i32(cu_k, self.device)
        bt = pa._i32(table, self.device)
        call("yf_exchange_decode", self._h, pool.handle, layer, ctypes.c_void_p(q.data_ptr()), hq,
             ctypes.c_void_p(cu.data_ptr()), ctypes.c_void_p(bt.data_ptr()), bt.shape[1], batch, max_seqlen_k,
             ctypes.c_float(scale), n_head_groups, n_seq, n_q_heads, ctypes.c_void_p(out.data_ptr()),
             ctypes.c_void_p(workspace.data_ptr()), workspace.numel(), pa._stream(self.device))
        return out

    def status(self, clear: bool = False) -> int:
        v = ctypes.c_uint32()
        call("yf_exchange_status", self._h, ctypes.byref(v), int(clear))
        return v.value

    @classmethod
    def connect(cls, rank: int, world: int, slot_floats: int, device: int = 0, group=None,
                wait_limit_us: int = 0) -> "PeerExchange":
        """Creates this rank's exchange and maps every other rank's area (collective call)."""
        ex = cls(rank, world, slot_floats, device, wait_limit_us)
        if world > 1:
            nb = _abi.YF_EXCHANGE_HANDLE_BYTES
            backend = torch.distributed.get_backend(group)
            where = ex.device if backend == "nccl" else torch.device("cpu")
            mine = torch.tensor(list(ex.handle()), dtype=torch.uint8, device=where)
            every = torch.empty(world * nb, dtype=torch.uint8, device=where)
            torch.distributed.all_gather_into_tensor(every, mine, group=group)
            every = every.cpu().numpy().tobytes()
            for r in range(world):
                if r != rank:
                    ex.open_peer(r, every[r * nb:(r + 1) * nb])
            torch.distributed.barrier(group=group)
        return ex

    @classmethod
    def emulated(cls, world: int, slot_floats: int, device: int = 0, wait_limit_us: int = 0):
        xs = [cls(r, world, slot_floats, device, wait_limit_us) for r in range(world)]
        for a in xs:
            for b in xs:
                if a is not b:
                    a.attach(b.rank, b)
            a.is_emulated = world > 1
        return xs

    is_emulated = False

    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            lib().yf_exchange_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ShardedLongDecode:
    """One rank's share of a sharded decode (batch entries, all of one length split alike).

    ``pool`` holds this rank's kv heads and key range; the caller writes the shard's keys into
    it (positions k - k0) and passes the shard's cu_seqlens_k / block table to step()."""

    def __init__(self, shard: LongShard, n_q_heads: int, n_kv_heads: int, head_dim: int, n_pages: int,
                 page_size: int = 16, group_size: int = 32, batch: int = 1, device: int = 0,
                 process_group=None, transport: str = "nccl", peer_exchange: "PeerExchange" = None):
        if n_q_heads % n_kv_heads:
            raise ValueError("n_q_heads must be a multiple of n_kv_heads")
        self.shard, self.batch, self.D = shard, batch, head_dim
        self.G = n_q_heads // n_kv_heads
        self.hq = shard.kv_heads * self.G  # q heads of this rank
        self.Hq = n_q_heads
        self.group = process_group
        self.dev = torch.device("cuda", device)
        self.pool = pa.PagedKvPool(1, n_pages, shard.kv_heads, head_dim, page_size, group_size, device=device)
        blk = packed_floats(batch, self.hq, head_dim)
        self.local = torch.zeros(blk, dtype=torch.float32, device=self.dev)
        self.gathered = torch.zeros(shard.world * blk, dtype=torch.float32, device=self.dev)
        n_o = batch * self.hq * head_dim
        self.o_part = self.local[:n_o].view(batch, self.hq, head_dim)
        self.lse_part = self.local[n_o:n_o + batch * self.hq].view(batch, self.hq)
        self.out = torch.empty((batch, n_q_heads, head_dim), dtype=torch.float16, device=self.dev)
        self._grp_out = None if batch == 1 or shard.n_head_groups == 1 else torch.empty(
            (shard.n_head_groups, batch * self.hq, head_dim), dtype=torch.float16, device=self.dev)
        # workspace for the shard's whole key range, so a context that grows step by step never
        # outgrows it (partial() still re-checks against the call's own max_seqlen_k)
        self.ws = self._workspace(max(shard.k1 - shard.k0, 1))
        if transport not in ("nccl", "p2p"):
            raise ValueError(f"transport {transport!r}: 'nccl' or 'p2p'")
        self.transport = transport
        self.peer = peer_exchange
        if transport == "p2p" and self.peer is None:
            self.peer = PeerExchange.connect(shard.rank, shard.world, blk, device, process_group)
        if self.peer is not None and self.peer.slot_floats != blk:
            raise ValueError("peer exchange slot size differs from the packed partial")

    def q_slice(self, q: torch.Tensor) -> torch.Tensor:
        """This rank's q heads of a full q [B, Hq, D]."""
        h0 = self.shard.kv_head0 * self.G
        return q[:, h0:h0 + self.hq].contiguous()

    def _workspace(self, max_seqlen_k: int) -> torch.Tensor:
        n = self.pool.workspace_size(self.hq, self.batch, 1, max_seqlen_k)
        return torch.empty(max(n, 16), dtype=torch.uint8, device=self.dev)

    def partial(self, q_local: torch.Tensor, cu_k, table, scale: float, max_seqlen_k: int):
        if self.pool.workspace_size(self.hq, self.batch, 1, max_seqlen_k) > self.ws.numel():
            self.ws = self._workspace(max_seqlen_k)  # a longer range than the shard was built for
        pa.dispatch_flash_decode_partial(q_local, self.pool, 0, cu_k, table, scale, max_seqlen_k=max_seqlen_k,
                                         o_part=self.o_part, lse_part=self.lse_part, workspace=self.ws)

    @property
    def fused(self) -> bool:
        """The whole step is one yf_exchange_decode (p2p between ranks on separate GPUs)."""
        return self.transport == "p2p" and not self.peer.is_emulated

    def exchange(self):
        if self.transport == "p2p":
            self.peer.push(self.local)
        else:
            gather_packed(self.local, self.gathered, self.shard.world, self.group)

    def combine(self) -> torch.Tensor:
        if self.transport == "p2p":
            rows = self.batch * self.hq
            return self.peer.combine(self.out, self.shard.n_head_groups, self.shard.n_seq, rows, self.hq, self.Hq,
                                     self.D, rows * self.D)
        flat = self.out.view(self.batch * self.Hq, self.D)
        for g, (oo, lo, stride, n_parts, rows) in enumerate(combine_views(self.shard, self.batch, self.hq, self.D)):
            # one head group: its rows are contiguous in the output when B == 1 or there is one group
            dst = self._grp_out[g] if self._grp_out is not None else flat[g * rows:(g + 1) * rows]
            pa.combine_partials(self.gathered[oo:], self.gathered[lo:], out=dst, n_parts=n_parts, rows=rows,
                                head_dim=self.D, o_part_stride=stride, lse_part_stride=stride)
        if self._grp_out is not None:
            self.out.view(self.batch, self.shard.n_head_groups, self.hq, self.D).copy_(
                self._grp_out.view(self.shard.n_head_groups, self.batch, self.hq, self.D).transpose(0, 1))
        return self.out

    def step(self, q_local: torch.Tensor, cu_k, table, scale: float, max_seqlen_k: int) -> torch.Tensor:
        """Partial over this shard, exchange, combine: the full f16 output [B, Hq, D] on every rank
        (with the p2p transport between GPUs, one fused launch)."""
        if self.fused:
            if self.pool.workspace_size(self.hq, self.batch, 1, max_seqlen_k) > self.ws.numel():
                self.ws = self._workspace(max_seqlen_k)
            return self.peer.decode(self.pool, q_local, cu_k, table, scale, max_seqlen_k, self.shard.n_head_groups,
                                    self.shard.n_seq, self.Hq, self.out, self.ws)
        self.partial(q_local, cu_k, table, scale, max_seqlen_k)
        self.exchange()
        return self.combine()

