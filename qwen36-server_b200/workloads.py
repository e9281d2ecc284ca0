"""Seeded synthetic workloads with the shapes of the five benchmark configurations.

The reference measures on its own prompts (not in its tree); these seeded
stand-ins carry the configurations' shapes, length distributions and value
distributions: K/V ~ N(0,1) (optionally with a fraction of +-8-sigma outliers),
q ~ N(0,1), 16-token pages scattered over a shared pool by a seeded
permutation so that every slot's page table is fragmented.

  decode_small   1 slot, ctx 4096, Hq 32 x D 128, Hkv 8
  decode_batch   16 slots, ctx ~ U[1024, 32768], Hq 32 x D 128, Hkv 8, 1% outliers at 8 sigma
  decode_long    1 slot, ctx 131072, Hq 16 x D 256, Hkv 2
  prefill_chunk  4 entries x (8192 restored prefix + 2048-token chunk), Hq 32 x D 128, Hkv 8
  mtp_verify     64 slots x 4 draft rows, ctx ~ U[4096, 65536], Hq 32 x D 128, Hkv 8, 36 layers
  tree_verify    mtp_verify's shape with an 8-node draft trie per slot (tree speculative verify)

"ctx" counts every key the step attends to, the step's own new rows included.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np


@dataclass
class Workload:
    name: str
    n_q_heads: int
    n_kv_heads: int
    head_dim: int
    ctx: np.ndarray              # keys per entry after the step's rows are written
    q_rows: np.ndarray           # query rows per entry (1 for decode)
    page_size: int = 16
    group_size: int = 32
    n_layers: int = 1
    outlier_frac: float = 0.0
    seed: int = 0
    extra_pages: int = 0
    block_table: np.ndarray = field(default=None, repr=False)
    n_pages: int = 0
    trie: Optional[np.ndarray] = field(default=None, repr=False)  # int32 [total_q, 2] subtree ranges

    def __post_init__(self):
        self.ctx = np.asarray(self.ctx, np.int64)
        self.q_rows = np.asarray(self.q_rows, np.int64)
        if self.block_table is None:
            self.block_table, self.n_pages = fragmented_tables(self.ctx, self.page_size, self.seed,
                                                               self.extra_pages)

    @property
    def batch(self) -> int:
        return len(self.ctx)

    @property
    def max_blocks(self) -> int:
        return self.block_table.shape[1]

    @property
    def prefix(self) -> np.ndarray:
        """Keys already in the pool before the step writes its own rows."""
        return self.ctx - self.q_rows

    @property
    def cu_k(self) -> np.ndarray:
        return np.concatenate([[0], np.cumsum(self.ctx)]).astype(np.int32)

    @property
    def cu_q(self) -> np.ndarray:
        return np.concatenate([[0], np.cumsum(self.q_rows)]).astype(np.int32)

    @property
    def kv_bytes_per_token(self) -> int:
        """Q8_0 bytes of one token of K and V in one layer: 2 * Hkv * (D + 2 * D / group)."""
        return 2 * self.n_kv_heads * (self.head_dim + 2 * self.head_dim // self.group_size)

    def kv_bytes(self, layers: Optional[int] = None) -> int:
        """Algorithmic KV bytes one step reads (every key of every entry, once per layer)."""
        return int(self.ctx.sum()) * self.kv_bytes_per_token * (layers or self.n_layers)

    def attn_flops(self) -> float:
        """QK^T + PV flops: 4 * D * Hq per (query row, visible key) pair."""
        pairs = 0
        for tk, tq in zip(self.ctx.tolist(), self.q_rows.tolist()):
            pairs += tq * (tk - tq) + tq * (tq + 1) // 2
        return 4.0 * self.head_dim * self.n_q_heads * pairs * self.n_layers


def fragmented_tables(ctx: np.ndarray, page_size: int, seed: int, extra_pages: int = 0):
    """Block tables drawn from one shared pool sized for the sum of contexts: the pool's
    page ids are permuted with a seeded generator and dealt out to the slots in order,
    so consecutive positions of a slot land on unrelated pages."""
    pages = (np.asarray(ctx) + page_size - 1) // page_size
    n_pages = max(int(pages.sum()) + extra_pages, 1)
    perm = np.random.default_rng(seed ^ 0x5EED).permutation(n_pages).astype(np.int32)
    max_blocks = max(int(pages.max()) if len(pages) else 1, 1)
    table = np.zeros((len(ctx), max_blocks), np.int32)
    off = 0
    for b, n in enumerate(pages.tolist()):
        table[b, :n] = perm[off:off + n]
        off += n
    return table, n_pages


def random_trie(rng: np.random.Generator, n: int, max_children: int = 3) -> np.ndarray:
    """A seeded token trie of n draft nodes in depth-first order, as int32 [n, 2] inclusive
    subtree ranges (node 0 is the root; a chain is [[j, n-1]]).  Each new node hangs under a node
    of the previous node's root path, which keeps every subtree a contiguous index range."""
    parent = [-1]
    for j in range(1, n):
        path = [j - 1]
        while parent[path[-1]] >= 0:
            path.append(parent[path[-1]])
        kids = [p for p in path if sum(1 for x in parent if x == p) < max_children]
        parent.append(int(rng.choice(kids)) if kids else j - 1)
    end = list(range(n))
    for j in range(n - 1, 0, -1):
        end[parent[j]] = max(end[parent[j]], end[j])
    return np.array([[j, end[j]] for j in range(n)], np.int32)


def decode_small(seed: int = 1) -> Workload:
    return Workload("decode_small", 32, 8, 128, ctx=[4096], q_rows=[1], seed=seed)


def decode_batch(seed: int = 2, n_slots: int = 16) -> Workload:
    rng = np.random.default_rng(seed)
    ctx = rng.integers(1024, 32768, size=n_slots, endpoint=True)
    return Workload("decode_batch", 32, 8, 128, ctx=ctx, q_rows=np.ones(n_slots), outlier_frac=0.01, seed=seed)


def decode_long(seed: int = 3, ctx: int = 131072) -> Workload:
    return Workload("decode_long", 16, 2, 256, ctx=[ctx], q_rows=[1], seed=seed)


def prefill_chunk(seed: int = 4, batch: int = 4, prefix: int = 8192, chunk: int = 2048) -> Workload:
    return Workload("prefill_chunk", 32, 8, 128, ctx=[prefix + chunk] * batch, q_rows=[chunk] * batch, seed=seed)


def prefill_rowscale(seed: int = 4, batch: int = 4, prefix: int = 8192, chunk: int = 2048) -> Workload:
    """prefill_chunk's shape over the pool format with one scale per row (group = head_dim)."""
    return Workload("prefill_rowscale", 32, 8, 128, ctx=[prefix + chunk] * batch, q_rows=[chunk] * batch,
                    group_size=128, seed=seed)


def prefill_d256(seed: int = 4, batch: int = 4, prefix: int = 8192, chunk: int = 2048) -> Workload:
    """A chunked prefill at decode_long's head shape (Hq 16 x D 256, Hkv 2)."""
    return Workload("prefill_d256", 16, 2, 256, ctx=[prefix + chunk] * batch, q_rows=[chunk] * batch, seed=seed)


def mtp_verify(seed: int = 5, n_slots: int = 64, drafts: int = 4, n_layers: int = 36) -> Workload:
    rng = np.random.default_rng(seed)
    ctx = rng.integers(4096, 65536, size=n_slots, endpoint=True)
    return Workload("mtp_verify", 32, 8, 128, ctx=ctx, q_rows=[drafts] * n_slots, n_layers=n_layers, seed=seed)


def tree_verify(seed: int = 6, n_slots: int = 64, nodes: int = 8, n_layers: int = 36) -> Workload:
    rng = np.random.default_rng(seed)
    ctx = rng.integers(4096, 65536, size=n_slots, endpoint=True)
    trie = np.concatenate([random_trie(rng, nodes) for _ in range(n_slots)])
    return Workload("tree_verify", 32, 8, 128, ctx=ctx, q_rows=[nodes] * n_slots, n_layers=n_layers, seed=seed,
                    trie=trie)


def subset(wl: Workload, entries, seed: int) -> Workload:
    """The entries ``entries`` of ``wl`` (one GPU's share of its slots) as a workload of their own,
    with a fragmented table over a pool sized for just those entries."""
    idx = list(entries)
    trie = None
    if wl.trie is not None:
        starts = np.concatenate([[0], np.cumsum(wl.q_rows)])
        trie = np.concatenate([wl.trie[starts[b]:starts[b + 1]] for b in idx]) if idx else wl.trie[:0]
    return Workload(wl.name, wl.n_q_heads, wl.n_kv_heads, wl.head_dim, ctx=wl.ctx[idx], q_rows=wl.q_rows[idx],
                    page_size=wl.page_size, group_size=wl.group_size, n_layers=wl.n_layers,
                    outlier_frac=wl.outlier_frac, seed=seed, trie=trie)


CONFIGS = {
    "decode_small": decode_small,
    "decode_batch": decode_batch,
    "decode_long": decode_long,
    "prefill_chunk": prefill_chunk,
    "prefill_rowscale": prefill_rowscale,
    "prefill_d256": prefill_d256,
    "mtp_verify": mtp_verify,
    "tree_verify": tree_verify,
}


def kv_rows_np(rng: np.random.Generator, n_rows: int, n_kv_heads: int, head_dim: int,
               outlier_frac: float = 0.0) -> np.ndarray:
    """f16 [n_rows, Hkv, D] ~ N(0,1) with a fraction of entries replaced by +-8."""
    x = rng.standard_normal((n_rows, n_kv_heads, head_dim), dtype=np.float32)
    if outlier_frac > 0:
        m = rng.random(x.shape) < outlier_frac
        x[m] = 8.0 * np.where(rng.random(int(m.sum())) < 0.5, -1.0, 1.0)
    return x.astype(np.float16)


def kv_rows_torch(gen, n_rows: int, n_kv_heads: int, head_dim: int, outlier_frac: float, device):
    """Device-side twin of kv_rows_np for full-size pools (same distribution, torch's RNG)."""
    import torch

    x = torch.randn((n_rows, n_kv_heads, head_dim), generator=gen, device=device, dtype=torch.float32)
    if outlier_frac > 0:
        u = torch.rand(x.shape, generator=gen, device=device)
        s = torch.where(torch.rand(x.shape, generator=gen, device=device) < 0.5, -8.0, 8.0)
        x = torch.where(u < outlier_frac, s, x)
    return x.to(torch.float16)
