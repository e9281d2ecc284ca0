"""Shared set-up for the GPU parity tests: a pool filled through the CUDA writer and the
oracle's image of the same pool."""
import numpy as np
import torch

from qwen36_server_b200 import workloads as W

TOL = 2e-3  # max |out - oracle| for attention outputs (f16 output, fp32 oracle over the dequantized cache)


def rows_of(wl):
    entry = np.repeat(np.arange(wl.batch), wl.ctx).astype(np.int32)
    pos = np.concatenate([np.arange(c) for c in wl.ctx]).astype(np.int32) if wl.batch else np.zeros(0, np.int32)
    return entry, pos


def filled_pool(yf, oracle, wl, seed=0, n_layers=1, layer=0, extra_pages=0, oracle_image=True):
    """Writes every key of every entry of ``wl`` into a new pool with launch_append_multi
    and returns (pool, oracle pool image or None, oracle desc, k, v)."""
    dev = torch.device("cuda", 0)
    n_pages = wl.n_pages + extra_pages
    pool = yf.PagedKvPool(n_layers, n_pages, wl.n_kv_heads, wl.head_dim, wl.page_size, wl.group_size, device=0)
    rng = np.random.default_rng(seed)
    n = int(wl.ctx.sum())
    k = W.kv_rows_np(rng, n, wl.n_kv_heads, wl.head_dim, wl.outlier_frac)
    v = W.kv_rows_np(rng, n, wl.n_kv_heads, wl.head_dim, wl.outlier_frac)
    yf.launch_append_multi(pool, layer, torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev), wl.cu_k,
                           np.zeros(wl.batch, np.int32), torch.from_numpy(wl.block_table).to(dev))
    desc = oracle.PoolDesc(n_layers, n_pages, wl.n_kv_heads, wl.head_dim, wl.page_size, wl.group_size)
    img = None
    if oracle_image:
        img = np.zeros(desc.pool_bytes, np.uint8)
        entry, pos = rows_of(wl)
        oracle.np_kv_write_rows(desc, img, layer, k, v, entry, pos, wl.block_table)
    return pool, img, desc, k, v


def pool_image(pool, n_layers=None):
    parts = [pool.layer_bytes_view(l).cpu().numpy() for l in range(n_layers or pool.n_layers)]
    return np.concatenate(parts)


def queries(wl, seed=1):
    rng = np.random.default_rng(seed)
    T = int(wl.q_rows.sum())
    return rng.standard_normal((T, wl.n_q_heads, wl.head_dim)).astype(np.float16)


def device_pool(yf, wl, seed=0, n_layers=1, layer=0, chunk_rows=1 << 18):
    """A pool holding every key of every entry of ``wl`` in ``layer``, the K/V rows drawn on the
    device (seeded N(0,1), with the workload's outliers) and written with launch_append_multi in
    bounded row chunks: the full-size workloads are too large to stage their f16 rows on the host."""
    dev = torch.device("cuda", 0)
    pool = yf.PagedKvPool(n_layers, wl.n_pages, wl.n_kv_heads, wl.head_dim, wl.page_size, wl.group_size, device=0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    bt = torch.from_numpy(wl.block_table).to(dev)
    for b in range(wl.batch):
        n = int(wl.ctx[b])
        for s in range(0, n, chunk_rows):
            m = min(chunk_rows, n - s)
            k = W.kv_rows_torch(gen, m, wl.n_kv_heads, wl.head_dim, wl.outlier_frac, dev)
            v = W.kv_rows_torch(gen, m, wl.n_kv_heads, wl.head_dim, wl.outlier_frac, dev)
            yf.launch_append_multi(pool, layer, k, v, [0, m], [s], bt[b:b + 1], max_rows=m)
    torch.cuda.synchronize()
    return pool


def gathered_image(oracle, pool, wl, entries, layer=0):
    """The pages of ``entries`` copied out of the device pool into a compact oracle image, with
    their block-table rows renumbered onto it: (desc, image, sub-workload of those entries)."""
    P = wl.page_size
    rows = [wl.block_table[b, :-(-int(wl.ctx[b]) // P)] for b in entries]
    pages = np.unique(np.concatenate(rows)) if rows else np.zeros(0, np.int32)
    where = {int(p): i for i, p in enumerate(pages.tolist())}
    width = max(len(r) for r in rows)
    table = np.zeros((len(entries), width), np.int32)
    for i, r in enumerate(rows):
        table[i, :len(r)] = [where[int(p)] for p in r.tolist()]
    view = pool.layer_bytes_view(layer).view(pool.n_pages, pool.page_bytes)
    img = view.index_select(0, torch.from_numpy(pages.astype(np.int64)).to(view.device)).cpu().numpy().reshape(-1)
    desc = oracle.PoolDesc(1, len(pages), wl.n_kv_heads, wl.head_dim, wl.page_size, wl.group_size)
    sub = W.Workload("sub", wl.n_q_heads, wl.n_kv_heads, wl.head_dim, ctx=wl.ctx[list(entries)],
                     q_rows=wl.q_rows[list(entries)], page_size=wl.page_size, group_size=wl.group_size,
                     block_table=table, n_pages=len(pages))
    return desc, img, sub
