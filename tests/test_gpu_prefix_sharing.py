"""Prefix restore by pointer: a second slot reuses the first slot's prefix pages through the
refcounted allocator instead of copying them (the reference's PageAllocator {free, refcount}
with retain/release, docs/plans/2026-08-27-tiered-kv-cache.md:313-323).  Both slots decode
against the oracle; freeing the first slot releases only its private pages, the shared prefix
stays with the second slot, and pages reused by a new writer leave the second slot's output
unchanged."""
import numpy as np
import pytest
import torch

from helpers import TOL, queries
from qwen36_server_b200 import workloads as W

pytestmark = pytest.mark.gpu


def test_shared_prefix_pages_by_retain(yf, oracle, cuda):
    P, H, D, Hq = 16, 8, 128, 32
    prefix, a_len, b_len = 288, 400, 350          # 18 whole prefix pages shared
    n_pages = 64
    pool = yf.PagedKvPool(1, n_pages, H, D, device=0)
    rng = np.random.default_rng(301)
    ka = W.kv_rows_np(rng, a_len, H, D)
    va = W.kv_rows_np(rng, a_len, H, D)
    kb = W.kv_rows_np(rng, b_len - prefix, H, D)
    vb = W.kv_rows_np(rng, b_len - prefix, H, D)

    a_pages = pool.alloc_pages(-(-a_len // P))
    shared = a_pages[:prefix // P]
    pool.retain_pages(shared)                      # slot B takes the prefix by reference
    b_own = pool.alloc_pages(-(-b_len // P) - len(shared))
    b_pages = shared + b_own
    assert all(pool.refcount(p) == 2 for p in shared)
    width = max(len(a_pages), len(b_pages))
    table = np.zeros((2, width), np.int32)
    table[0, :len(a_pages)] = a_pages
    table[1, :len(b_pages)] = b_pages
    bt = torch.from_numpy(table).to(cuda)
    # A writes all of its rows; B writes only the rows after the shared prefix
    yf.launch_append_multi(pool, 0, torch.from_numpy(ka).to(cuda), torch.from_numpy(va).to(cuda), [0, a_len], [0],
                           bt[0:1])
    yf.launch_append_multi(pool, 0, torch.from_numpy(kb).to(cuda), torch.from_numpy(vb).to(cuda),
                           [0, b_len - prefix], [prefix], bt[1:2])
    cu = np.array([0, a_len, a_len + b_len])
    wl = W.Workload("share", Hq, H, D, ctx=[a_len, b_len], q_rows=[1, 1], block_table=table, n_pages=n_pages)
    q = queries(wl, 302)
    qd = torch.from_numpy(q).to(cuda)
    scale = yf.default_scale(D)
    got = yf.dispatch_flash_decode_paged(qd, pool, 0, cu, bt, scale).float().cpu().numpy()
    assert pool.status() == 0
    # oracle: slot B's keys are A's first 288 rows followed by its own
    desc = oracle.PoolDesc(1, n_pages, H, D)
    img = np.zeros(desc.pool_bytes, np.uint8)
    oracle.c_kv_write_rows(desc, img, 0, np.concatenate([ka, kb]), np.concatenate([va, vb]),
                           np.r_[np.zeros(a_len, np.int32), np.ones(b_len - prefix, np.int32)],
                           np.r_[np.arange(a_len), np.arange(prefix, b_len)].astype(np.int32), table)
    assert np.array_equal(pool.layer_bytes_view(0).cpu().numpy(), img)
    ref = oracle.c_attn(desc, img, 0, q, np.arange(3), cu, table, scale)
    assert np.abs(got - ref).max() <= TOL
    before_b = yf.dispatch_flash_decode_paged(qd[1:2], pool, 0, [0, b_len], bt[1:2], scale).float().cpu().numpy()
    assert np.abs(before_b[0] - ref[1]).max() <= TOL

    # slot A finishes: its private pages return to the free list, the shared prefix stays
    free0 = pool.free_count()
    pool.free_pages(a_pages)
    assert pool.free_count() == free0 + len(a_pages) - len(shared)
    assert all(pool.refcount(p) == 1 for p in shared)
    # a new slot C takes the freed pages (A's private ones among them) and overwrites them
    c_pages = pool.alloc_pages(len(a_pages) - len(shared))
    assert set(c_pages) == set(a_pages[len(shared):])   # the free list hands A's pages out again
    c_len = len(c_pages) * P
    kc = W.kv_rows_np(rng, c_len, H, D) * 3
    vc = W.kv_rows_np(rng, c_len, H, D) * 3
    ct = torch.tensor([c_pages], dtype=torch.int32, device=cuda)
    yf.launch_append_multi(pool, 0, torch.from_numpy(kc.astype(np.float16)).to(cuda),
                           torch.from_numpy(vc.astype(np.float16)).to(cuda), [0, c_len], [0], ct)
    after = yf.dispatch_flash_decode_paged(qd[1:2], pool, 0, [0, b_len], bt[1:2], scale).float().cpu().numpy()
    assert pool.status() == 0
    assert np.array_equal(after, before_b)
    pool.free_pages(b_pages)
    pool.free_pages(c_pages)
    assert pool.free_count() == n_pages
    pool.close()
