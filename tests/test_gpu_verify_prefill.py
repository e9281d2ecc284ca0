"""MTP verify and causal chunked prefill on the GPU against the oracle, and the prefix
snapshot export/restore round trip."""
import numpy as np
import pytest
import torch

from helpers import TOL, filled_pool, queries
from qwen36_server_b200 import workloads as W

pytestmark = pytest.mark.gpu


def run_prefill(yf, pool, wl, q, cuda, layer=0):
    return yf.forward_attn_prefill_paged(torch.from_numpy(q).to(cuda), pool, layer, wl.cu_q, wl.cu_k,
                                         torch.from_numpy(wl.block_table).to(cuda),
                                         yf.default_scale(wl.head_dim)).float().cpu().numpy()


def test_mtp_verify_four_drafts(yf, oracle, cuda):
    """8 slots x 4 draft rows (16 query rows per kv head), row j sees ctx - 4 + j + 1 keys."""
    rng = np.random.default_rng(81)
    ctx = rng.integers(5, 3000, size=8)
    wl = W.Workload("v", 32, 8, 128, ctx=ctx, q_rows=[4] * 8, seed=82)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=83)
    q = queries(wl, 84)
    got = yf.forward_verify_paged(torch.from_numpy(q).to(cuda), pool, 0, wl.cu_q, wl.cu_k,
                                  torch.from_numpy(wl.block_table).to(cuda), yf.default_scale(128))
    ref = oracle.c_attn(desc, img, 0, q, wl.cu_q, wl.cu_k, wl.block_table, yf.default_scale(128))
    assert np.abs(got.float().cpu().numpy() - ref).max() <= TOL
    assert pool.status() == 0
    pool.close()


def test_verify_head_dim_256(yf, oracle, cuda):
    """Long-context shape (Hq 16 x D 256, Hkv 2) with 2 draft rows: 16 rows per kv head in two row groups."""
    wl = W.Workload("v", 16, 2, 256, ctx=[700, 33], q_rows=[2, 2], seed=85)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=86)
    q = queries(wl, 87)
    got = run_prefill(yf, pool, wl, q, cuda)
    ref = oracle.c_attn(desc, img, 0, q, wl.cu_q, wl.cu_k, wl.block_table, yf.default_scale(256))
    assert np.abs(got - ref).max() <= TOL
    pool.close()


@pytest.mark.parametrize("P,G", [(16, 32), (64, 128)])
def test_chunked_prefill_with_prefix(yf, oracle, cuda, P, G):
    """Ragged chunks over restored prefixes: (prefix 100, chunk 40), (0, 17), (37, 1)."""
    wl = W.Workload("p", 8, 2, 128, ctx=[140, 17, 38], q_rows=[40, 17, 1], page_size=P, group_size=G, seed=88)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=89)
    q = queries(wl, 90)
    got = run_prefill(yf, pool, wl, q, cuda)
    ref = oracle.c_attn(desc, img, 0, q, wl.cu_q, wl.cu_k, wl.block_table, yf.default_scale(128))
    assert np.abs(got - ref).max() <= TOL
    assert pool.status() == 0
    pool.close()


def test_snapshot_export_restore_roundtrip(yf, oracle, cuda):
    """Pages exported to pinned host memory and restored into freshly allocated pages give the
    same bytes and the same attention output (no requantization)."""
    wl = W.Workload("s", 8, 2, 128, ctx=[200], q_rows=[1], seed=91, extra_pages=20)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=92, n_layers=2, layer=1)
    q = queries(wl, 93)
    before = yf.dispatch_flash_decode_paged(torch.from_numpy(q).to(cuda), pool, 1, wl.cu_k,
                                            torch.from_numpy(wl.block_table).to(cuda), 0.1)
    pages = wl.block_table[0, :13].tolist()
    snap = pool.export_pages(1, pages)
    torch.cuda.synchronize()
    used = set(pages)
    fresh = [p for p in range(pool.n_pages) if p not in used][:13]
    pool.restore_pages(1, fresh, snap)
    table2 = wl.block_table.copy()
    table2[0, :13] = fresh
    after = yf.dispatch_flash_decode_paged(torch.from_numpy(q).to(cuda), pool, 1, wl.cu_k,
                                           torch.from_numpy(table2).to(cuda), 0.1)
    torch.cuda.synchronize()
    assert torch.equal(before, after)
    full = pool.layer_bytes_view(1).cpu().numpy().reshape(pool.n_pages, -1)
    assert np.array_equal(full[fresh], full[pages])
    dsnap = snap.to(cuda)                    # a device-resident snapshot restores the same way
    pool.restore_pages(1, fresh[::-1], dsnap)
    torch.cuda.synchronize()
    full = pool.layer_bytes_view(1).cpu().numpy().reshape(pool.n_pages, -1)
    assert np.array_equal(full[fresh[::-1]], full[pages])
    pool.close()
