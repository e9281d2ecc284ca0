"""KV write (Q8_0 quantize-and-scatter) on the GPU: pool bytes bit-exact with the oracle."""
import os

import numpy as np
import pytest
import torch

from helpers import filled_pool, pool_image, rows_of
from qwen36_server_b200 import _abi
from qwen36_server_b200 import workloads as W

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.mark.parametrize("D,P,G", [(128, 16, 32), (256, 16, 32), (256, 64, 32), (256, 64, 256), (128, 64, 128)])
def test_multi_writer_bit_exact(yf, oracle, cuda, D, P, G):
    wl = W.Workload("w", 2 * 2, 2, D, ctx=[1, 15, 16, 17, 130, 300], q_rows=[1] * 6, page_size=P, group_size=G,
                    outlier_frac=0.01, seed=D + P + G)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=3, n_layers=2, layer=1, extra_pages=3)
    assert pool.status() == 0
    assert np.array_equal(pool_image(pool), img)
    pool.close()


@pytest.mark.parametrize("D,P,G", [(128, 16, 32), (256, 64, 256)])
def test_single_row_writer_and_offsets(yf, oracle, cuda, D, P, G):
    """Decode-style appends (one row per slot at arbitrary positions), on top of existing rows."""
    wl = W.Workload("w", 4, 4, D, ctx=[40, 70, 129], q_rows=[1] * 3, page_size=P, group_size=G, seed=9)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=5)
    rng = np.random.default_rng(6)
    bt = torch.from_numpy(wl.block_table).to(cuda)
    for step in range(3):
        pos = np.array([3 + step, 63 + step, 128 - step], np.int32)   # overwrite inside and across pages
        k = W.kv_rows_np(rng, 3, 4, D, 0.02)
        v = W.kv_rows_np(rng, 3, 4, D, 0.02)
        yf.kv_append_paged(pool, 0, torch.from_numpy(k).to(cuda), torch.from_numpy(v).to(cuda), pos, bt)
        oracle.np_kv_write_rows(desc, img, 0, k, v, np.arange(3), pos, wl.block_table)
    assert pool.status() == 0
    assert np.array_equal(pool_image(pool), img)
    pool.close()


def test_gpu_quantizer_matches_gguf_golden(yf, oracle, cuda):
    """The device quantizer against gguf-py's Q8_0 bytes directly: golden groups are packed
    four to a 128-dim K row and read back from the pool through the layout functions."""
    g = np.load(os.path.join(GOLDEN, "q8_0_gguf.npz"))
    x, d, qs = g["x"], g["d"], g["qs"]
    n = x.shape[0] // 4
    rows = x[: 4 * n].reshape(n, 1, 128)
    wl = W.Workload("g", 1, 1, 128, ctx=[n], q_rows=[1], seed=1)
    pool = yf.PagedKvPool(1, wl.n_pages, 1, 128, device=0)
    kt = torch.from_numpy(np.ascontiguousarray(rows)).to(cuda)
    yf.launch_append_multi(pool, 0, kt, kt, [0, n], [0], torch.from_numpy(wl.block_table).to(cuda))
    img = pool_image(pool)
    desc = oracle.PoolDesc(1, wl.n_pages, 1, 128)
    for kv in (0, 1):
        got_q = np.zeros((n, 128), np.int8)
        got_d = np.zeros((n, 4), np.uint16)
        koff, voff, ksoff, vsoff = oracle.layout_maps(desc)
        for r in range(n):
            base = oracle.np_tile_base(desc, 0, wl.block_table[0, r // 16:r // 16 + 1], np.zeros(1), np.array([r % 16]))[0]
            off = (voff if kv else koff)[r % 16]
            got_q[r] = oracle.from_excess128(img[base + off])
            so = (vsoff if kv else ksoff)[r % 16]
            got_d[r] = img[base + so] | (img[base + so + 1].astype(np.uint16) << 8)
        assert np.array_equal(got_q.reshape(-1, 32), qs[: 4 * n])
        assert np.array_equal(got_d.reshape(-1), d[: 4 * n].view(np.uint16))
    pool.close()


def test_out_of_range_rows_are_skipped_and_flagged(yf, oracle, cuda):
    pool = yf.PagedKvPool(1, 4, 2, 128, device=0)
    k = torch.ones((2, 2, 128), dtype=torch.float16, device=cuda)
    bt = torch.tensor([[0, 1], [2, 9]], dtype=torch.int32, device=cuda)   # page 9 does not exist
    yf.kv_append_paged(pool, 0, k, k, [32, 5], bt)                       # pos 32 is past the table
    assert pool.status() == _abi.YF_DEV_BAD_POS
    yf.kv_append_paged(pool, 0, k, k, [0, 20], bt)                       # entry 1 -> page 9
    st = pool.status()
    assert st == _abi.YF_DEV_BAD_PAGE
    img = pool_image(pool)
    desc = oracle.PoolDesc(1, 4, 2, 128)
    ref = np.zeros(desc.pool_bytes, np.uint8)
    ones = np.ones((2, 2, 128), np.float16)
    # the valid rows: entry 1 at position 5 (first call) and entry 0 at position 0 (second call)
    oracle.np_kv_write_rows(desc, ref, 0, ones, ones, [1, 0], [5, 0], np.array([[0, 1], [2, 9]]))
    assert np.array_equal(img, ref)
    with pytest.raises(yf.YfError) as e:
        yf.kv_append_paged(pool, 3, k, k, [0, 0], bt)
    assert e.value.code == _abi.YF_E_RANGE
    pool.close()


@pytest.mark.parametrize("D,P,G", [(128, 16, 32), (256, 64, 32), (128, 64, 128)])
def test_tile_writer_mid_tile_chunks_keep_earlier_rows(yf, oracle, cuda, D, P, G):
    """Chunks of >= 16 rows (the staged tile writer) starting mid-tile on top of existing rows:
    the partly covered tiles keep their other tokens; then a chunk that runs past the table, one on
    a bad page and one longer than max_rows are skipped or clamped and flagged."""
    H = 3
    wl = W.Workload("t", H, H, D, ctx=[300, 200], q_rows=[1, 1], page_size=P, group_size=G, seed=17,
                    outlier_frac=0.02)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=18)
    bt = torch.from_numpy(wl.block_table).to(cuda)
    rng = np.random.default_rng(19)
    # entry 0: 40 rows at 37; entry 1: 23 rows at 100
    cu, start = [0, 40, 63], [37, 100]
    k = W.kv_rows_np(rng, 63, H, D, 0.02)
    v = W.kv_rows_np(rng, 63, H, D, 0.02)
    yf.launch_append_multi(pool, 0, torch.from_numpy(k).to(cuda), torch.from_numpy(v).to(cuda), cu, start, bt)
    assert pool.status() == 0
    oracle.np_kv_write_rows(desc, img, 0, k, v, np.r_[np.zeros(40), np.ones(23)].astype(np.int32),
                            np.r_[np.arange(37, 77), np.arange(100, 123)].astype(np.int32), wl.block_table)
    assert np.array_equal(pool_image(pool), img)
    # past the end of entry 1's table: rows from its capacity on are skipped (BAD_POS)
    cap = wl.max_blocks * P
    k2 = W.kv_rows_np(rng, 40, H, D)
    yf.launch_append_multi(pool, 0, torch.from_numpy(k2).to(cuda), torch.from_numpy(k2).to(cuda), [0, 0, 40],
                           [0, cap - 8], bt)
    assert pool.status() & _abi.YF_DEV_BAD_POS
    oracle.np_kv_write_rows(desc, img, 0, k2[:8], k2[:8], np.ones(8, np.int32), np.arange(cap - 8, cap).astype(np.int32),
                            wl.block_table)
    assert np.array_equal(pool_image(pool), img)
    # a bad page id in the table: that tile is skipped (BAD_PAGE), the others are written
    bad = wl.block_table.copy()
    bad[0, 1] = 10 ** 6
    k3 = W.kv_rows_np(rng, 3 * P, H, D)
    yf.launch_append_multi(pool, 0, torch.from_numpy(k3).to(cuda), torch.from_numpy(k3).to(cuda), [0, 3 * P, 3 * P],
                           [0, 0], torch.from_numpy(bad).to(cuda))
    assert pool.status() == _abi.YF_DEV_BAD_PAGE
    keep = np.r_[np.arange(0, P), np.arange(2 * P, 3 * P)]
    oracle.np_kv_write_rows(desc, img, 0, k3[keep], k3[keep], np.zeros(len(keep), np.int32), keep.astype(np.int32),
                            wl.block_table)
    assert np.array_equal(pool_image(pool), img)
    # more rows than max_rows: clamped to max_rows and flagged
    k4 = W.kv_rows_np(rng, 50, H, D)
    yf.launch_append_multi(pool, 0, torch.from_numpy(k4).to(cuda), torch.from_numpy(k4).to(cuda), [0, 50, 50], [5, 0],
                           bt, max_rows=32)
    assert pool.status() == _abi.YF_DEV_BAD_ROWS
    oracle.np_kv_write_rows(desc, img, 0, k4[:32], k4[:32], np.zeros(32, np.int32), np.arange(5, 37).astype(np.int32),
                            wl.block_table)
    assert np.array_equal(pool_image(pool), img)
    pool.close()
