"""Snapshot wire records (pages.kv) built and checked on the GPU against the oracle."""
import numpy as np
import pytest
import torch

from helpers import pool_image

pytestmark = pytest.mark.gpu


def random_pool(yf, cuda, L, pages, H, D, P, seed):
    pool = yf.PagedKvPool(L, pages, H, D, P, 32, device=0)
    g = torch.Generator(device=cuda)
    g.manual_seed(seed)
    for layer in range(L):
        view = pool.layer_bytes_view(layer)
        view.copy_(torch.randint(0, 256, view.shape, generator=g, device=cuda, dtype=torch.uint8))
    return pool


@pytest.mark.parametrize("L,H,D,P", [(2, 8, 128, 16), (3, 2, 256, 64)])
def test_export_matches_oracle_records(yf, oracle, cuda, L, H, D, P):
    pool = random_pool(yf, cuda, L, 9, H, D, P, seed=180)
    pages = [7, 0, 3, 8]
    hashes = [0x0123456789ABCDEF, 1, 2 ** 63 - 5, 42]
    idx = [10, 11, 12, 13]
    rec = pool.export_records(pages, hashes, idx).cpu().numpy()
    desc = oracle.PoolDesc(L, 9, H, D, P, 32)
    ref = oracle.page_records(desc, pool_image(pool), pages, hashes, idx)
    assert rec.size == len(pages) * pool.record_bytes == ref.size
    assert np.array_equal(rec, ref)
    assert pool.status() == 0
    pool.close()


def test_import_restores_intact_records_only(yf, oracle, cuda):
    src = random_pool(yf, cuda, 2, 6, 8, 128, 16, seed=181)
    rec = src.export_records([5, 1, 2], [9, 9, 9], [0, 1, 2])
    dst = random_pool(yf, cuda, 2, 6, 8, 128, 16, seed=182)
    before = pool_image(dst)
    bad = rec.clone()
    rb = src.record_bytes
    bad[rb + 20 + 777] ^= 0x01          # one payload bit of record 1
    bad[2 * rb + 12] ^= 0x10            # record 2's payload_len
    ok = dst.import_records([0, 3, 4], bad).cpu().numpy()
    assert ok.tolist() == [1, 0, 0]
    got, s_img = pool_image(dst), pool_image(src)
    pb = dst.page_bytes
    lb = 6 * pb
    for layer in range(2):
        assert np.array_equal(got[layer * lb:layer * lb + pb], s_img[layer * lb + 5 * pb:layer * lb + 6 * pb])
        for p in (1, 2, 3, 4, 5):       # rejected records and other pages untouched
            sl = slice(layer * lb + p * pb, layer * lb + (p + 1) * pb)
            assert np.array_equal(got[sl], before[sl])
    ok = dst.import_records([3, 4], rec[rb:]).cpu().numpy()
    assert ok.tolist() == [1, 1]
    src.close()
    dst.close()
