"""Snapshot wire records (pages.kv) built and checked on the GPU against the oracle: the
reference's page entry { chain_hash, prev_hash, tokens[], payload } with a CRC-32C over the
token ids and the payload (docs/plans/2026-08-27-tiered-kv-cache.md:141-145,237-251)."""
import numpy as np
import pytest
import torch

from helpers import pool_image
from qwen36_server_b200 import _abi

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
    prev = [0, 0x0123456789ABCDEF, 1, 2 ** 63 - 5]
    idx = [10, 11, 12, 13]
    tokens = np.random.default_rng(181).integers(0, 151936, (4, P)).astype(np.int32)
    rec = pool.export_records(pages, hashes, idx, prev_hashes=prev, tokens=tokens).cpu().numpy()
    desc = oracle.PoolDesc(L, 9, H, D, P, 32)
    ref = oracle.page_records(desc, pool_image(pool), pages, hashes, idx, prev_hashes=prev, tokens=tokens)
    assert rec.size == len(pages) * pool.record_bytes == ref.size
    assert np.array_equal(rec, ref)
    # without hashes or tokens the fields are zeros and the page id stands in for the index
    rec0 = pool.export_records(pages).cpu().numpy()
    ref0 = oracle.page_records(desc, pool_image(pool), pages, [0] * 4, pages)
    assert np.array_equal(rec0, ref0)
    assert pool.status() == 0
    # a page id outside the pool: flagged, and its header says length 0
    bad = pool.export_records([1, 99]).cpu().numpy()
    assert pool.status() == _abi.YF_DEV_BAD_PAGE
    assert not bad[pool.record_bytes:pool.record_bytes + 32].any()
    pool.close()


def test_import_restores_intact_matching_records_only(yf, oracle, cuda):
    src = random_pool(yf, cuda, 2, 6, 8, 128, 16, seed=181)
    tok = np.arange(3 * 16, dtype=np.int32).reshape(3, 16)
    rec = src.export_records([5, 1, 2], [9, 9, 9], [0, 1, 2], tokens=tok)
    dst = random_pool(yf, cuda, 2, 6, 8, 128, 16, seed=182)
    before = pool_image(dst)
    rb = src.record_bytes
    hdr = 32 + 4 * 16
    bad = rec.clone()
    bad[rb + hdr + 777] ^= 0x01          # one payload bit of record 1
    bad[2 * rb + 24] ^= 0x10             # record 2's payload_len
    ok = dst.import_records([0, 3, 4], bad).cpu().numpy()
    assert ok.tolist() == [_abi.YF_REC_RESTORED, _abi.YF_REC_REJECTED, _abi.YF_REC_REJECTED]
    got, s_img = pool_image(dst), pool_image(src)
    pb = dst.page_bytes
    lb = 6 * pb
    for layer in range(2):
        assert np.array_equal(got[layer * lb:layer * lb + pb], s_img[layer * lb + 5 * pb:layer * lb + 6 * pb])
        for p in (1, 2, 3, 4, 5):       # rejected records and other pages untouched
            sl = slice(layer * lb + p * pb, layer * lb + (p + 1) * pb)
            assert np.array_equal(got[sl], before[sl])
    # a flipped token id breaks the CRC too
    bad2 = rec.clone()
    bad2[32 + 4 * 3] ^= 0x01
    assert dst.import_records([3], bad2).cpu().numpy().tolist() == [_abi.YF_REC_REJECTED]
    # intact records of another prefix (a chain-hash collision): not restored
    other = tok.copy()
    other[1, 7] += 1
    ok = dst.import_records([3, 4], rec[rb:], expect_hashes=[9, 9], expect_tokens=other[1:]).cpu().numpy()
    assert ok.tolist() == [_abi.YF_REC_MISMATCH, _abi.YF_REC_RESTORED]
    ok = dst.import_records([3], rec[rb:], expect_hashes=[8]).cpu().numpy()
    assert ok.tolist() == [_abi.YF_REC_MISMATCH]
    got = pool_image(dst)
    for layer in range(2):
        sl3 = slice(layer * lb + 3 * pb, layer * lb + 4 * pb)
        assert np.array_equal(got[sl3], before[sl3])
        assert np.array_equal(got[layer * lb + 4 * pb:layer * lb + 5 * pb],
                              s_img[layer * lb + 2 * pb:layer * lb + 3 * pb])
    ok = dst.import_records([3], rec[rb:], expect_hashes=[9], expect_tokens=tok[1:2]).cpu().numpy()
    assert ok.tolist() == [_abi.YF_REC_RESTORED]
    assert dst.status() == 0
    src.close()
    dst.close()
