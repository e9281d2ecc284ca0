"""The tcgen05 verify kernel (keys as the MMA's M, N = 16 or 32 query rows per kv head; the pool
option YF_VERIFY_TCGEN05) against the oracle, and against the default split-KV verify kernel on
the same inputs."""
import numpy as np
import pytest
import torch

from helpers import TOL, filled_pool, queries
from qwen36_server_b200 import _abi
from qwen36_server_b200 import workloads as W

pytestmark = pytest.mark.gpu


def verify(yf, pool, wl, q, cuda, trie=None):
    qd = torch.from_numpy(q).to(cuda)
    bt = torch.from_numpy(wl.block_table).to(cuda)
    if trie is None:
        out = yf.forward_verify_paged(qd, pool, 0, wl.cu_q, wl.cu_k, bt, yf.default_scale(wl.head_dim))
    else:
        out = yf.forward_verify_tree_paged(qd, pool, 0, wl.cu_q, wl.cu_k, bt, yf.default_scale(wl.head_dim), trie)
    return out.float().cpu().numpy()


@pytest.mark.parametrize("drafts,P", [(4, 16), (8, 16), (2, 64), (3, 16)])
def test_verify_tc_ragged_lengths(yf, oracle, cuda, drafts, P):
    """Lengths around the 128-key tile edges and past one chunk of key tiles (8192+ keys), 16 or
    32 rows per kv head (2..8 drafts x 4 q heads), 16- and 64-token pages; twice in a row (the
    chunk merge's counters reset) and equal to the split-KV kernel within the tolerance."""
    ctx = np.array([drafts, 100, 127, 128, 129, 3000, 9000, 20001])
    wl = W.Workload("vt", 32, 8, 128, ctx=ctx, q_rows=[drafts] * len(ctx), page_size=P, seed=301 + drafts)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=302)
    pool.set_options(verify_kernel=_abi.YF_VERIFY_TCGEN05)
    q = queries(wl, 303)
    ref = oracle.c_attn(desc, img, 0, q, wl.cu_q, wl.cu_k, wl.block_table, yf.default_scale(128))
    got = verify(yf, pool, wl, q, cuda)
    assert np.isfinite(got).all()
    err = np.abs(got - ref).max()
    assert err <= TOL, err
    again = verify(yf, pool, wl, q, cuda)
    assert np.array_equal(got, again)
    pool.set_options(verify_kernel=_abi.YF_VERIFY_AUTO)
    alt = verify(yf, pool, wl, q, cuda)
    assert np.abs(alt - ref).max() <= TOL
    assert pool.status() == 0
    pool.close()


def test_verify_tc_bad_page_and_short_entries(yf, oracle, cuda):
    """A page id past the pool is skipped (its keys masked) and flagged; entries with no
    committed keys (every key a draft) attend causally among their drafts only."""
    wl = W.Workload("vb", 32, 8, 128, ctx=[4, 300, 1000], q_rows=[4, 4, 4], seed=311)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=312)
    pool.set_options(verify_kernel=_abi.YF_VERIFY_TCGEN05)
    q = queries(wl, 313)
    ref = oracle.c_attn(desc, img, 0, q, wl.cu_q, wl.cu_k, wl.block_table, yf.default_scale(128))
    assert np.abs(verify(yf, pool, wl, q, cuda) - ref).max() <= TOL
    assert pool.status() == 0
    bad = wl.block_table.copy()
    bad[2, 5] = 10 ** 6
    wl_bad = W.Workload("vb", 32, 8, 128, ctx=[4, 300, 1000], q_rows=[4, 4, 4], block_table=bad, n_pages=wl.n_pages)
    got = verify(yf, pool, wl_bad, q, cuda)
    assert pool.status() == _abi.YF_DEV_BAD_PAGE
    ref_bad = oracle.c_attn(desc, img, 0, q, wl.cu_q, wl.cu_k, bad, yf.default_scale(128))
    assert np.abs(got - ref_bad).max() <= TOL
    pool.close()


def test_verify_tc_tree(yf, oracle, cuda):
    """Tree verify of 8-node tries (32 rows per kv head) on the tensor-core kernel against the
    oracle's trie-masked attention; a chain equals causal verify."""
    rng = np.random.default_rng(321)
    ctx = np.array([8, 200, 5000, 12000])
    trie = np.concatenate([W.random_trie(rng, 8) for _ in ctx])
    wl = W.Workload("vtt", 32, 8, 128, ctx=ctx, q_rows=[8] * 4, seed=322, trie=trie)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=323)
    pool.set_options(verify_kernel=_abi.YF_VERIFY_TCGEN05)
    q = queries(wl, 324)
    got = verify(yf, pool, wl, q, cuda, trie=trie)
    ref = oracle.np_attn_tree(desc, img, 0, q, wl.cu_q, wl.cu_k, wl.block_table, yf.default_scale(128), trie)
    assert np.abs(got - ref).max() <= TOL
    chain = np.array([[j, 7] for j in range(8)] * 4, np.int32)
    got_chain = verify(yf, pool, wl, q, cuda, trie=chain)
    causal = verify(yf, pool, wl, q, cuda)
    assert np.abs(got_chain - causal).max() <= 1e-3
    assert pool.status() == 0
    pool.close()
