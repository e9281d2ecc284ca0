"""Tree speculative verify (trie_ranges mask) on the GPU against the oracle."""
import numpy as np
import pytest
import torch

from helpers import TOL, filled_pool, queries
from qwen36_server_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _tries(oracle, wl, seed):
    rng = np.random.default_rng(seed)
    return np.concatenate([W.random_trie(rng, int(t)) for t in wl.q_rows]).astype(np.int32)


def _run(yf, pool, wl, q, ranges, cuda):
    return yf.forward_verify_tree_paged(torch.from_numpy(q).to(cuda), pool, 0, wl.cu_q, wl.cu_k,
                                        torch.from_numpy(wl.block_table).to(cuda), yf.default_scale(wl.head_dim),
                                        torch.from_numpy(ranges).to(cuda)).float().cpu().numpy()


@pytest.mark.parametrize("Hq,H,D", [(32, 8, 128), (16, 2, 256)])
def test_random_tries_match_oracle(yf, oracle, cuda, Hq, H, D):
    """Ragged entries with tries of 1 .. 64 draft nodes over prefixes of 0 .. 3000 keys."""
    q_rows = [1, 5, 8, 16, 33, 64]
    ctx = [q + c for q, c in zip(q_rows, [0, 17, 300, 1500, 3000, 64])]
    wl = W.Workload("tree", Hq, H, D, ctx=ctx, q_rows=q_rows, seed=140)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=141)
    q = queries(wl, 142)
    ranges = _tries(oracle, wl, 143)
    got = _run(yf, pool, wl, q, ranges, cuda)
    ref = oracle.np_attn_tree(desc, img, 0, q, wl.cu_q, wl.cu_k, wl.block_table, yf.default_scale(D), ranges)
    assert np.abs(got - ref).max() <= TOL
    assert pool.status() == 0
    pool.close()


def test_chain_trie_equals_causal_verify(yf, oracle, cuda):
    """Chain ranges give the causal MTP verify: same output as forward_verify_paged (which runs
    the persistent schedule) within rounding, and the oracle's causal rows."""
    rng = np.random.default_rng(150)
    wl = W.Workload("v", 32, 8, 128, ctx=rng.integers(5, 4000, size=8), q_rows=[4] * 8, seed=151)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=152)
    q = queries(wl, 153)
    chain = np.concatenate([[[j, 3] for j in range(4)]] * 8).astype(np.int32)
    got = _run(yf, pool, wl, q, chain, cuda)
    causal = yf.forward_verify_paged(torch.from_numpy(q).to(cuda), pool, 0, wl.cu_q, wl.cu_k,
                                     torch.from_numpy(wl.block_table).to(cuda),
                                     yf.default_scale(128)).float().cpu().numpy()
    ref = oracle.c_attn(desc, img, 0, q, wl.cu_q, wl.cu_k, wl.block_table, yf.default_scale(128))
    assert np.abs(got - causal).max() <= 1e-3
    assert np.abs(got - ref).max() <= TOL
    pool.close()


def test_bad_ranges_flag_and_limits(yf, oracle, cuda):
    """A range outside the entry's block is clamped and flags YF_DEV_BAD_ROWS; more than 64
    draft rows or a missing range array is refused on the host."""
    wl = W.Workload("tree", 8, 2, 128, ctx=[50], q_rows=[6], seed=160)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=161)
    q = queries(wl, 162)
    bad = np.array([[0, 9], [1, 5], [2, 2], [3, 5], [4, 5], [5, 5]], np.int32)   # end 9 > 5
    _run(yf, pool, wl, q, bad, cuda)
    assert pool.status() & yf._abi.YF_DEV_BAD_ROWS
    good = np.array([[0, 5], [1, 5], [2, 2], [3, 5], [4, 5], [5, 5]], np.int32)
    got = _run(yf, pool, wl, q, good, cuda)
    ref = oracle.np_attn_tree(desc, img, 0, q, wl.cu_q, wl.cu_k, wl.block_table, yf.default_scale(128), good)
    assert np.abs(got - ref).max() <= TOL and pool.status() == 0
    big = W.Workload("tree", 8, 2, 128, ctx=[80], q_rows=[65], seed=163)
    with pytest.raises(yf.YfError):
        yf.forward_verify_tree_paged(torch.zeros((65, 8, 128), dtype=torch.float16, device=cuda), pool, 0, big.cu_q,
                                     big.cu_k, torch.from_numpy(big.block_table[:, :1]).to(cuda), 0.088,
                                     torch.zeros((65, 2), dtype=torch.int32, device=cuda))
    L = yf.lib()
    assert L.yf_attn_verify_tree(pool.handle, 0, 1, 8, 1, 1, 1, 1, 1, 6, 50, 0.088, None, 1, None, 0, None) != 0
    pool.close()
