"""Causal chunked prefill on the tcgen05 tensor-core kernel against the oracle."""
import numpy as np
import pytest
import torch

from helpers import TOL, filled_pool, queries
from qwen36_server_b200 import _abi
from qwen36_server_b200 import workloads as W

pytestmark = pytest.mark.gpu


def run_prefill(yf, pool, wl, q, cuda, tc=True):
    pool.set_options(prefill_kernel=_abi.YF_PREFILL_AUTO if tc else _abi.YF_PREFILL_SPLITKV)
    try:
        out = yf.forward_attn_prefill_paged(torch.from_numpy(q).to(cuda), pool, 0, wl.cu_q, wl.cu_k,
                                            torch.from_numpy(wl.block_table).to(cuda), yf.default_scale(wl.head_dim))
        return out.float().cpu().numpy()
    finally:
        pool.set_options(prefill_kernel=_abi.YF_PREFILL_AUTO)


def test_prefill_tc_ragged(yf, oracle, cuda):
    """Ragged entries (prefix, chunk): (0, 300), (1000, 257), (64, 128), (5, 1) at Hq 32 x D 128,
    Hkv 8: full and partial 128-row blocks, causal diagonal tiles, a one-row chunk."""
    wl = W.Workload("pf", 32, 8, 128, ctx=[300, 1257, 192, 6], q_rows=[300, 257, 128, 1], seed=131)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=132)
    q = queries(wl, 133)
    got = run_prefill(yf, pool, wl, q, cuda)
    ref = oracle.c_attn(desc, img, 0, q, wl.cu_q, wl.cu_k, wl.block_table, yf.default_scale(128))
    assert np.isfinite(got).all()
    err = np.abs(got - ref).max()
    assert err <= TOL, err
    assert pool.status() == 0
    pool.close()


def test_prefill_chunk_config_full_size(yf, oracle, cuda):
    """The 4 x (8192 restored prefix + 2048-token chunk) workload: the tensor-core kernel agrees
    with the split-KV kernel on every row, and with the oracle on windows of rows (first, middle
    and last positions of each entry, each checked as a short causal block with its own key count)."""
    wl = W.prefill_chunk()
    pool, _, desc, _, _ = filled_pool(yf, oracle, wl, seed=141, oracle_image=False)
    q = queries(wl, 142)
    got = run_prefill(yf, pool, wl, q, cuda)
    alt = run_prefill(yf, pool, wl, q, cuda, tc=False)
    assert np.isfinite(got).all()
    assert np.abs(got - alt).max() <= TOL
    img = pool.layer_bytes_view(0).cpu().numpy()
    for b in range(wl.batch):
        q0, tq, tk = int(wl.cu_q[b]), int(wl.q_rows[b]), int(wl.ctx[b])
        for start in (0, 1001, tq - 4):
            n = 4
            rows = slice(q0 + start, q0 + start + n)
            sub_tk = tk - tq + start + n            # keys the last row of the window sees
            ref = oracle.c_attn(desc, img, 0, q[rows], np.array([0, n]), np.array([0, sub_tk]),
                                wl.block_table[b:b + 1], yf.default_scale(128))
            assert np.abs(got[rows] - ref).max() <= TOL, (b, start)
    assert pool.status() == 0
    pool.close()


@pytest.mark.parametrize("P", [16, 64])
def test_prefill_tc_row_scale(yf, oracle, cuda, P):
    """The pool format with one scale per row (group = head_dim, the reference's own int8 pool):
    the tensor-core kernel reads the 4160-byte tiles and their per-row scales.  Ragged entries as
    above, 16- and 64-token pages, against the oracle and the split-KV kernel."""
    wl = W.Workload("pfr", 32, 8, 128, ctx=[300, 1257, 192, 6, 3000], q_rows=[300, 257, 128, 1, 700],
                    group_size=128, page_size=P, seed=151)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=152)
    q = queries(wl, 153)
    got = run_prefill(yf, pool, wl, q, cuda)
    ref = oracle.c_attn(desc, img, 0, q, wl.cu_q, wl.cu_k, wl.block_table, yf.default_scale(128))
    assert np.isfinite(got).all()
    assert np.abs(got - ref).max() <= TOL
    alt = run_prefill(yf, pool, wl, q, cuda, tc=False)
    assert np.abs(got - alt).max() <= TOL
    assert pool.status() == 0
    pool.close()


@pytest.mark.parametrize("group,P", [(32, 16), (256, 16), (32, 64)])
def test_prefill_d256_against_oracle(yf, oracle, cuda, group, P):
    """Causal chunked prefill at D 256 (Hq 16, Hkv 2: decode_long's head shape) on the D=256
    tcgen05 kernel: ragged chunks over prefixes (full and partial 64-key tiles, a one-row chunk),
    32-dim scale groups and one scale per row, 16- and 64-token pages, against the oracle and
    against the split-KV kernel."""
    wl = W.Workload("pf256", 16, 2, 256, ctx=[300, 2257, 129, 1, 5000], q_rows=[300, 257, 128, 1, 1000],
                    group_size=group, page_size=P, seed=161)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=162)
    q = queries(wl, 163)
    got = run_prefill(yf, pool, wl, q, cuda)
    ref = oracle.c_attn(desc, img, 0, q, wl.cu_q, wl.cu_k, wl.block_table, yf.default_scale(256))
    assert np.isfinite(got).all()
    assert np.abs(got - ref).max() <= TOL
    alt = run_prefill(yf, pool, wl, q, cuda, tc=False)
    assert np.abs(got - alt).max() <= TOL
    again = run_prefill(yf, pool, wl, q, cuda)
    assert np.array_equal(got, again)
    assert pool.status() == 0
    pool.close()


def test_prefill_d256_full_size(yf, oracle, cuda):
    """The 4 x (8192 prefix + 2048 chunk) D=256 workload: the tensor-core kernel agrees with the
    split-KV kernel on every row and with the oracle on windows of rows."""
    wl = W.prefill_d256()
    pool, _, desc, _, _ = filled_pool(yf, oracle, wl, seed=171, oracle_image=False)
    q = queries(wl, 172)
    got = run_prefill(yf, pool, wl, q, cuda)
    alt = run_prefill(yf, pool, wl, q, cuda, tc=False)
    assert np.isfinite(got).all()
    assert np.abs(got - alt).max() <= TOL
    img = pool.layer_bytes_view(0).cpu().numpy()
    for b in range(wl.batch):
        q0, tq, tk = int(wl.cu_q[b]), int(wl.q_rows[b]), int(wl.ctx[b])
        for start in (0, 777, tq - 4):
            n = 4
            rows = slice(q0 + start, q0 + start + n)
            ref = oracle.c_attn(desc, img, 0, q[rows], np.array([0, n]), np.array([0, tk - tq + start + n]),
                                wl.block_table[b:b + 1], yf.default_scale(256))
            assert np.abs(got[rows] - ref).max() <= TOL, (b, start)
    assert pool.status() == 0
    pool.close()
