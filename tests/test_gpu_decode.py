"""Batched paged decode on the GPU against the oracle (max |err| <= 2e-3)."""
import numpy as np
import pytest
import torch

from helpers import TOL, filled_pool, queries
from qwen36_server_b200 import _abi
from qwen36_server_b200 import workloads as W

pytestmark = pytest.mark.gpu


def run_decode(yf, pool, wl, q, cuda, **kw):
    return yf.dispatch_flash_decode_paged(torch.from_numpy(q).to(cuda), pool, kw.pop("layer", 0), wl.cu_k,
                                          torch.from_numpy(wl.block_table).to(cuda), kw.pop("scale", None)
                                          or yf.default_scale(wl.head_dim), **kw).float().cpu().numpy()


@pytest.mark.parametrize("G", [32, 256])
def test_probe_lengths_shuffled_pages(yf, oracle, cuda, G):
    """The reference probe's parity sweep (src/bin/decode_gqa_probe.rs:25-63): q [1,16,256],
    Hkv 2, 64-token pages in the probe's xorshift order, lengths 1..1025, scale 0.0625,
    tolerance 2e-3 -- here against the oracle, for Q8_0 groups and the engine's row scale."""
    lengths = [1, 15, 16, 17, 63, 64, 65, 127, 128, 129, 257, 1025]
    max_blocks = -(-max(lengths) // 64)
    pages = oracle.shuffled_pages(max_blocks + 7).astype(np.int32)
    wl_all = W.Workload("probe", 16, 2, 256, ctx=[max(lengths)], q_rows=[1], page_size=64, group_size=G,
                        block_table=pages[None, :max_blocks], n_pages=max_blocks + 7)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl_all, seed=21)
    q = np.random.default_rng(22).standard_normal((1, 16, 256)).astype(np.float16)
    for n in lengths:
        blocks = -(-n // 64)
        wl = W.Workload("probe", 16, 2, 256, ctx=[n], q_rows=[1], page_size=64, group_size=G,
                        block_table=pages[None, :blocks], n_pages=max_blocks + 7)
        got = run_decode(yf, pool, wl, q, cuda, scale=0.0625)
        ref = oracle.c_attn(desc, img, 0, q, np.array([0, 1]), wl.cu_k, wl.block_table, 0.0625)
        err = np.abs(got - ref).max()
        assert np.isfinite(got).all() and err <= TOL, (n, err)
    assert pool.status() == 0
    pool.close()


def test_decode_small_config(yf, oracle, cuda):
    wl = W.decode_small()
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=31)
    q = queries(wl, 32)
    got = run_decode(yf, pool, wl, q, cuda)
    ref = oracle.c_attn(desc, img, 0, q, wl.cu_q, wl.cu_k, wl.block_table, yf.default_scale(128))
    assert np.abs(got - ref).max() <= TOL
    pool.close()


def test_decode_batch_ragged_with_outliers(yf, oracle, cuda):
    """16 slots of ragged length (1%-outlier K/V), fragmented tables, many split-KV chunks."""
    rng = np.random.default_rng(41)
    ctx = rng.integers(1, 6000, size=16)
    ctx[3], ctx[7] = 1, 16
    wl = W.Workload("b", 32, 8, 128, ctx=ctx, q_rows=np.ones(16), outlier_frac=0.01, seed=42)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=43)
    q = queries(wl, 44)
    ref = oracle.c_attn(desc, img, 0, q, wl.cu_q, wl.cu_k, wl.block_table, yf.default_scale(128))
    got = run_decode(yf, pool, wl, q, cuda)
    assert np.abs(got - ref).max() <= TOL
    # the schedule must not change the result beyond rounding: persistent with 3 copy stages;
    # chunked with 8-tile chunks merged by the last CTA or by the separate combine kernel; one chunk
    chunked = {"schedule": _abi.YF_SCHED_CHUNKED}
    for opts in ({"copy_stages": 3}, {**chunked, "chunk_tiles": 8},
                 {**chunked, "chunk_tiles": 8, "merge": _abi.YF_MERGE_SEPARATE},
                 {**chunked, "chunk_tiles": 24, "copy_stages": 3}, {**chunked, "chunk_tiles": 100000}):
        pool.set_options(**opts)
        try:
            alt = run_decode(yf, pool, wl, q, cuda)
            alt2 = run_decode(yf, pool, wl, q, cuda)   # counters reset between calls
        finally:
            pool.set_options(schedule=0, chunk_tiles=0, copy_stages=0, merge=0)
        assert np.abs(alt - ref).max() <= TOL, opts
        assert np.array_equal(alt, alt2), opts
    assert pool.status() == 0
    pool.close()


def test_decode_batch_full_size_sampled(yf, oracle, cuda):
    """The full 16-slot ctx U[1024, 32768] workload on the GPU; the oracle checks three slots
    (shortest, longest and one more) through a sub-batch of their table rows."""
    wl = W.decode_batch()
    pool, _, desc, k, v = filled_pool(yf, oracle, wl, seed=51, oracle_image=False)
    q = queries(wl, 52)
    got = run_decode(yf, pool, wl, q, cuda)
    assert np.isfinite(got).all()
    img = pool.layer_bytes_view(0).cpu().numpy()
    pick = sorted({int(np.argmin(wl.ctx)), int(np.argmax(wl.ctx)), 5})
    sub = W.Workload("s", 32, 8, 128, ctx=wl.ctx[pick], q_rows=np.ones(len(pick)),
                     block_table=wl.block_table[pick], n_pages=wl.n_pages)
    ref = oracle.c_attn(desc, img, 0, q[pick], sub.cu_q, sub.cu_k, sub.block_table, yf.default_scale(128))
    assert np.abs(got[pick] - ref).max() <= TOL
    pool.close()


def test_zero_length_and_bad_pages(yf, oracle, cuda):
    wl = W.Workload("z", 8, 2, 128, ctx=[0, 5, 40], q_rows=[1, 1, 1], seed=61)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=62)
    q = queries(wl, 63)
    got = run_decode(yf, pool, wl, q, cuda)
    assert not got[0].any()                                  # no keys -> zeros
    ref = oracle.c_attn(desc, img, 0, q, wl.cu_q, wl.cu_k, wl.block_table, yf.default_scale(128))
    assert np.abs(got - ref).max() <= TOL
    assert pool.status() == 0
    # a generous max_seqlen_k sizes the persistent grid for far more tiles than exist: the
    # partition shrinks to the real tile count
    wide = np.zeros((wl.batch, 256), np.int32)
    wide[:, :wl.max_blocks] = wl.block_table
    wl_wide = W.Workload("z", 8, 2, 128, ctx=[0, 5, 40], q_rows=[1, 1, 1], block_table=wide, n_pages=wl.n_pages)
    got = run_decode(yf, pool, wl_wide, q, cuda, max_seqlen_k=4096)
    assert np.abs(got - ref).max() <= TOL and not got[0].any()
    bad = wl.block_table.copy()
    bad[2, 1] = 10_000                                       # a page id past the pool
    wl_bad = W.Workload("z", 8, 2, 128, ctx=[0, 5, 40], q_rows=[1, 1, 1], block_table=bad, n_pages=wl.n_pages)
    got = run_decode(yf, pool, wl_bad, q, cuda)
    assert pool.status() == _abi.YF_DEV_BAD_PAGE
    ref = oracle.c_attn(desc, img, 0, q, wl.cu_q, wl.cu_k, bad, yf.default_scale(128))   # oracle skips it too
    assert np.abs(got - ref).max() <= TOL
    pool.close()


def test_workspace_and_argument_errors(yf, oracle, cuda):
    wl = W.Workload("e", 32, 8, 128, ctx=[30000, 20000], q_rows=[1, 1], seed=71)
    pool = yf.PagedKvPool(1, wl.n_pages, 8, 128, device=0)
    q = torch.zeros((2, 32, 128), dtype=torch.float16, device=cuda)
    bt = torch.from_numpy(wl.block_table).to(cuda)
    need = pool.workspace_size(32, 2, 1, 30000)
    assert need > 0
    small = torch.empty(need - 16, dtype=torch.uint8, device=cuda)
    with pytest.raises(yf.YfError) as e:
        yf.dispatch_flash_decode_paged(q, pool, 0, wl.cu_k, bt, 0.1, workspace=small)
    assert e.value.code == _abi.YF_E_WORKSPACE
    with pytest.raises(yf.YfError) as e:
        yf.dispatch_flash_decode_paged(q[:, :30], pool, 0, wl.cu_k, bt, 0.1)
    assert e.value.code == _abi.YF_E_INVALID
    with pytest.raises(yf.YfError) as e:
        yf.dispatch_flash_decode_paged(q, pool, 0, wl.cu_k, bt, 0.1, max_seqlen_k=10 ** 6)
    assert e.value.code == _abi.YF_E_RANGE
    pool.close()


@pytest.mark.parametrize("schedule", [0, 2])
def test_long_context_split_merges(yf, oracle, cuda, schedule):
    """One slot, 2 kv heads, D 256 (the long-context decode shape) at 20000 keys: the default
    cluster schedule (clusters of 8 CTAs per kv head, merged through distributed shared memory,
    then per column slice by the last cluster) and the persistent schedule (each unit cut into
    ~100 pieces merged cooperatively) agree with the oracle, twice in a row."""
    wl = W.Workload("long", 16, 2, 256, ctx=[20000], q_rows=[1], seed=121)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=122)
    pool.set_options(schedule=schedule)
    q = queries(wl, 123)
    ref = oracle.c_attn(desc, img, 0, q, wl.cu_q, wl.cu_k, wl.block_table, yf.default_scale(256))
    for _ in range(2):
        got = run_decode(yf, pool, wl, q, cuda)
        assert np.abs(got - ref).max() <= TOL
    assert pool.status() == 0
    pool.close()


@pytest.mark.parametrize("ctx", [[1], [15, 16, 17], [0, 300, 5000, 1], [65, 1025, 40000, 7, 130, 2049, 0, 4096]])
def test_cluster_schedule_ragged_few_units(yf, oracle, cuda, ctx):
    """Few units of very different lengths (one to eight entries x 2 kv heads): one entry runs on
    the cluster schedule (one cluster per unit: output written by the cluster merge), several on
    the persistent schedule, which balances unequal lengths; zero-length entries give zeros."""
    n = len(ctx)
    wl = W.Workload("fu", 16, 2, 256, ctx=ctx, q_rows=np.ones(n), seed=124 + n)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=125)
    q = queries(wl, 126)
    ref = oracle.c_attn(desc, img, 0, q, wl.cu_q, wl.cu_k, wl.block_table, yf.default_scale(256))
    for _ in range(2):
        got = run_decode(yf, pool, wl, q, cuda)
        assert np.abs(got - ref).max() <= TOL, ctx
    for b in range(n):
        if ctx[b] == 0:
            assert not got[b].any()
    assert pool.status() == 0
    pool.close()
