"""Bounded waits on the GPU: a merge that waits for parts that never arrive gives up after the
pool's wait limit, flags YF_DEV_TIMEOUT without faulting, and the pool is usable again once its
status is cleared.  The failure is planted on the host (an arrival counter preset so that the
count can never complete); no GPU fault, trap or endless wait is involved."""
import numpy as np
import pytest
import torch

from helpers import TOL, filled_pool, queries
from qwen36_server_b200 import _abi
from qwen36_server_b200 import workloads as W

pytestmark = pytest.mark.gpu


def test_merge_wait_times_out_and_pool_recovers(yf, oracle, cuda):
    # one long entry, two kv heads on the persistent schedule: each kv head's unit is split over
    # many CTAs, and the CTAs whose range ends inside it wait on its arrival counter (the default
    # cluster schedule for so few units never waits)
    wl = W.Workload("to", 16, 2, 256, ctx=[20000], q_rows=[1], seed=141)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=142)
    q = queries(wl, 143)
    ref = oracle.c_attn(desc, img, 0, q, wl.cu_q, wl.cu_k, wl.block_table, yf.default_scale(256))
    qd = torch.from_numpy(q).to(cuda)
    bt = torch.from_numpy(wl.block_table).to(cuda)
    scale = yf.default_scale(256)
    pool.set_options(wait_limit_us=20000, schedule=_abi.YF_SCHED_PERSISTENT)   # 20 ms instead of 1 s
    pool.plant_counter(0, 0xFFFF)          # unit (entry 0, kv head 0): the count never reaches its parts
    got = yf.dispatch_flash_decode_paged(qd, pool, 0, wl.cu_k, bt, scale).float().cpu().numpy()
    st = pool.status()                      # reads and clears; clearing a timeout resets the counters
    assert st & _abi.YF_DEV_TIMEOUT, st
    # kv head 1's unit was not disturbed
    assert np.abs(got[:, 8:] - ref[:, 8:]).max() <= TOL
    # the pool works again after the clear, twice in a row (counters back at zero between calls)
    for _ in range(2):
        got = yf.dispatch_flash_decode_paged(qd, pool, 0, wl.cu_k, bt, scale).float().cpu().numpy()
        assert pool.status() == 0
        assert np.abs(got - ref).max() <= TOL
    pool.close()


def test_copy_ring_wait_limit_is_a_pool_option(yf, oracle, cuda):
    """A short wait limit does not disturb a healthy call: copies complete well inside 2 ms."""
    wl = W.Workload("wl", 32, 8, 128, ctx=[3000, 50, 9000], q_rows=[1, 1, 1], seed=144)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=145)
    pool.set_options(wait_limit_us=2000)
    q = queries(wl, 146)
    got = yf.dispatch_flash_decode_paged(torch.from_numpy(q).to(cuda), pool, 0, wl.cu_k,
                                         torch.from_numpy(wl.block_table).to(cuda), yf.default_scale(128))
    ref = oracle.c_attn(desc, img, 0, q, wl.cu_q, wl.cu_k, wl.block_table, yf.default_scale(128))
    assert pool.status() == 0
    assert np.abs(got.float().cpu().numpy() - ref).max() <= TOL
    pool.close()
