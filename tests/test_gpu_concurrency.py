"""Two pools decoded at once from two host threads on two streams, with the persistent decode
launched plainly (the default) and cooperatively: each grid is one resident wave whose CTAs
only wait for one another, and the library's per-device launch caches are shared safely, so
every concurrent result equals the serial one and no wait gives up."""
import threading

import numpy as np
import pytest
import torch

from helpers import filled_pool, queries
from qwen36_server_b200 import workloads as W

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("launch", [0, 1])
def test_two_threads_two_streams_two_pools(yf, oracle, cuda, launch):
    wls = [W.Workload("c0", 32, 8, 128, ctx=np.random.default_rng(151).integers(500, 9000, 16),
                      q_rows=np.ones(16), seed=152),
           W.Workload("c1", 16, 2, 256, ctx=[30000], q_rows=[1], seed=153)]
    pools, qs, bts = [], [], []
    for i, wl in enumerate(wls):
        pool, _, _, _, _ = filled_pool(yf, oracle, wl, seed=160 + i, oracle_image=False)
        pool.set_options(launch=launch)
        pools.append(pool)
        qs.append(torch.from_numpy(queries(wl, 170 + i)).to(cuda))
        bts.append(torch.from_numpy(wl.block_table).to(cuda))

    def run(i):
        return yf.dispatch_flash_decode_paged(qs[i], pools[i], 0, wls[i].cu_k, bts[i],
                                              yf.default_scale(wls[i].head_dim))

    serial = [run(i).clone() for i in range(2)]
    torch.cuda.synchronize()
    results = [[], []]
    errors = []

    def worker(i):
        try:
            s = torch.cuda.Stream(cuda)
            with torch.cuda.stream(s):
                for _ in range(30):
                    results[i].append(run(i).clone())
            s.synchronize()
        except Exception as e:   # surfaced below
            errors.append(e)

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(2)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    torch.cuda.synchronize()
    for i in range(2):
        assert pools[i].status() == 0
        assert len(results[i]) == 30
        for r in results[i]:
            assert torch.equal(r, serial[i])
        pools[i].close()
