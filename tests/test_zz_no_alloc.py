"""yf_attn_decode_noalloc: decode attention for callers that cannot allocate device memory.

Engines whose device memory is planned once at start-up (weights plus the KV pool, handed out
by their own allocator) cannot hand the FFI layer a fresh workspace buffer, and a cudaMalloc of
their own would break that plan.  This entry point keeps the split-KV partials in a fixed array
built into the library instead.  The test calls it through the C ABI and checks it against the
ordinary workspace-taking yf_attn_decode, twice in a row (the shared array keeps the previous
call's contents), and checks that a call needing more than the built-in 16 MiB is refused.
"""
import ctypes

import numpy as np
import pytest
import torch

from helpers import TOL, filled_pool, queries
from qwen36_server_b200 import _abi
from qwen36_server_b200 import workloads as W

pytestmark = pytest.mark.gpu

SCRATCH_LIMIT = 16 << 20


def test_noalloc_decode_matches_workspace_decode(yf, oracle, cuda):
    L = yf.lib()
    rng = np.random.default_rng(101)
    ctx = rng.integers(1024, 12000, size=16)
    wl = W.Workload("na", 32, 8, 128, ctx=ctx, q_rows=np.ones(16), outlier_frac=0.01, seed=102)
    pool, _, _, _, _ = filled_pool(yf, oracle, wl, seed=103, oracle_image=False)
    q = torch.from_numpy(queries(wl, 104)).to(cuda)
    cu = torch.from_numpy(wl.cu_k).to(cuda)
    bt = torch.from_numpy(wl.block_table).to(cuda)
    max_k = int(wl.ctx.max())
    need = pool.workspace_size(32, wl.batch, 1, max_k)
    assert 0 < need <= SCRATCH_LIMIT          # the call really uses scratch, and it fits
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    ref = torch.empty_like(q)
    ws = torch.empty(need, dtype=torch.uint8, device=cuda)
    _abi.check(L.yf_attn_decode(pool.handle, 0, P(q), 32, P(cu), P(bt), wl.max_blocks, wl.batch, max_k,
                                ctypes.c_float(0.088), P(ref), P(ws), need, stream), "yf_attn_decode")
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        _abi.check(L.yf_attn_decode_noalloc(pool.handle, 0, P(q), 32, P(cu), P(bt), wl.max_blocks, wl.batch,
                                            max_k, ctypes.c_float(0.088), P(out), stream),
                   "yf_attn_decode_noalloc")
        torch.cuda.synchronize()
        assert torch.isfinite(out).all()
        assert (out.float() - ref.float()).abs().max().item() <= TOL
    assert pool.status() == 0
    pool.close()


def test_noalloc_decode_refuses_oversized_calls(yf, cuda):
    L = yf.lib()
    # 1100 slots (past the persistent schedule's batch limit) of up to 64K keys with 2 kv heads:
    # the chunked split plan needs about 36 MiB of partials
    pool = yf.PagedKvPool(1, 64, 2, 128, device=0)
    batch, max_k = 1100, 65536
    assert pool.workspace_size(32, batch, 1, max_k) > SCRATCH_LIMIT
    q = torch.zeros((batch, 32, 128), dtype=torch.float16, device=cuda)
    cu = torch.zeros(batch + 1, dtype=torch.int32, device=cuda)
    bt = torch.zeros((batch, max_k // 16), dtype=torch.int32, device=cuda)
    out = torch.empty_like(q)
    rc = L.yf_attn_decode_noalloc(pool.handle, 0, ctypes.c_void_p(q.data_ptr()), 32, ctypes.c_void_p(cu.data_ptr()),
                                  ctypes.c_void_p(bt.data_ptr()), max_k // 16, batch, max_k, ctypes.c_float(0.088),
                                  ctypes.c_void_p(out.data_ptr()), None)
    assert rc == _abi.YF_E_WORKSPACE
    assert b"scratch" in L.yf_last_error()
    pool.close()
