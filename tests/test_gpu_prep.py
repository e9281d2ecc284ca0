"""Fused attention prep + Q8_0 KV append on the GPU against the oracle: q, gate and the pool
bytes bit-exact."""
import numpy as np
import pytest
import torch

from helpers import pool_image
from qwen36_server_b200 import workloads as W

pytestmark = pytest.mark.gpu


def rope_tables(n_pos, rope_dim, theta=1e7):
    if rope_dim == 0:
        return None, None
    inv = theta ** (-np.arange(0, rope_dim, 2, dtype=np.float64) / rope_dim)
    ang = np.arange(n_pos, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def run_case(yf, oracle, cuda, Hq, H, D, rope_dim, offset, rows, starts, seed):
    rng = np.random.default_rng(seed)
    ctx = [s + r for s, r in zip(starts, rows)]
    wl = W.Workload("prep", Hq, H, D, ctx=ctx, q_rows=rows, seed=seed)
    T = int(sum(rows))
    qg = (rng.standard_normal((T, Hq, 2 * D)) * 2).astype(np.float16)
    k = (rng.standard_normal((T, H, D)) * 2).astype(np.float16)
    v = rng.standard_normal((T, H, D)).astype(np.float16)
    wq = (rng.standard_normal(D) * 0.2).astype(np.float32)
    wk = (rng.standard_normal(D) * 0.2).astype(np.float32)
    cos, sin = rope_tables(max(ctx) + 1, rope_dim)
    cu = np.concatenate([[0], np.cumsum(rows)]).astype(np.int32)
    start = np.asarray(starts, np.int32)
    pool = yf.PagedKvPool(1, wl.n_pages, H, D, device=0)
    t = lambda a: None if a is None else torch.from_numpy(a).to(cuda)  # noqa: E731
    q_out, gate_out = yf.attn_prepare_append(pool, 0, t(qg), t(k), t(v), t(wq), t(wk), 1e-6, t(cos), t(sin),
                                             rope_dim, cu, start, t(wl.block_table), norm_weight_offset=offset)
    entry = np.repeat(np.arange(len(rows)), rows).astype(np.int32)
    pos = np.concatenate([np.arange(s, s + r) for s, r in zip(starts, rows)]).astype(np.int32)
    rq, rg, rk = oracle.np_attn_prep(qg, k, wq, wk, 1e-6, offset, cos, sin, rope_dim, pos)
    assert np.array_equal(q_out.cpu().numpy().view(np.uint16), rq.view(np.uint16))
    assert np.array_equal(gate_out.cpu().numpy().view(np.uint16), rg.view(np.uint16))
    desc = oracle.PoolDesc(1, wl.n_pages, H, D)
    img = np.zeros(desc.pool_bytes, np.uint8)
    oracle.np_kv_write_rows(desc, img, 0, rk, v, entry, pos, wl.block_table)
    got = pool_image(pool)
    assert np.array_equal(got, img)
    assert pool.status() == 0
    return pool, wl, rk, v, cu, start, got


@pytest.mark.parametrize("Hq,H,D,rope_dim,offset", [(32, 8, 128, 32, 1), (16, 2, 256, 64, 1), (8, 2, 128, 0, 0),
                                                    (8, 2, 256, 256, 0)])
def test_prep_matches_oracle_bit_exact(yf, oracle, cuda, Hq, H, D, rope_dim, offset):
    pool, *_ = run_case(yf, oracle, cuda, Hq, H, D, rope_dim, offset, rows=[1, 5, 17], starts=[0, 33, 250], seed=170)
    pool.close()


def test_prep_equals_separate_append(yf, oracle, cuda):
    """The fused K/V bytes equal yf_kv_append_paged_multi of the prep's f16 K and the input V."""
    pool, wl, rk, v, cu, start, fused = run_case(yf, oracle, cuda, 32, 8, 128, 32, 1, rows=[3, 16],
                                                 starts=[5, 100], seed=171)
    pool.close()
    pool2 = yf.PagedKvPool(1, wl.n_pages, 8, 128, device=0)
    yf.launch_append_multi(pool2, 0, torch.from_numpy(rk).to(cuda), torch.from_numpy(v).to(cuda), cu, start,
                           torch.from_numpy(wl.block_table).to(cuda))
    assert np.array_equal(pool_image(pool2), fused)
    pool2.close()


def test_prep_bad_position_and_limits(yf, cuda):
    """A position past the rope table flags YF_DEV_BAD_POS and writes nothing for that row; an
    unsupported rope_dim is refused on the host."""
    wl = W.Workload("prep", 8, 2, 128, ctx=[20], q_rows=[2], seed=172)
    pool = yf.PagedKvPool(1, wl.n_pages, 2, 128, device=0)
    qg = torch.zeros((2, 8, 256), dtype=torch.float16, device=cuda)
    k = torch.zeros((2, 2, 128), dtype=torch.float16, device=cuda)
    w = torch.zeros(128, dtype=torch.float32, device=cuda)
    cos = torch.ones((10, 16), dtype=torch.float32, device=cuda)
    bt = torch.from_numpy(wl.block_table).to(cuda)
    yf.attn_prepare_append(pool, 0, qg, k, k, w, w, 1e-6, cos, cos, 32, [0, 2], [18], bt)
    assert pool.status() & yf._abi.YF_DEV_BAD_POS
    assert not pool_image(pool).any()
    with pytest.raises(yf.YfError):
        yf.attn_prepare_append(pool, 0, qg, k, k, w, w, 1e-6, cos, cos, 24, [0, 2], [0], bt)
    pool.close()
