"""The NVLink partial exchange (yf_exchange_push / yf_exchange_combine) with ranks emulated on one
GPU: every rank's exchange area is attached to the others, every rank pushes, then every rank
combines (no kernel waits on another launch).  The result must equal the all-gather + combine
path and the oracle, over several steps (the two buffers alternate), and a flag that nobody
raises must end the combine's wait with YF_DEV_TIMEOUT and no output written."""
import numpy as np
import pytest
import torch

from helpers import TOL
from qwen36_server_b200 import _abi
from qwen36_server_b200 import sharding as S

pytestmark = pytest.mark.gpu


def packed_parts(rng, world, batch, hq, D, empty_rows=()):
    """Random packed partials [world][packed_floats] with a few -inf lse rows."""
    blk = S.packed_floats(batch, hq, D)
    rows = batch * hq
    buf = np.zeros((world, blk), np.float32)
    o = rng.standard_normal((world, rows, D)).astype(np.float32)
    lse = (rng.standard_normal((world, rows)) * 3).astype(np.float32)
    for r, i in empty_rows:
        lse[r, i] = -np.inf
    buf[:, :rows * D] = o.reshape(world, -1)
    buf[:, rows * D:rows * D + rows] = lse
    return buf, o, lse


def expected(oracle, o, lse, n_hg, n_seq, batch, hq, D):
    """Output [batch, n_hg * hq, D]: head group g merges ranks s * n_hg + g."""
    out = np.zeros((batch, n_hg * hq, D), np.float32)
    for g in range(n_hg):
        ids = [s * n_hg + g for s in range(n_seq)]
        m = oracle.np_combine(o[ids], lse[ids]).reshape(batch, hq, D)
        out[:, g * hq:(g + 1) * hq] = m
    return out


@pytest.mark.parametrize("n_hg,n_seq,batch,hq,D", [(1, 1, 1, 8, 256), (2, 1, 1, 8, 256), (2, 2, 3, 8, 256),
                                                   (1, 4, 1, 8, 256), (2, 4, 2, 4, 128), (4, 2, 1, 16, 64)])
def test_exchange_matches_oracle(yf, oracle, cuda, n_hg, n_seq, batch, hq, D):
    world = n_hg * n_seq
    rows = batch * hq
    blk = S.packed_floats(batch, hq, D)
    xs = S.PeerExchange.emulated(world, blk, device=0)
    rng = np.random.default_rng(1000 + world * 10 + batch)
    outs = [torch.full((batch, n_hg * hq, D), float("nan"), dtype=torch.float16, device=cuda) for _ in range(world)]
    for step in range(3):  # buffers 1, 0, 1: a stale buffer would show
        buf, o, lse = packed_parts(rng, world, batch, hq, D, empty_rows=[(0, 0), (world - 1, rows - 1)])
        if step == 2:
            lse[:, 1] = -np.inf  # a row no rank has keys for: zeros
            buf[:, rows * D + 1] = -np.inf
        local = torch.from_numpy(buf).to(cuda)
        for r in range(world):
            xs[r].push(local[r])
        for r in range(world):
            xs[r].combine(outs[r], n_hg, n_seq, rows, hq, n_hg * hq, D, rows * D)
        ref = expected(oracle, o, lse, n_hg, n_seq, batch, hq, D)
        for r in range(world):
            got = outs[r].float().cpu().numpy()
            assert np.isfinite(got).all(), (step, r)
            assert np.abs(got - ref).max() <= TOL, (step, r)
        # the all-gather path on the same partials gives the same bits
        if n_hg == 1 or batch == 1:
            g = local.view(-1)
            for gi, (oo, lo, stride, n_parts, rws) in enumerate(
                    S.combine_views(S.long_context_plan(world, n_hg, 64 * world)[0], batch, hq, D)):
                alt = yf.combine_partials(g[oo:], g[lo:], n_parts=n_parts, rows=rws, head_dim=D, o_part_stride=stride,
                                          lse_part_stride=stride).float().cpu().numpy()
                want = outs[0].float().cpu().numpy().reshape(batch, n_hg, hq, D)[:, gi].reshape(rws, D)
                assert np.array_equal(alt, want), (step, gi)
    for x in xs:
        assert x.status() == 0
        x.close()


def test_exchange_wait_times_out_and_recovers(yf, cuda):
    """Rank 1 never pushes: rank 0's combine gives up after its 20 ms limit, flags
    YF_DEV_TIMEOUT and leaves the output untouched; once rank 1 pushes, the same step combines."""
    world, batch, hq, D = 2, 1, 8, 128
    rows, blk = batch * hq, S.packed_floats(batch, hq, D)
    xs = S.PeerExchange.emulated(world, blk, device=0, wait_limit_us=20000)
    rng = np.random.default_rng(77)
    buf, _, _ = packed_parts(rng, world, batch, hq, D)
    local = torch.from_numpy(buf).to(cuda)
    out = torch.full((batch, 2 * hq, D), 7.0, dtype=torch.float16, device=cuda)
    xs[0].push(local[0])
    xs[0].combine(out, 2, 1, rows, hq, 2 * hq, D, rows * D)
    assert xs[0].status(clear=True) == _abi.YF_DEV_TIMEOUT
    assert (out == 7.0).all()
    assert xs[0].status() == 0
    xs[1].push(local[1])
    xs[0].combine(out, 2, 1, rows, hq, 2 * hq, D, rows * D)
    xs[1].combine(out, 2, 1, rows, hq, 2 * hq, D, rows * D)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all() and not (out == 7.0).all()
    assert xs[0].status() == 0 and xs[1].status() == 0
    for x in xs:
        x.close()


def test_exchange_rejects_bad_arguments(yf, cuda):
    blk = S.packed_floats(1, 8, 128)
    x = S.PeerExchange(0, 2, blk, device=0)
    out = torch.empty((1, 16, 128), dtype=torch.float16, device=cuda)
    with pytest.raises(_abi.YfError):  # rank 1's area is not mapped
        x.push(torch.zeros(blk, device=cuda))
    with pytest.raises(_abi.YfError):  # 3 x 1 parts != world 2
        x.combine(out, 3, 1, 8, 8, 16, 128, 8 * 128)
    with pytest.raises(_abi.YfError):  # lse past the slot
        x.combine(out, 2, 1, 8, 8, 16, 128, blk)
    with pytest.raises(_abi.YfError):
        S.PeerExchange(2, 2, blk, device=0)
    y = S.PeerExchange(1, 2, blk + 4, device=0)
    with pytest.raises(_abi.YfError):  # slot sizes differ
        x.attach(1, y)
    y.close()
    x.close()


def _long_shard_data(yf, oracle, cuda, ctx, Hq, H, D, batch, seed):
    """K/V of `batch` entries of ctx keys, the unsharded GPU decode of them, and q."""
    rng = np.random.default_rng(seed)
    from qwen36_server_b200 import workloads as W
    wl = W.Workload("xd", Hq, H, D, ctx=[ctx] * batch, q_rows=[1] * batch, seed=seed)
    pool = yf.PagedKvPool(1, wl.n_pages, H, D, 16, 32, device=0)
    bt = torch.from_numpy(wl.block_table).to(cuda)
    ks, vs = [], []
    for b in range(batch):
        k = torch.from_numpy(W.kv_rows_np(rng, ctx, H, D, 0.0)).to(cuda)
        v = torch.from_numpy(W.kv_rows_np(rng, ctx, H, D, 0.0)).to(cuda)
        yf.launch_append_multi(pool, 0, k, v, [0, ctx], [0], bt[b:b + 1])
        ks.append(k)
        vs.append(v)
    q = torch.from_numpy(rng.standard_normal((batch, Hq, D)).astype(np.float16)).to(cuda)
    return wl, pool, bt, ks, vs, q


@pytest.mark.parametrize("batch,schedule", [(1, _abi.YF_SCHED_AUTO), (3, _abi.YF_SCHED_AUTO),
                                            (1, _abi.YF_SCHED_CHUNKED)])
def test_exchange_decode_world1(yf, oracle, cuda, batch, schedule):
    """yf_exchange_decode with one rank: the cluster kernel stores its partial into the area,
    raises its own flag and merges in its last CTA (the fused launch), or with the chunked
    schedule the partial + push + combine fallback; either equals the plain decode, over steps
    that alternate the two buffers."""
    ctx, Hq, H, D = 9000, 16, 2, 256
    wl, pool, bt, _, _, q = _long_shard_data(yf, oracle, cuda, ctx, Hq, H, D, batch, 501 + batch)
    pool.set_options(schedule=schedule)
    scale = yf.default_scale(D)
    cu = torch.tensor([i * ctx for i in range(batch + 1)], dtype=torch.int32, device=cuda)
    ref = yf.dispatch_flash_decode_paged(q, pool, 0, cu, bt, scale).float().cpu().numpy()
    x = S.PeerExchange(0, 1, S.packed_floats(batch, Hq, D), device=0)
    ws = torch.empty(max(pool.workspace_size(Hq, batch, 1, ctx), 16), dtype=torch.uint8, device=cuda)
    out = torch.full((batch, Hq, D), float("nan"), dtype=torch.float16, device=cuda)
    for _ in range(3):
        out.fill_(float("nan"))
        x.decode(pool, q, cu, bt, scale, ctx, 1, 1, Hq, out, ws)
        got = out.float().cpu().numpy()
        assert np.isfinite(got).all()
        assert np.abs(got - ref).max() <= 2e-3
    assert x.status() == 0 and pool.status() == 0
    x.close()
    pool.close()


def test_exchange_decode_refuses_emulated_ranks(yf, cuda):
    """Ranks attached on one GPU would wait on one another inside one launch: refused."""
    blk = S.packed_floats(1, 8, 256)
    xs = S.PeerExchange.emulated(2, blk, device=0)
    pool = yf.PagedKvPool(1, 8, 1, 256, 16, 32, device=0)
    q = torch.zeros((1, 8, 256), dtype=torch.float16, device=cuda)
    out = torch.empty((1, 16, 256), dtype=torch.float16, device=cuda)
    ws = torch.empty(1 << 20, dtype=torch.uint8, device=cuda)
    with pytest.raises(_abi.YfError) as e:
        xs[0].decode(pool, q, [0, 16], torch.zeros((1, 1), dtype=torch.int32, device=cuda), 0.1, 16, 2, 1, 16, out, ws)
    assert e.value.code == _abi.YF_E_UNSUPPORTED
    for x in xs:
        x.close()
    pool.close()
