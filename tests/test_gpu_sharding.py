"""Sharded long-context decode kernels against the oracle: the partial decode (O and lse over a
key range), the LSE combine, and the whole sharded decode at world 2/4/8 emulated on one GPU
(each shard its own pool; the all-gather replaced by copies in rank order)."""
import numpy as np
import pytest
import torch

from helpers import TOL, filled_pool, queries
from qwen36_server_b200 import sharding as S
from qwen36_server_b200 import workloads as W

pytestmark = pytest.mark.gpu


def test_combine_kernel_matches_oracle(yf, oracle, cuda):
    rng = np.random.default_rng(5)
    for n_parts, rows, D in [(1, 3, 128), (3, 40, 256), (5, 17, 64), (2, 1, 4)]:
        o = rng.standard_normal((n_parts, rows, D)).astype(np.float32)
        lse = (rng.standard_normal((n_parts, rows)) * 4).astype(np.float32)
        lse[rng.random((n_parts, rows)) < 0.2] = -np.inf
        lse[:, 0] = -np.inf  # a row no part has keys for
        got = yf.combine_partials(torch.from_numpy(o).to(cuda), torch.from_numpy(lse).to(cuda)).float().cpu().numpy()
        ref = oracle.np_combine(o, lse)
        assert np.isfinite(got).all()
        assert np.abs(got - ref).max() <= TOL, (n_parts, rows, D)
        assert (got[0] == 0).all()
    # packed per part: [O | lse | pad] with one stride, as the all-gathered buffer holds them
    n_parts, rows, D = 4, 16, 256
    blk = S.packed_floats(1, rows, D)
    buf = np.zeros(n_parts * blk, np.float32)
    o = rng.standard_normal((n_parts, rows, D)).astype(np.float32)
    lse = rng.standard_normal((n_parts, rows)).astype(np.float32)
    for k in range(n_parts):
        buf[k * blk:k * blk + rows * D] = o[k].reshape(-1)
        buf[k * blk + rows * D:k * blk + rows * D + rows] = lse[k]
    g = torch.from_numpy(buf).to(cuda)
    got = yf.combine_partials(g, g[rows * D:], n_parts=n_parts, rows=rows, head_dim=D, o_part_stride=blk,
                              lse_part_stride=blk).float().cpu().numpy()
    assert np.abs(got - oracle.np_combine(o, lse)).max() <= TOL


def test_decode_partial_matches_oracle(yf, oracle, cuda):
    """O normalised over each entry's keys and lse = ln sum exp(q.k * scale); an entry without keys
    gives O = 0 and lse = -inf; combining one part gives the plain decode output."""
    wl = W.Workload("part", 16, 2, 256, ctx=[0, 1, 300, 5000], q_rows=[1, 1, 1, 1], seed=71)
    pool, img, desc, _, _ = filled_pool(yf, oracle, wl, seed=72)
    q = queries(wl, 73)
    bt = torch.from_numpy(wl.block_table).to(cuda)
    qd = torch.from_numpy(q).to(cuda)
    scale = yf.default_scale(256)
    o, lse = yf.dispatch_flash_decode_partial(qd, pool, 0, wl.cu_k, bt, scale)
    o, lse = o.cpu().numpy(), lse.cpu().numpy()
    G = 8
    for b in range(wl.batch):
        tk = int(wl.ctx[b])
        for h in range(2):
            K, V = oracle.np_dequant_entry(desc, img, 0, wl.block_table[b], tk, h)
            ro, rl = oracle.np_partial_decode(q[b, h * G:(h + 1) * G], K, V, scale)
            assert np.abs(o[b, h * G:(h + 1) * G] - ro).max() <= TOL, (b, h)
            if tk == 0:
                assert np.isneginf(lse[b, h * G:(h + 1) * G]).all()
            else:
                assert np.abs(lse[b, h * G:(h + 1) * G] - rl).max() <= 1e-2, (b, h)
    full = yf.dispatch_flash_decode_paged(qd, pool, 0, wl.cu_k, bt, scale).float().cpu().numpy()
    one = yf.combine_partials(torch.from_numpy(o).to(cuda).view(1, -1, 256),
                              torch.from_numpy(lse).to(cuda).view(1, -1)).float().cpu().numpy()
    assert np.abs(one.reshape(full.shape) - full).max() <= TOL
    assert pool.status() == 0
    pool.close()


@pytest.mark.parametrize("transport", ["nccl", "p2p"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_long_decode_emulated(yf, oracle, cuda, world, transport):
    """The decode_long shape (Hq 16 x D 256, Hkv 2) over 20000 keys split as world ranks would
    split it: every rank's combined output equals the unsharded decode and the oracle.  "nccl"
    stands the all-gather in with copies; "p2p" runs the peer exchange's push of every rank,
    then every rank's combine."""
    ctx, Hq, H, D = 20000, 16, 2, 256
    rng = np.random.default_rng(90 + world)
    k = W.kv_rows_np(rng, ctx, H, D, 0.0)
    v = W.kv_rows_np(rng, ctx, H, D, 0.0)
    q = rng.standard_normal((1, Hq, D)).astype(np.float16)
    scale = yf.default_scale(D)
    # unsharded reference on one pool
    wl = W.Workload("long", Hq, H, D, ctx=[ctx], q_rows=[1], seed=91)
    full_pool = yf.PagedKvPool(1, wl.n_pages, H, D, 16, 32, device=0)
    kd, vd = torch.from_numpy(k).to(cuda), torch.from_numpy(v).to(cuda)
    bt_full = torch.from_numpy(wl.block_table).to(cuda)
    yf.launch_append_multi(full_pool, 0, kd, vd, [0, ctx], [0], bt_full)
    qd = torch.from_numpy(q).to(cuda)
    ref_gpu = yf.dispatch_flash_decode_paged(qd, full_pool, 0, [0, ctx], bt_full, scale).float().cpu().numpy()
    desc = oracle.PoolDesc(1, wl.n_pages, H, D, 16, 32)
    img = np.zeros(desc.pool_bytes, np.uint8)
    oracle.np_kv_write_rows(desc, img, 0, k, v, np.zeros(ctx, np.int32), np.arange(ctx, dtype=np.int32),
                            wl.block_table)
    ref = oracle.c_attn(desc, img, 0, q, np.array([0, 1]), np.array([0, ctx]), wl.block_table, scale)

    plan = S.long_context_plan(world, H, ctx)
    xs = S.PeerExchange.emulated(world, S.packed_floats(1, Hq // plan[0].n_head_groups, D)) \
        if transport == "p2p" else [None] * world
    ranks = []
    for sh in plan:
        n = sh.k1 - sh.k0
        pages = max(1, -(-n // 16))
        r = S.ShardedLongDecode(sh, Hq, H, D, n_pages=pages, device=0, transport=transport,
                                peer_exchange=xs[sh.rank])
        bt = torch.arange(pages, dtype=torch.int32, device=cuda).view(1, pages)
        if n:
            ks = kd[sh.k0:sh.k1, sh.kv_head0:sh.kv_head0 + sh.kv_heads].contiguous()
            vs = vd[sh.k0:sh.k1, sh.kv_head0:sh.kv_head0 + sh.kv_heads].contiguous()
            yf.launch_append_multi(r.pool, 0, ks, vs, [0, n], [0], bt)
        r.partial(r.q_slice(qd), [0, n], bt, scale, max_seqlen_k=max(n, 1))
        ranks.append(r)
    if transport == "p2p":
        for r in ranks:
            r.exchange()
    else:
        gathered = torch.cat([r.local for r in ranks])
        for r in ranks:
            r.gathered.copy_(gathered)
    for r in ranks:
        got = r.combine().float().cpu().numpy()
        assert np.abs(got - ref_gpu).max() <= TOL, r.shard
        assert np.abs(got - ref).max() <= TOL, r.shard
        assert r.pool.status() == 0
    for r in ranks:
        r.pool.close()
    for x in xs:
        if x is not None:
            assert x.status() == 0
            x.close()
    full_pool.close()
