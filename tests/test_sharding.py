"""Host side of the long-context decode split across GPUs, on CPU: the shard plan, the
packed-partials layout, and the all-gather + LSE merge run as gloo ranks against one
unsharded attention (numpy partials stand in for the per-shard kernel)."""
import os
import socket

import numpy as np
import pytest
import torch

import __graft_entry__ as graft

graft.load_package()  # spawned gloo ranks import this module without the conftest
from qwen36_server_b200 import sharding as S  # noqa: E402


def test_plan_covers_every_head_and_key_once():
    for world, H, ctx in [(1, 2, 131072), (2, 2, 131072), (4, 2, 131072), (8, 2, 131072), (2, 4, 1000),
                          (8, 4, 50), (4, 4, 17)]:
        plan = S.long_context_plan(world, H, ctx)
        owned = np.zeros((H, ctx), np.int32)
        for r, sh in enumerate(plan):
            assert sh.rank == r and r == sh.seq * sh.n_head_groups + sh.head_group
            assert sh.k0 % 16 == 0 and 0 <= sh.k0 <= sh.k1 <= ctx
            owned[sh.kv_head0:sh.kv_head0 + sh.kv_heads, sh.k0:sh.k1] += 1
        assert (owned == 1).all(), (world, H, ctx)
    with pytest.raises(ValueError):
        S.long_context_plan(3, 2, 100)
    with pytest.raises(ValueError):
        S.long_context_plan(2, 3, 100)


def _problem(seed, H=2, G=8, D=64, ctx=1500):
    O = graft.load_oracle()
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((H * G, D)).astype(np.float16)
    kq, kd = O.np_quantize_q8(rng.standard_normal((ctx, H, D)).astype(np.float32), 32)
    vq, vd = O.np_quantize_q8(rng.standard_normal((ctx, H, D)).astype(np.float32), 32)
    K = kq.astype(np.float64) * np.repeat(kd.astype(np.float64), 32, axis=-1)
    V = vq.astype(np.float64) * np.repeat(vd.astype(np.float64), 32, axis=-1)
    return q, K, V, 1.0 / np.sqrt(D)


def _rank_packed(sh, q, K, V, scale, G):
    """This rank's packed partial [O | lse] (numpy partials standing in for the kernel)."""
    O = graft.load_oracle()
    D = q.shape[1]
    hq = sh.kv_heads * G
    o = np.zeros((hq, D))
    lse = np.zeros(hq)
    for j in range(sh.kv_heads):
        h = sh.kv_head0 + j
        o[j * G:(j + 1) * G], lse[j * G:(j + 1) * G] = O.np_partial_decode(
            q[h * G:(h + 1) * G], K[sh.k0:sh.k1, h], V[sh.k0:sh.k1, h], scale)
    buf = np.zeros(S.packed_floats(1, hq, D), np.float32)
    buf[:hq * D] = o.reshape(-1)
    buf[hq * D:hq * D + hq] = lse
    return buf


def _combine_gathered(sh, gathered, Hq, D):
    O = graft.load_oracle()
    hq = Hq // sh.n_head_groups
    out = np.zeros((Hq, D))
    for g, (oo, lo, stride, n, rows) in enumerate(S.combine_views(sh, 1, hq, D)):
        o_parts = np.stack([gathered[oo + k * stride: oo + k * stride + rows * D].reshape(rows, D) for k in range(n)])
        l_parts = np.stack([gathered[lo + k * stride: lo + k * stride + rows] for k in range(n)])
        out[g * rows:(g + 1) * rows] = O.np_combine(o_parts, l_parts)
    return out


def _full(q, K, V, scale, G):
    O = graft.load_oracle()
    H = K.shape[1]
    return np.concatenate([O.np_partial_decode(q[h * G:(h + 1) * G], K[:, h], V[:, h], scale)[0] for h in range(H)])


@pytest.mark.parametrize("world,H", [(1, 2), (2, 2), (4, 2), (8, 2), (2, 4)])
def test_packed_layout_merges_to_unsharded(world, H):
    G = 4
    q, K, V, scale = _problem(7 + world, H=H, G=G, ctx=700)
    plan = S.long_context_plan(world, H, K.shape[0])
    gathered = np.concatenate([_rank_packed(sh, q, K, V, scale, G) for sh in plan])
    got = _combine_gathered(plan[0], gathered, H * G, q.shape[1])
    assert np.abs(got - _full(q, K, V, scale, G)).max() < 1e-5


def _worker(rank, world, port, H, G, out_q):
    import torch.distributed as dist
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        q, K, V, scale = _problem(11, H=H, G=G, ctx=2000)
        sh = S.long_context_plan(world, H, K.shape[0])[rank]
        local = torch.from_numpy(_rank_packed(sh, q, K, V, scale, G))
        gathered = torch.empty(world * local.numel(), dtype=torch.float32)
        S.gather_packed(local, gathered, world)
        got = _combine_gathered(sh, gathered.numpy(), H * G, q.shape[1])
        err = float(np.abs(got - _full(q, K, V, scale, G)).max())
        dist.destroy_process_group()
        out_q.put((rank, err))
    except Exception as e:  # reported to the parent
        out_q.put((rank, repr(e)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_ranks_all_gather_and_merge(world):
    """Each rank holds one shard, all-gathers the packed partials and merges them: every rank
    ends with the unsharded output."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 2, 8, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=90) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, err in res:
        assert isinstance(err, float), (rank, err)
        assert err < 1e-5, (rank, err)


def test_lpt_partition_balances_and_covers_every_slot():
    from qwen36_server_b200 import workloads as W

    wl = W.decode_batch()
    for n in (1, 2, 4, 8, 16):
        bins = S.lpt_partition(wl.ctx, n)
        flat = sorted(i for b in bins for i in b)
        assert flat == list(range(wl.batch))
        loads = [int(wl.ctx[b].sum()) for b in bins]
        # LPT's bound: no bin exceeds the mean by more than the largest single slot
        assert max(loads) <= wl.ctx.sum() / n + wl.ctx.max()
        assert S.lpt_partition(wl.ctx, n) == bins          # deterministic
    assert S.lpt_partition([5, 5, 5, 5], 2) == [[0, 2], [1, 3]]
    assert S.lpt_partition([9, 1, 1, 1], 2) == [[0], [1, 2, 3]]
    mv = W.mtp_verify(n_layers=1)
    bins = S.lpt_partition(mv.ctx, 8)
    loads = [int(mv.ctx[b].sum()) for b in bins]
    assert max(loads) / (sum(loads) / 8) < 1.05                # 64 slots over 8 GPUs: within 5%
