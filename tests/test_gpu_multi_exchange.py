"""The sharded long-context decode on two and four GPUs, one process per GPU: the fused exchange
(yf_exchange_decode: each rank's cluster decode stores its partial into every rank's exchange
area over NVLink and merges in its last CTA) and the NCCL all-gather transport against the
unsharded decode on each rank's own GPU.  Split by kv heads and by key ranges.  Skipped with
fewer GPUs than ranks."""
import multiprocessing as mp
import os
import socket
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, H: int, transport: str, q_out):
    import datetime

    os.environ["NCCL_NVLS_ENABLE"] = "0"  # plain peer transport in every library this test uses
    sys.path.insert(0, REPO)
    import __graft_entry__ as graft

    yf = graft.load_package()
    import torch.distributed as dist
    from qwen36_server_b200 import sharding as S
    from qwen36_server_b200 import workloads as W

    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        ctx, Hq, D = 20000, 16, 256
        rng = np.random.default_rng(700 + H)
        k = torch.from_numpy(W.kv_rows_np(rng, ctx, H, D, 0.0)).to(dev)
        v = torch.from_numpy(W.kv_rows_np(rng, ctx, H, D, 0.0)).to(dev)
        scale = yf.default_scale(D)
        # the unsharded decode on this GPU
        wl = W.Workload("m", Hq, H, D, ctx=[ctx], q_rows=[1], seed=701)
        full = yf.PagedKvPool(1, wl.n_pages, H, D, 16, 32, device=rank)
        bt_full = torch.from_numpy(wl.block_table).to(dev)
        yf.launch_append_multi(full, 0, k, v, [0, ctx], [0], bt_full)
        sh = S.long_context_plan(world, H, ctx)[rank]
        n = sh.k1 - sh.k0
        pages = max(1, -(-n // 16))
        sd = S.ShardedLongDecode(sh, Hq, H, D, n_pages=pages, device=rank, transport=transport)
        bt = torch.arange(pages, dtype=torch.int32, device=dev).view(1, pages)
        yf.launch_append_multi(sd.pool, 0, k[sh.k0:sh.k1, sh.kv_head0:sh.kv_head0 + sh.kv_heads].contiguous(),
                               v[sh.k0:sh.k1, sh.kv_head0:sh.kv_head0 + sh.kv_heads].contiguous(), [0, n], [0], bt)
        worst = 0.0
        for step in range(4):
            q = torch.from_numpy(np.random.default_rng(710 + step).standard_normal((1, Hq, D))
                                 .astype(np.float16)).to(dev)
            ref = yf.dispatch_flash_decode_paged(q, full, 0, [0, ctx], bt_full, scale).float()
            dist.barrier()
            got = sd.step(sd.q_slice(q), [0, n], bt, scale, max_seqlen_k=n).float()
            torch.cuda.synchronize()
            assert torch.isfinite(got).all(), step
            worst = max(worst, (got - ref).abs().max().item())
        st = sd.pool.status() | (sd.peer.status() if sd.peer is not None else 0)
        fused = sd.fused if transport == "p2p" else False
        dist.barrier()
        if sd.peer is not None:
            sd.peer.close()
        dist.destroy_process_group()
        q_out.put((rank, worst, st, fused, None))
    except Exception as e:  # reported to the test process
        q_out.put((rank, None, None, None, repr(e)))


@pytest.mark.parametrize("transport", ["p2p", "nccl"])
@pytest.mark.parametrize("H", [2, 1])
@pytest.mark.parametrize("world", [2, 4])
def test_sharded_decode_multi_gpu(world, H, transport):
    """world 2: kv heads split (H 2) or key ranges split (H 1); world 4: both (H 2: 2 head
    groups x 2 key ranges) or four key ranges (H 1)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    port = _free_port()
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, H, transport, q_out)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    for _ in range(world):
        results.append(q_out.get(timeout=300))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank did not exit")
    for rank, worst, st, fused, err in sorted(results):
        assert err is None, (rank, err)
        assert st == 0, (rank, st)
        assert worst <= 2e-3, (rank, worst)
        if transport == "p2p":
            assert fused, rank
