"""Parity at the full shapes of the five benchmark configurations.

Every attention output is compared with the oracle's double-precision attention over the
dequantized cache (max |err| <= 2e-3, the bar of the reference's decode probe,
src/bin/decode_gqa_probe.rs:25-63, which sweeps every length it serves):

  decode_batch   all 16 slots, ctx ~ U[1024, 32768], 1% outliers; KV bytes of a slot bit-exact
  decode_long    1 x 131072 keys, Hq 16 x D 256, Hkv 2, every q head: unsharded, and the kv-head x
                 sequence sharding of 2, 4 and 8 ranks (emulated on one GPU, all-gather by copies)
  prefill_chunk  4 x (8192 prefix + 2048 chunk): 256 rows of every entry, spread over the chunk
  mtp_verify     one layer of 64 slots x 4 drafts, ctx ~ U[4096, 65536], every row of every slot

The pools are filled on the device (the f16 rows of these shapes are too large to stage on the
host) and the checked entries' pages are gathered into a compact oracle image.  Each test prints
its largest error.
"""
import numpy as np
import pytest
import torch

from helpers import TOL, device_pool, gathered_image, queries
from qwen36_server_b200 import sharding as S
from qwen36_server_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _report(name, err):
    print(f"\n[parity] {name}: max|err| = {err:.3e} (bar {TOL:.0e})")


def test_decode_batch_every_slot(yf, oracle, cuda):
    wl = W.decode_batch()
    pool = device_pool(yf, wl, seed=201)
    q = queries(wl, 202)
    got = yf.dispatch_flash_decode_paged(torch.from_numpy(q).to(cuda), pool, 0, wl.cu_k,
                                         torch.from_numpy(wl.block_table).to(cuda),
                                         yf.default_scale(128)).float().cpu().numpy()
    assert pool.status() == 0
    worst = 0.0
    for lo in range(0, wl.batch, 8):
        ent = list(range(lo, min(lo + 8, wl.batch)))
        desc, img, sub = gathered_image(oracle, pool, wl, ent)
        ref = oracle.c_attn(desc, img, 0, q[ent], sub.cu_q, sub.cu_k, sub.block_table, yf.default_scale(128))
        err = float(np.abs(got[ent] - ref).max())
        worst = max(worst, err)
        assert err <= TOL, (ent, err)
    _report("decode_batch, 16 of 16 slots", worst)
    # the same seeded rows of slot 0 quantized by the oracle give the pool's bytes exactly
    gen = torch.Generator(device=cuda)
    gen.manual_seed(201)
    n0 = int(wl.ctx[0])
    k = W.kv_rows_torch(gen, n0, 8, 128, wl.outlier_frac, cuda).cpu().numpy()
    v = W.kv_rows_torch(gen, n0, 8, 128, wl.outlier_frac, cuda).cpu().numpy()
    desc, img, sub = gathered_image(oracle, pool, wl, [0])
    mine = np.zeros_like(img)
    oracle.c_kv_write_rows(desc, mine, 0, k, v, np.zeros(n0, np.int32), np.arange(n0, dtype=np.int32),
                           sub.block_table)
    used = -(-n0 // 16) * pool.page_bytes
    assert np.array_equal(mine[:used], img[:used])
    pool.close()


def _decode_long_pool(yf, cuda, ctx=131072, seed=211):
    wl = W.decode_long(ctx=ctx)
    pool = device_pool(yf, wl, seed=seed)
    q = queries(wl, seed + 1)
    return wl, pool, q


def test_decode_long_unsharded(yf, oracle, cuda):
    wl, pool, q = _decode_long_pool(yf, cuda)
    scale = yf.default_scale(256)
    got = yf.dispatch_flash_decode_paged(torch.from_numpy(q).to(cuda), pool, 0, wl.cu_k,
                                         torch.from_numpy(wl.block_table).to(cuda), scale).float().cpu().numpy()
    assert pool.status() == 0
    desc, img, sub = gathered_image(oracle, pool, wl, [0])
    ref = oracle.c_attn(desc, img, 0, q, sub.cu_q, sub.cu_k, sub.block_table, scale)
    err = float(np.abs(got - ref).max())
    _report("decode_long 131072 keys, 16 q heads", err)
    assert err <= TOL
    pool.close()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_decode_long_sharded(yf, oracle, cuda, world):
    """Each rank's shard (kv head group x page-aligned key range) in its own pool, partial decode,
    packed partials gathered in rank order, LSE combine: every rank's output equals the oracle."""
    ctx, Hq, H, D = 131072, 16, 2, 256
    wl = W.decode_long(ctx=ctx)
    gen = torch.Generator(device=cuda)
    gen.manual_seed(220 + world)
    k = W.kv_rows_torch(gen, ctx, H, D, 0.0, cuda)
    v = W.kv_rows_torch(gen, ctx, H, D, 0.0, cuda)
    q = queries(wl, 230 + world)
    qd = torch.from_numpy(q).to(cuda)
    scale = yf.default_scale(D)
    full = yf.PagedKvPool(1, wl.n_pages, H, D, device=0)
    bt_full = torch.from_numpy(wl.block_table).to(cuda)
    yf.launch_append_multi(full, 0, k, v, [0, ctx], [0], bt_full)
    desc, img, sub = gathered_image(oracle, full, wl, [0])
    ref = oracle.c_attn(desc, img, 0, q, sub.cu_q, sub.cu_k, sub.block_table, scale)
    full.close()
    ranks = []
    for sh in S.long_context_plan(world, H, ctx):
        n = sh.k1 - sh.k0
        pages = max(1, -(-n // 16))
        r = S.ShardedLongDecode(sh, Hq, H, D, n_pages=pages, device=0)
        bt = torch.arange(pages, dtype=torch.int32, device=cuda).view(1, pages)
        if n:
            ks = k[sh.k0:sh.k1, sh.kv_head0:sh.kv_head0 + sh.kv_heads].contiguous()
            vs = v[sh.k0:sh.k1, sh.kv_head0:sh.kv_head0 + sh.kv_heads].contiguous()
            yf.launch_append_multi(r.pool, 0, ks, vs, [0, n], [0], bt)
        r.partial(r.q_slice(qd), [0, n], bt, scale, max_seqlen_k=max(n, 1))
        ranks.append(r)
    gathered = torch.cat([r.local for r in ranks])
    worst = 0.0
    for r in ranks:
        r.gathered.copy_(gathered)
        got = r.combine().float().cpu().numpy()
        err = float(np.abs(got - ref).max())
        worst = max(worst, err)
        assert err <= TOL, (r.shard, err)
        assert r.pool.status() == 0
    _report(f"decode_long 131072 keys sharded over {world} ranks", worst)
    for r in ranks:
        r.pool.close()


def test_prefill_chunk_rows_across_every_entry(yf, oracle, cuda):
    """Rows 0, 8, 16, ... and the last row of every entry's 2048-row chunk (257 rows per entry),
    each checked as a one-row causal block at its own key count."""
    wl = W.prefill_chunk()
    pool = device_pool(yf, wl, seed=241)
    q = queries(wl, 242)
    got = yf.forward_attn_prefill_paged(torch.from_numpy(q).to(cuda), pool, 0, wl.cu_q, wl.cu_k,
                                        torch.from_numpy(wl.block_table).to(cuda),
                                        yf.default_scale(128)).float().cpu().numpy()
    assert pool.status() == 0
    worst = 0.0
    for b in range(wl.batch):
        desc, img, sub = gathered_image(oracle, pool, wl, [b])
        tq, tk = int(wl.q_rows[b]), int(wl.ctx[b])
        rows = np.unique(np.concatenate([np.arange(0, tq, 8), [tq - 1]]))
        n = len(rows)
        sub_ctx = tk - tq + rows + 1
        table = np.repeat(sub.block_table, n, axis=0)
        cu_k = np.concatenate([[0], np.cumsum(sub_ctx)])
        ref = oracle.c_attn(desc, img, 0, q[int(wl.cu_q[b]) + rows], np.arange(n + 1), cu_k, table,
                            yf.default_scale(128))
        err = float(np.abs(got[int(wl.cu_q[b]) + rows] - ref).max())
        worst = max(worst, err)
        assert err <= TOL, (b, err)
    _report("prefill_chunk, 257 rows of each of 4 entries", worst)
    pool.close()


def test_mtp_verify_one_layer_every_slot(yf, oracle, cuda):
    wl = W.mtp_verify(n_layers=1)
    pool = device_pool(yf, wl, seed=251)
    q = queries(wl, 252)
    got = yf.forward_verify_paged(torch.from_numpy(q).to(cuda), pool, 0, wl.cu_q, wl.cu_k,
                                  torch.from_numpy(wl.block_table).to(cuda),
                                  yf.default_scale(128)).float().cpu().numpy()
    assert pool.status() == 0
    worst = 0.0
    for lo in range(0, wl.batch, 8):
        ent = list(range(lo, lo + 8))
        desc, img, sub = gathered_image(oracle, pool, wl, ent)
        rows = np.concatenate([np.arange(wl.cu_q[b], wl.cu_q[b + 1]) for b in ent])
        ref = oracle.c_attn(desc, img, 0, q[rows], sub.cu_q, sub.cu_k, sub.block_table, yf.default_scale(128))
        err = float(np.abs(got[rows] - ref).max())
        worst = max(worst, err)
        assert err <= TOL, (ent, err)
    _report("mtp_verify one layer, 64 of 64 slots x 4 rows", worst)
    pool.close()
