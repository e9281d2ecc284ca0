"""The C ABI without a GPU: exported symbols, layout functions, the page allocator of a
host-only pool and host-side argument validation."""
import ctypes
import os
import re

import numpy as np
import pytest

from qwen36_server_b200 import _abi

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "yfattn.h")


def declared_functions():
    src = open(HEADER).read()
    return re.findall(r"^YF_API [^;]*?\b(yf_\w+)\(", src, flags=re.M)


def test_library_exports_every_declared_symbol(yf):
    names = declared_functions()
    assert len(names) >= 20
    L = yf.lib()
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(_abi.SIGNATURES), set(names) ^ set(_abi.SIGNATURES)
    assert L.yf_abi_version() == 2


@pytest.mark.parametrize("D,P,G", [(128, 16, 32), (256, 64, 32), (256, 64, 256), (128, 16, 128), (256, 16, 32)])
def test_layout_offsets_match_oracle(yf, oracle, D, P, G):
    L = yf.lib()
    d = _abi.PoolDesc(1, 4, 2, D, P, G, -1, 0, None)
    od = oracle.PoolDesc(1, 4, 2, D, P, G)
    ko, vo, kso, vso = oracle.layout_maps(od)
    lk = np.array([[L.yf_pool_tile_offset(ctypes.byref(d), 0, t, x) for x in range(D)] for t in range(16)])
    lv = np.array([[L.yf_pool_tile_offset(ctypes.byref(d), 1, t, x) for x in range(D)] for t in range(16)])
    assert np.array_equal(lk, ko) and np.array_equal(lv, vo)
    for t in range(16):
        for s in range(D // G):
            assert L.yf_pool_scale_offset(ctypes.byref(d), 0, t, s) == kso[t, s]
            assert L.yf_pool_scale_offset(ctypes.byref(d), 1, t, s) == vso[t, s]
    every = np.concatenate([ko.ravel(), vo.ravel(), kso.ravel(), kso.ravel() + 1, vso.ravel(), vso.ravel() + 1])
    assert np.array_equal(np.sort(every), np.arange(od.tile_bytes))  # a bijection onto the tile
    assert L.yf_pool_page_head_bytes(ctypes.byref(d)) == od.page_head_bytes
    assert L.yf_pool_bytes(ctypes.byref(d)) == od.pool_bytes
    assert L.yf_pool_tile_offset(ctypes.byref(d), 0, 16, 0) == -1


def test_unsupported_shapes_are_refused(yf):
    for D, P, G in [(64, 16, 32), (128, 32, 32), (128, 16, 64)]:
        desc = _abi.PoolDesc(1, 4, 2, D, P, G, -1, 0, None)
        h = ctypes.c_void_p()
        assert yf.lib().yf_pool_create(ctypes.byref(desc), ctypes.byref(h)) == _abi.YF_E_UNSUPPORTED
        assert b"built for" in yf.lib().yf_last_error()


def test_page_allocator(yf):
    pool = yf.PagedKvPool(2, 10, 8, 128, device=None)
    assert pool.free_count() == 10
    a = pool.alloc_pages(4)
    assert a == [0, 1, 2, 3] and pool.free_count() == 6
    assert all(pool.refcount(p) == 1 for p in a)
    pool.retain_pages([1, 2])          # a prefix shared with a second slot
    pool.free_pages(a)
    assert pool.free_count() == 8 and pool.refcount(1) == 1 and pool.refcount(0) == 0
    with pytest.raises(yf.YfError) as e:
        pool.free_pages([0])           # already free
    assert e.value.code == _abi.YF_E_STATE
    with pytest.raises(yf.YfError) as e:
        pool.free_pages([1, 1])        # one reference left, two drops: nothing changes
    assert e.value.code == _abi.YF_E_STATE and pool.refcount(1) == 1
    pool.free_pages([1, 2])
    assert pool.free_count() == 10
    with pytest.raises(yf.YfError) as e:
        pool.alloc_pages(11)
    assert e.value.code == _abi.YF_E_NOMEM and pool.free_count() == 10
    with pytest.raises(yf.YfError) as e:
        pool.retain_pages([3])
    assert e.value.code == _abi.YF_E_STATE
    with pytest.raises(yf.YfError) as e:
        pool.free_pages([10])
    assert e.value.code == _abi.YF_E_RANGE
    # freed pages come back LIFO: a fragmented table after interleaved frees
    x = pool.alloc_pages(6)
    pool.free_pages([x[1], x[4]])
    assert sorted(pool.alloc_pages(2)) == sorted([x[1], x[4]])
    pool.close()


def test_device_calls_on_host_only_pool_are_invalid(yf):
    pool = yf.PagedKvPool(1, 4, 2, 128, device=None)
    L = yf.lib()
    rc = L.yf_attn_decode(pool.handle, 0, 16, 8, 16, 16, 1, 1, 16, ctypes.c_float(0.1), 16, None, 0, None)
    assert rc == _abi.YF_E_INVALID
    rc = L.yf_kv_append_paged(pool.handle, 0, 16, 16, 16, 16, 1, 1, None)
    assert rc == _abi.YF_E_INVALID
    v = ctypes.c_uint32()
    assert L.yf_pool_status(pool.handle, ctypes.byref(v), 0) == _abi.YF_E_INVALID
    pool.close()


def test_workspace_size_plan(yf):
    pool = yf.PagedKvPool(1, 4, 8, 128, device=None)
    L = yf.lib()
    row = 8 * 129 * 4   # one partial: rows_per_cta x (D + 1) floats
    # few units: the cluster schedule, one cluster per unit for 8 units of 4 tiles (no partials)
    assert L.yf_attn_workspace_size(pool.handle, 32, 1, 1, 64) == 0
    # the same units over two entries (lengths may differ): persistent, 4 CTAs x 2 partial slots
    assert L.yf_attn_workspace_size(pool.handle, 32, 2, 1, 64) == 4 * 2 * row
    # persistent decode: two partial slots per CTA, at least 16 tiles per CTA, at most 4 CTAs/SM
    pool.set_options(schedule=_abi.YF_SCHED_PERSISTENT)
    assert L.yf_attn_workspace_size(pool.handle, 32, 1, 1, 64) == 2 * 2 * row   # 32 tiles -> 2 CTAs
    pool.set_options(schedule=_abi.YF_SCHED_AUTO)
    ws = L.yf_attn_workspace_size(pool.handle, 32, 16, 1, 32768)
    assert ws == 148 * 4 * 2 * row        # 128 units: persistent
    # past the persistent batch limit the chunked plan applies; short keys need no split
    assert L.yf_attn_workspace_size(pool.handle, 32, 2000, 1, 256) == 0
    assert L.yf_attn_workspace_size(pool.handle, 30, 16, 1, 32768) == 0   # Hq not a multiple of Hkv
    pool.close()
    long_pool = yf.PagedKvPool(1, 4, 2, 256, device=None)
    row256 = 8 * 257 * 4
    # one 131072-key entry, 2 kv heads, D 256: clusters of 8 CTAs, one wave of them (on a host-only
    # pool the estimate 2 x 148 / 8 = 37 clusters) -> 18 clusters per unit, one partial each
    assert L.yf_attn_workspace_size(long_pool.handle, 16, 1, 1, 131072) == 2 * 18 * row256
    # persistent: at most max(1.75 x 148, 128 per unit) = 259 CTAs instead of a full 4-per-SM wave
    long_pool.set_options(schedule=_abi.YF_SCHED_PERSISTENT)
    assert L.yf_attn_workspace_size(long_pool.handle, 16, 1, 1, 131072) == 259 * 2 * row256
    long_pool.close()


def test_attention_options_are_explicit_and_validated(yf):
    """The pool's options replace every hidden tuning switch: zero is the default, unknown values
    are refused and leave the options unchanged, and the workspace query follows the schedule."""
    pool = yf.PagedKvPool(1, 4096, 8, 128, device=None)
    assert pool.options() == {"schedule": 0, "chunk_tiles": 0, "copy_stages": 0, "merge": 0,
                              "prefill_kernel": 0, "wait_limit_us": 0, "launch": 0,
                              "verify_kernel": 0}
    pool.set_options(schedule=_abi.YF_SCHED_CHUNKED, chunk_tiles=8, wait_limit_us=20000)
    assert pool.options()["schedule"] == 1 and pool.options()["chunk_tiles"] == 8
    for bad in ({"schedule": 3}, {"copy_stages": 2}, {"merge": 5}, {"prefill_kernel": -1},
                {"chunk_tiles": -1}, {"wait_limit_us": 61_000_000}, {"launch": 2},
                {"verify_kernel": 2}):
        with pytest.raises(yf.YfError) as e:
            pool.set_options(**bad)
        assert e.value.code == _abi.YF_E_INVALID, bad
    assert pool.options()["chunk_tiles"] == 8
    o = _abi.AttnOptions()
    o.reserved[3] = 1
    assert yf.lib().yf_pool_set_options(pool.handle, ctypes.byref(o)) == _abi.YF_E_INVALID
    # the chunked schedule sizes its workspace by chunks, the persistent one by CTAs
    L = yf.lib()
    chunked = L.yf_attn_workspace_size(pool.handle, 32, 16, 1, 32768)
    pool.set_options(schedule=0, chunk_tiles=0)
    persistent = L.yf_attn_workspace_size(pool.handle, 32, 16, 1, 32768)
    assert chunked > 0 and persistent > 0 and chunked != persistent
    assert L.yf_pool_plant_counter(pool.handle, 0, 1, None) == _abi.YF_E_INVALID   # host-only pool


def test_exchange_arguments_are_validated_without_a_device(yf):
    """yf_exchange_create refuses a bad rank, world or slot size before any CUDA call, leaving
    the output null; the other exchange entry points refuse null handles."""
    L = yf.lib()
    h = ctypes.c_void_p()
    for device, rank, world, slot in [(0, 0, 0, 16), (0, 2, 2, 16), (0, -1, 2, 16), (0, 0, 65, 16),
                                      (0, 0, 2, 6), (0, 0, 2, 0)]:
        assert L.yf_exchange_create(device, rank, world, slot, ctypes.byref(h)) == _abi.YF_E_INVALID
        assert not h.value
    assert L.yf_exchange_create(0, 0, 2, 16, None) == _abi.YF_E_INVALID
    buf = (ctypes.c_uint8 * _abi.YF_EXCHANGE_HANDLE_BYTES)()
    assert L.yf_exchange_handle(None, buf) == _abi.YF_E_INVALID
    assert L.yf_exchange_push(None, None, None) == _abi.YF_E_INVALID
    bits = ctypes.c_uint32()
    assert L.yf_exchange_status(None, ctypes.byref(bits), 0) == _abi.YF_E_INVALID
    assert L.yf_exchange_destroy(None) == _abi.YF_OK
