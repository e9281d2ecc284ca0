"""ctypes binding of libyfattn.so (the C ABI declared in include/yfattn.h).

The library is loaded from this package directory.  There is no fallback: if
the shared object is missing the import fails and says how to build it.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libyfattn.so")

YF_OK = 0
YF_E_INVALID = 1
YF_E_UNSUPPORTED = 2
YF_E_NOMEM = 3
YF_E_CUDA = 4
YF_E_RANGE = 5
YF_E_WORKSPACE = 6
YF_E_STATE = 7

YF_DEV_BAD_PAGE = 1
YF_DEV_LEN_OVERFLOW = 2
YF_DEV_BAD_POS = 4
YF_DEV_BAD_ROWS = 8
YF_DEV_TIMEOUT = 16
YF_DEV_SMEM_ALIGN = 32

YF_SCHED_AUTO = 0
YF_SCHED_CHUNKED = 1
YF_SCHED_PERSISTENT = 2
YF_MERGE_IN_KERNEL = 0
YF_MERGE_SEPARATE = 1
YF_PREFILL_AUTO = 0
YF_PREFILL_SPLITKV = 1
YF_LAUNCH_PLAIN = 0
YF_VERIFY_AUTO = 0
YF_VERIFY_TCGEN05 = 1
YF_LAUNCH_COOPERATIVE = 1
YF_POOL_COUNTERS = 65536 + 4096
YF_REC_REJECTED = 0
YF_REC_RESTORED = 1
YF_REC_MISMATCH = 2
YF_EXCHANGE_HANDLE_BYTES = 64

ERROR_NAMES = {
    YF_E_INVALID: "YF_E_INVALID", YF_E_UNSUPPORTED: "YF_E_UNSUPPORTED", YF_E_NOMEM: "YF_E_NOMEM",
    YF_E_CUDA: "YF_E_CUDA", YF_E_RANGE: "YF_E_RANGE", YF_E_WORKSPACE: "YF_E_WORKSPACE", YF_E_STATE: "YF_E_STATE",
}


class YfError(RuntimeError):
    """A non-zero return code of the C ABI, with yf_last_error()'s message."""

    def __init__(self, code: int, func: str, msg: str):
        super().__init__(f"{func}: {ERROR_NAMES.get(code, code)}: {msg}")
        self.code = code


class PoolDesc(ctypes.Structure):
    _fields_ = [
        ("n_layers", ctypes.c_int32), ("n_pages", ctypes.c_int32), ("n_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32), ("page_size", ctypes.c_int32), ("group_size", ctypes.c_int32),
        ("device", ctypes.c_int32), ("reserved", ctypes.c_int32), ("device_mem", ctypes.c_void_p),
    ]


class AttnOptions(ctypes.Structure):
    """yf_attn_options: the pool's explicit attention choices (all zero = the defaults)."""
    _fields_ = [
        ("schedule", ctypes.c_int32), ("chunk_tiles", ctypes.c_int32), ("copy_stages", ctypes.c_int32),
        ("merge", ctypes.c_int32), ("prefill_kernel", ctypes.c_int32), ("wait_limit_us", ctypes.c_uint32),
        ("launch", ctypes.c_int32), ("verify_kernel", ctypes.c_int32), ("reserved", ctypes.c_int32 * 8),
    ]


_i32, _u32, _sz, _vp, _f32 = ctypes.c_int32, ctypes.c_uint32, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_float
_ci = ctypes.c_int
_P_i32 = ctypes.POINTER(ctypes.c_int32)

# name -> (restype, argtypes); every function of include/yfattn.h
SIGNATURES = {
    "yf_last_error": (ctypes.c_char_p, []),
    "yf_abi_version": (_ci, []),
    "yf_pool_page_head_bytes": (_sz, [_vp]),
    "yf_pool_bytes": (_sz, [_vp]),
    "yf_pool_tile_offset": (ctypes.c_int64, [_vp, _ci, _ci, _ci]),
    "yf_pool_scale_offset": (ctypes.c_int64, [_vp, _ci, _ci, _ci]),
    "yf_pool_create": (_ci, [_vp, ctypes.POINTER(_vp)]),
    "yf_pool_destroy": (_ci, [_vp]),
    "yf_pool_get_desc": (_ci, [_vp, _vp]),
    "yf_pool_layer_ptr": (_ci, [_vp, _i32, ctypes.POINTER(_vp)]),
    "yf_pool_alloc_pages": (_ci, [_vp, _i32, _vp]),
    "yf_pool_retain_pages": (_ci, [_vp, _i32, _vp]),
    "yf_pool_free_pages": (_ci, [_vp, _i32, _vp]),
    "yf_pool_free_count": (_ci, [_vp, _P_i32]),
    "yf_pool_refcount": (_ci, [_vp, _i32, _P_i32]),
    "yf_pool_status": (_ci, [_vp, ctypes.POINTER(_u32), _ci]),
    "yf_pool_set_options": (_ci, [_vp, _vp]),
    "yf_pool_get_options": (_ci, [_vp, _vp]),
    "yf_pool_plant_counter": (_ci, [_vp, _i32, _u32, _vp]),
    "yf_kv_append_paged": (_ci, [_vp, _i32, _vp, _vp, _vp, _vp, _i32, _i32, _vp]),
    "yf_kv_append_paged_multi": (_ci, [_vp, _i32, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp]),
    "yf_attn_prepare_append": (_ci, [_vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _f32, _i32, _vp, _vp, _i32, _i32,
                                     _vp, _vp, _vp, _i32, _i32, _i32, _vp, _vp, _vp]),
    "yf_attn_workspace_size": (_sz, [_vp, _i32, _i32, _i32, _i32]),
    "yf_attn_decode": (_ci, [_vp, _i32, _vp, _i32, _vp, _vp, _i32, _i32, _i32, _f32, _vp, _vp, _sz, _vp]),
    "yf_attn_decode_noalloc": (_ci, [_vp, _i32, _vp, _i32, _vp, _vp, _i32, _i32, _i32, _f32, _vp, _vp]),
    "yf_attn_prefill": (_ci, [_vp, _i32, _vp, _i32, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _f32, _vp, _vp, _sz,
                              _vp]),
    "yf_attn_verify_tree": (_ci, [_vp, _i32, _vp, _i32, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _f32, _vp, _vp, _vp,
                                  _sz, _vp]),
    "yf_attn_decode_partial": (_ci, [_vp, _i32, _vp, _i32, _vp, _vp, _i32, _i32, _i32, _f32, _vp, _vp, _vp, _sz,
                                     _vp]),
    "yf_attn_combine": (_ci, [_vp, ctypes.c_int64, _vp, ctypes.c_int64, _i32, _i32, _i32, _vp, _vp]),
    "yf_pool_record_bytes": (_sz, [_vp]),
    "yf_pool_export_records": (_ci, [_vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "yf_pool_import_records": (_ci, [_vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp]),
    "yf_exchange_create": (_ci, [_i32, _i32, _i32, ctypes.c_int64, ctypes.POINTER(_vp)]),
    "yf_exchange_destroy": (_ci, [_vp]),
    "yf_exchange_handle": (_ci, [_vp, _vp]),
    "yf_exchange_open_peer": (_ci, [_vp, _i32, _vp]),
    "yf_exchange_attach": (_ci, [_vp, _i32, _vp]),
    "yf_exchange_set_wait_limit": (_ci, [_vp, _u32]),
    "yf_exchange_push": (_ci, [_vp, _vp, _vp]),
    "yf_exchange_combine": (_ci, [_vp, _i32, _i32, _i32, _i32, _i32, _i32, ctypes.c_int64, _vp, _vp]),
    "yf_exchange_decode": (_ci, [_vp, _vp, _i32, _vp, _i32, _vp, _vp, _i32, _i32, _i32, _f32, _i32, _i32, _i32, _vp,
                                 _vp, _sz, _vp]),
    "yf_exchange_status": (_ci, [_vp, ctypes.POINTER(_u32), _ci]),
    "yf_pool_export_pages": (_ci, [_vp, _i32, _i32, _vp, _vp, _vp]),
    "yf_pool_restore_pages": (_ci, [_vp, _i32, _i32, _vp, _vp, _vp]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Loads libyfattn.so (no fallback) and declares every exported signature."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is not built: run `python qwen36-server_b200/build.py` "
                              "or __graft_entry__.build()")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int, func: str) -> None:
    if rc != YF_OK:
        msg = lib().yf_last_error()
        raise YfError(rc, func, msg.decode() if msg else "")


def call(name: str, *args) -> None:
    """Calls an int-returning entry point and raises YfError on a non-zero code."""
    check(getattr(lib(), name)(*args), name)
