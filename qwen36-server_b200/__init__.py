"""B200 (sm_100a) paged Q8_0 KV attention for the yforge engine's attention path.

libyfattn.so (csrc/, C ABI in include/yfattn.h) holds the kernels; this
package is the host-side mirror of the engine's operator surface
(paged_attn.py) plus the seeded workloads (workloads.py).
"""
from ._abi import YfError, lib  # noqa: F401
from .paged_attn import (  # noqa: F401
    PagedKvPool,
    attn_prepare_append,
    combine_partials,
    default_scale,
    dispatch_flash_decode_paged,
    dispatch_flash_decode_partial,
    forward_attn_prefill_paged,
    forward_verify_paged,
    forward_verify_tree_paged,
    kv_append_paged,
    launch_append_multi,
)
