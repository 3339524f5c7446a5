"""pagedkv — B200-native (sm_100a) paged KV-cache decode path.

Kernels live in ``libpagedkv_b200.so`` (C ABI: include/pagedkv.h), built
in-tree by :mod:`pagedkv.build`. The Python functions keep the names,
arguments and preconditions of the reference's
``engine.kernels.paged_attention`` module so they can be installed in its
place (:func:`pagedkv.integration.install`).
"""
from .paged_attention import (
    copy_blocks,
    kv_append,
    kv_append_rope,
    kv_write_prefill,
    last_decode_launch_info,
    pad_block_tables,
    paged_attention_decode,
    paged_attention_decode_append,
    paged_attention_decode_batched,
    paged_attention_decode_v1,
    paged_attention_decode_v2,
    read_error_flags,
)

__all__ = [
    "copy_blocks",
    "kv_append",
    "kv_append_rope",
    "kv_write_prefill",
    "last_decode_launch_info",
    "pad_block_tables",
    "paged_attention_decode",
    "paged_attention_decode_append",
    "paged_attention_decode_batched",
    "paged_attention_decode_v1",
    "paged_attention_decode_v2",
    "read_error_flags",
]

__version__ = "0.1.0"
