"""ctypes binding of the pagedkv C ABI (include/pagedkv.h).

The shared library is built in-tree by ``pagedkv.build``. There is no
fallback: if the library is missing or fails to load, every operation raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).with_name("libpagedkv_b200.so")
HEADER_PATH = Path(__file__).resolve().parent.parent.parent / "include" / "pagedkv.h"

PAGEDKV_OK = 0
PAGEDKV_ERR_INVALID_ARGUMENT = 1
PAGEDKV_ERR_UNSUPPORTED = 2
PAGEDKV_ERR_CUDA = 3
PAGEDKV_ERR_WORKSPACE = 4

DTYPE_F16 = 0
DTYPE_BF16 = 1
DTYPE_F32 = 2  # prefill-write sources only

EFLAG_BLOCK_ID_RANGE = 0x1
EFLAG_SLOT_RANGE = 0x2
EFLAG_SEQ_LEN_RANGE = 0x4
EFLAG_COPY_RANGE = 0x8
EFLAG_PIPE_TIMEOUT = 0x10

_EFLAG_NAMES = {
    EFLAG_BLOCK_ID_RANGE: "block-table entry outside [0, num_blocks)",
    EFLAG_SLOT_RANGE: "slot outside [0, num_blocks * block_size)",
    EFLAG_SEQ_LEN_RANGE: "seq_len larger than the block table covers",
    EFLAG_COPY_RANGE: "copy_blocks src/dst outside [0, num_blocks)",
    EFLAG_PIPE_TIMEOUT: "a bounded pipeline wait timed out",
}

_c_i32 = ctypes.c_int32
_c_i64 = ctypes.c_int64
_c_vp = ctypes.c_void_p
_c_f32 = ctypes.c_float
_c_sz = ctypes.c_size_t

# (name, restype, argtypes) for every entry point of include/pagedkv.h.
_SIGNATURES = [
    ("pagedkv_version", ctypes.c_char_p, []),
    ("pagedkv_last_error", ctypes.c_char_p, []),
    (
        "pagedkv_decode_attention",
        ctypes.c_int,
        [
            _c_vp, _c_i64, _c_i64,          # out, strides
            _c_vp, _c_i64, _c_i64,          # q, strides
            _c_vp, _c_vp,                   # k_cache, v_cache
            _c_vp, _c_i64,                  # block_tables, stride
            _c_vp, _c_i32,                  # seq_lens, uniform_seq_len
            _c_i32, _c_i32, _c_i32, _c_i32,  # num_seqs, hq, hkv, head_dim
            _c_i64, _c_i32, _c_i32,         # num_blocks, block_size, max_blocks_per_seq
            _c_f32, _c_i32,                 # scale, dtype
            _c_vp, _c_sz, _c_vp,            # workspace, bytes, stream
        ],
    ),
    (
        "pagedkv_decode_attention_append",
        ctypes.c_int,
        [
            _c_vp, _c_i64, _c_i64,          # out, strides
            _c_vp, _c_i64, _c_i64,          # q, strides
            _c_vp, _c_vp,                   # k_cache, v_cache
            _c_vp, _c_i64,                  # block_tables, stride
            _c_vp,                          # seq_lens
            _c_i32, _c_i32, _c_i32, _c_i32,  # num_seqs, hq, hkv, head_dim
            _c_i64, _c_i32, _c_i32,         # num_blocks, block_size, max_blocks_per_seq
            _c_vp, _c_i64, _c_i64,          # k_new, strides
            _c_vp, _c_i64, _c_i64,          # v_new, strides
            _c_vp, _c_vp, _c_i64,           # cos, sin, row stride
            _c_f32, _c_i32,                 # scale, dtype
            _c_vp, _c_sz, _c_vp,            # workspace, bytes, stream
        ],
    ),
    (
        "pagedkv_decode_attention_workspace_size",
        _c_sz,
        [_c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32],
    ),
    (
        "pagedkv_kv_append",
        ctypes.c_int,
        [
            _c_vp, _c_vp,
            _c_vp, _c_i64, _c_i64,
            _c_vp, _c_i64, _c_i64,
            _c_vp, _c_i32, _c_i32, _c_i32, _c_i64, _c_i32, _c_i32,
            _c_vp,
        ],
    ),
    (
        "pagedkv_copy_blocks",
        ctypes.c_int,
        [_c_vp, _c_vp, _c_i32, _c_vp, _c_i32, _c_i64, _c_i64, _c_vp],
    ),
    (
        "pagedkv_kv_append_rope",
        ctypes.c_int,
        [
            _c_vp, _c_i64, _c_i64,                  # q_out, strides
            _c_vp, _c_i64, _c_i64, _c_i32,          # q, strides, num_q_heads
            _c_vp, _c_vp,                           # k_cache, v_cache
            _c_vp, _c_i64, _c_i64,                  # k_new, strides
            _c_vp, _c_i64, _c_i64,                  # v_new, strides
            _c_vp, _c_vp, _c_i64,                   # cos, sin, row stride
            _c_vp, _c_i32, _c_i32, _c_i32, _c_i64, _c_i32, _c_i32,
            _c_vp,
        ],
    ),
    (
        "pagedkv_kv_write_prefill",
        ctypes.c_int,
        [
            _c_vp, _c_vp, _c_vp, _c_vp, _c_i32,     # k/v pool pointer arrays, k/v source pointer arrays, layers
            _c_i64, _c_i64, _c_i64, _c_i64, _c_i32,  # k/v source strides, source dtype
            _c_vp, _c_i32, _c_i32,                  # block_ids, blocks to write, tokens
            _c_i32, _c_i32, _c_i64, _c_i32, _c_i32,  # kv heads, head_dim, num_blocks, block_size, dtype
            _c_vp,
        ],
    ),
    (
        "pagedkv_decode_attention_noalloc",
        ctypes.c_int,
        [
            _c_vp, _c_i64, _c_i64,
            _c_vp, _c_i64, _c_i64,
            _c_vp, _c_vp,
            _c_vp, _c_i64,
            _c_vp, _c_i32,
            _c_i32, _c_i32, _c_i32, _c_i32,
            _c_i64, _c_i32, _c_i32,
            _c_f32, _c_i32,
            _c_vp,
        ],
    ),
    ("pagedkv_read_error_flags", ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32), _c_i32, _c_vp]),
    ("pagedkv_last_decode_launches", _c_i32, []),
    ("pagedkv_last_decode_kernel", ctypes.c_char_p, []),
]

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Load (once) and return the pagedkv shared library; raise if absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"pagedkv native library not found at {LIB_PATH}; build it with "
                    "`python -m pagedkv.build` (there is no CPU fallback)"
                )
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, restype, argtypes in _SIGNATURES:
                fn = getattr(handle, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = handle
    return _lib


def declared_symbols() -> list[str]:
    """Names of the entry points this binding declares."""
    return [name for name, _, _ in _SIGNATURES]


def check(rc: int, what: str) -> None:
    if rc != PAGEDKV_OK:
        msg = lib().pagedkv_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed (pagedkv status {rc}): {msg}")


def describe_error_flags(flags: int) -> str:
    parts = [text for bit, text in _EFLAG_NAMES.items() if flags & bit]
    return "; ".join(parts) if parts else "none"
