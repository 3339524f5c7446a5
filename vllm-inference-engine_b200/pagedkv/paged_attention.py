"""B200 paged decode attention with the reference's Python interface.

Drop-in for the kernel entry points of the reference module
``engine/kernels/paged_attention.py``:

* ``paged_attention_decode_batched`` (reference :634-698)
* ``paged_attention_decode_v1`` (reference :254-305) and
  ``paged_attention_decode_v2`` (reference :419-470)
* ``paged_attention_decode`` (reference stub :86-99, list-of-lists tables)
* ``pad_block_tables`` (reference :473-505)

plus the two pool-write operations of the same path:

* ``kv_append`` — the decode append of paged_attention_integration.py:150-160,
  one launch per layer through a slot mapping;
* ``copy_blocks`` — the copy-on-write block copy over all layers.

Same argument names, shapes and meaning; the same ``AssertionError`` for the
preconditions the reference asserts. Every call launches the sm_100a kernels of
``libpagedkv_b200.so`` on the current torch CUDA stream. There is no Triton,
no CPU path and no fallback: a CPU tensor or a missing library raises.

Beyond the reference: bf16 pools are accepted as well as fp16, and q/out may
be strided views (last dimension contiguous).

Streams: every decode-attention call on a device uses ONE cached workspace
of that device (the tensor-core kernel's cross-CTA completion flags and
split-K partial sums; a CUDA graph captured through this module bakes the
same buffer in). Decode-attention calls (or graph replays) that could run at
the same time on one device — issued on two streams without an event between
them — race on it and must not be made; calls from one stream, or ordered by
events, are safe. Callers that need concurrent decodes on one device pass
their own workspaces through the C ABI (``pagedkv_decode_attention``).
"""
from __future__ import annotations

import ctypes
import os
from typing import Any, Sequence

import torch

from . import _native

_DEBUG = os.environ.get("PAGEDKV_DEBUG", "0") not in ("", "0")

_DTYPES = {torch.float16: _native.DTYPE_F16, torch.bfloat16: _native.DTYPE_BF16}

# Split-K scratch, one cached buffer per device, grown on demand; shared by
# every stream of the device (see the module docstring).
_workspaces: dict[int, torch.Tensor] = {}
# Workspace bytes per launch shape (the query is a host-side computation).
_ws_sizes: dict[tuple, int] = {}
_retired_workspaces: list[torch.Tensor] = []


def _workspace(idx: int, nbytes: int) -> torch.Tensor | None:
    if nbytes == 0:
        return None
    buf = _workspaces.get(idx)
    if buf is None or buf.numel() < nbytes:
        if buf is not None:
            # A CUDA graph captured earlier may still point at the old buffer.
            _retired_workspaces.append(buf)
        size = max(nbytes, 1 << 20)
        # zero-filled once: the first 8 KiB are completion flags the kernels
        # expect at zero and leave at zero
        buf = torch.zeros(size, dtype=torch.uint8, device=torch.device("cuda", idx))
        _workspaces[idx] = buf
    return buf


# The current stream's raw handle without building a torch Stream object
# (about 10x cheaper per call); torch builds without the binding use the
# public route.
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream_handle(device: torch.device | int) -> int:
    idx = device if isinstance(device, int) else device.index
    if idx is None:
        idx = torch.cuda.current_device()
    if _raw_stream is not None:
        return _raw_stream(idx)
    return torch.cuda.current_stream(idx).cuda_stream


def _launch(idx: int, fn, *args) -> int:
    """Call the C entry ``fn(*args, stream)`` with device ``idx`` current and
    its current torch stream as the last argument."""
    if torch.cuda.current_device() == idx:
        return fn(*args, _stream_handle(idx))
    with torch.cuda.device(idx):
        return fn(*args, _stream_handle(idx))


def _qo_ok(t: torch.Tensor) -> bool:
    s0, s1, s2 = t.stride()
    return s2 == 1 and s0 % 8 == 0 and s1 % 8 == 0 and t.data_ptr() % 16 == 0


def _device_guard(device: torch.device):
    if device.index is not None and torch.cuda.current_device() != device.index:
        return torch.cuda.device(device)
    return None


def _debug_check(device: torch.device, what: str) -> None:
    if _DEBUG:
        flags = read_error_flags(device, clear=True)
        if flags:
            raise RuntimeError(f"{what}: device error flags 0x{flags:x} ({_native.describe_error_flags(flags)})")


def read_error_flags(device: torch.device | str | int | None = None, clear: bool = True) -> int:
    """Return (and by default clear) the device error word the kernels set when
    they skip an out-of-range block id, slot or length. Synchronises the stream.

    A reported pipeline timeout (``EFLAG_PIPE_TIMEOUT``) means a decode launch
    gave up part way, possibly leaving completion flags set in its workspace
    header; the header of this device's cached workspace is zeroed again here,
    so the next launch starts from the state the kernels expect."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if dev.type == "cuda" and dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    out = _native.ctypes.c_uint32(0)
    guard = _device_guard(dev)
    if guard is not None:
        with guard:
            rc = _native.lib().pagedkv_read_error_flags(_native.ctypes.byref(out), int(clear), _stream_handle(dev))
    else:
        rc = _native.lib().pagedkv_read_error_flags(_native.ctypes.byref(out), int(clear), _stream_handle(dev))
    _native.check(rc, "pagedkv_read_error_flags")
    flags = int(out.value)
    if flags & _native.EFLAG_PIPE_TIMEOUT:
        ws = _workspaces.get(dev.index)
        if ws is not None:
            ws[:8192].zero_()  # the cross-CTA completion flags
            torch.cuda.synchronize(dev)
    return flags


def _decode_into(
    out: torch.Tensor,
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor | None,
    uniform_seq_len: int,
    scale: float,
) -> None:
    """Launch decode attention writing into ``out`` ([N, Hq, D])."""
    assert k_cache.is_contiguous() and v_cache.is_contiguous(), "KV pool tensors must be contiguous"
    kshape = k_cache.shape
    assert v_cache.shape == kshape, "k_cache and v_cache must have the same shape"
    num_seqs, num_q_heads, head_dim = q.shape
    num_blocks, block_size, num_kv_heads, _ = kshape
    if num_seqs == 0:
        return
    if block_tables.stride(-1) != 1:
        block_tables = block_tables.contiguous()
    if seq_lens is not None and not seq_lens.is_contiguous():
        seq_lens = seq_lens.contiguous()
    qq = q if _qo_ok(q) else q.contiguous()
    oo = out if _qo_ok(out) else torch.empty(q.shape, dtype=q.dtype, device=q.device)
    dtype = _DTYPES[q.dtype]
    max_blocks = block_tables.shape[1]
    idx = q.get_device()
    lib = _native.lib()
    key = (idx, num_seqs, num_q_heads, num_kv_heads, head_dim, block_size, max_blocks, dtype)
    nbytes = _ws_sizes.get(key)
    if nbytes is None:
        nbytes = lib.pagedkv_decode_attention_workspace_size(
            num_seqs, num_q_heads, num_kv_heads, head_dim, block_size, max_blocks, dtype
        )
        _ws_sizes[key] = nbytes
    ws = _workspace(idx, nbytes)
    qs, os_ = qq.stride(), oo.stride()
    rc = _launch(
        idx, lib.pagedkv_decode_attention,
        oo.data_ptr(), os_[0], os_[1],
        qq.data_ptr(), qs[0], qs[1],
        k_cache.data_ptr(), v_cache.data_ptr(),
        block_tables.data_ptr(), block_tables.stride(0),
        seq_lens.data_ptr() if seq_lens is not None else None, int(uniform_seq_len),
        num_seqs, num_q_heads, num_kv_heads, head_dim,
        num_blocks, block_size, max_blocks,
        float(scale), dtype,
        ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
    )
    if rc:
        _native.check(rc, "pagedkv_decode_attention")
    if oo is not out:
        out.copy_(oo)
    if _DEBUG:
        _debug_check(q.device, "paged decode attention")


class _NullCtx:
    def __enter__(self):
        return None

    def __exit__(self, *exc):
        return False


def paged_attention_decode_batched(
    q: torch.Tensor,            # [num_seqs, num_q_heads, head_dim] (fp16/bf16, cuda)
    k_cache: torch.Tensor,      # [num_blocks, block_size, num_kv_heads, head_dim]
    v_cache: torch.Tensor,      # [num_blocks, block_size, num_kv_heads, head_dim]
    block_tables: torch.Tensor,  # [num_seqs, max_blocks_per_seq] (int32, cuda)
    seq_lens: torch.Tensor,     # [num_seqs] (int32, cuda)
    scale: float,
) -> torch.Tensor:
    """Batched decode attention over paged K/V (reference paged_attention.py:634-698).

    Same preconditions as the reference (asserted identically), output
    ``torch.empty_like(q)`` filled by the sm_100a kernel.
    """
    assert q.is_cuda and k_cache.is_cuda and v_cache.is_cuda
    assert block_tables.is_cuda and seq_lens.is_cuda
    assert q.dtype in _DTYPES and k_cache.dtype == q.dtype and v_cache.dtype == q.dtype
    assert block_tables.dtype == torch.int32 and seq_lens.dtype == torch.int32

    num_seqs, num_q_heads, head_dim = q.shape
    num_blocks, block_size, num_kv_heads, head_dim_k = k_cache.shape
    assert head_dim == head_dim_k, f"Head dimensions must match: {head_dim} vs {head_dim_k}"
    assert num_q_heads % num_kv_heads == 0, (
        f"num_q_heads ({num_q_heads}) must be divisible by num_kv_heads ({num_kv_heads})"
    )
    assert block_tables.shape[0] == num_seqs
    assert seq_lens.shape[0] == num_seqs

    out = torch.empty_like(q)
    _decode_into(out, q, k_cache, v_cache, block_tables, seq_lens, 0, scale)
    return out


def _single_sequence(q, k_cache, v_cache, block_table, seq_len, scale) -> torch.Tensor:
    assert q.is_cuda and k_cache.is_cuda and v_cache.is_cuda and block_table.is_cuda
    assert q.dtype in _DTYPES and k_cache.dtype == q.dtype and v_cache.dtype == q.dtype
    assert block_table.dtype == torch.int32

    num_q_heads, head_dim = q.shape
    num_blocks, block_size, num_kv_heads, head_dim_k = k_cache.shape
    assert head_dim == head_dim_k, f"Head dimensions must match: {head_dim} vs {head_dim_k}"
    assert num_q_heads % num_kv_heads == 0, (
        f"num_q_heads ({num_q_heads}) must be divisible by num_kv_heads ({num_kv_heads})"
    )
    seq_len = int(seq_len)
    num_blocks_for_seq = (seq_len + block_size - 1) // block_size
    assert block_table.shape[0] >= num_blocks_for_seq, (
        f"block_table size ({block_table.shape[0]}) smaller than needed ({num_blocks_for_seq})"
    )
    out = torch.empty_like(q)
    table = block_table.reshape(1, -1)
    if table.shape[1] == 0:
        table = torch.zeros((1, 1), dtype=torch.int32, device=q.device)
    _decode_into(out.unsqueeze(0), q.unsqueeze(0), k_cache, v_cache, table, None, seq_len, scale)
    return out


def paged_attention_decode_v1(
    q: torch.Tensor,            # [num_q_heads, head_dim]
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_table: torch.Tensor,  # 1D int32 cuda tensor of physical block IDs
    seq_len: int,
    scale: float,
) -> torch.Tensor:
    """Single-sequence decode attention (reference paged_attention.py:254-305).

    The reference's v1 makes three passes over K; this build serves v1 and v2
    with the same one-pass kernel (identical mathematics), so v1 == v2 here.
    """
    return _single_sequence(q, k_cache, v_cache, block_table, seq_len, scale)


def paged_attention_decode_v2(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_table: torch.Tensor,
    seq_len: int,
    scale: float,
) -> torch.Tensor:
    """Single-sequence online-softmax decode attention (reference :419-470)."""
    return _single_sequence(q, k_cache, v_cache, block_table, seq_len, scale)


def _raw_lists(block_tables: Sequence[Any]) -> list[list[int]]:
    raw: list[list[int]] = []
    for bt in block_tables:
        if hasattr(bt, "physical_block_ids"):
            raw.append(list(bt.physical_block_ids))
        elif isinstance(bt, (list, tuple)):
            raw.append(list(bt))
        else:
            raise TypeError(f"Unsupported block table type: {type(bt)}")
    return raw


def pad_block_tables(
    block_tables: Sequence[Any],
    device: torch.device | str = "cuda",
) -> torch.Tensor:
    """List of lists (or objects with ``.physical_block_ids``) -> zero-padded
    int32 tensor [num_seqs, max(1, max_len)] on ``device`` (reference :473-505).

    Same result as the reference; built on the host and moved with a single
    copy instead of one device copy per row.
    """
    num_seqs = len(block_tables)
    if num_seqs == 0:
        return torch.empty((0, 0), dtype=torch.int32, device=device)
    raw = _raw_lists(block_tables)
    max_len = max(1, max((len(r) for r in raw), default=0))
    host = torch.zeros((num_seqs, max_len), dtype=torch.int32)
    for i, row in enumerate(raw):
        if row:
            host[i, : len(row)] = torch.tensor(row, dtype=torch.int32)
    dev = torch.device(device)
    if dev.type == "cuda":
        return host.pin_memory().to(dev, non_blocking=True)
    return host.to(dev)


def paged_attention_decode(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: list[list[int]],
    seq_lens: list[int],
    scale: float,
) -> torch.Tensor:
    """The reference's list-based entry (paged_attention.py:86-99), which there
    falls back to the PyTorch reference; here it runs the batched kernel."""
    tables = pad_block_tables(block_tables, device=q.device)
    lens = torch.tensor(list(seq_lens), dtype=torch.int32).to(q.device)
    return paged_attention_decode_batched(q, k_cache, v_cache, tables, lens, scale)


def kv_append(
    k_new: torch.Tensor,        # [num_tokens, num_kv_heads, head_dim]
    v_new: torch.Tensor,        # [num_tokens, num_kv_heads, head_dim]
    k_cache: torch.Tensor,      # [num_blocks, block_size, num_kv_heads, head_dim]
    v_cache: torch.Tensor,
    slot_mapping: torch.Tensor,  # [num_tokens] int64; slot = block_id * block_size + offset
) -> None:
    """Write one layer's new K/V rows into the pool in place, bit-exact.

    Equivalent to ``k_cache[slot // BS, slot % BS] = k_new[i]`` (and V) for
    every token with ``slot >= 0`` — the assignment the reference performs per
    sequence at paged_attention_integration.py:150-160 — in one launch.
    """
    assert k_new.is_cuda and v_new.is_cuda and k_cache.is_cuda and v_cache.is_cuda and slot_mapping.is_cuda
    assert k_cache.dtype in _DTYPES and v_cache.dtype == k_cache.dtype
    assert k_new.dtype == k_cache.dtype and v_new.dtype == k_cache.dtype, "new K/V must match the pool dtype"
    assert slot_mapping.dtype == torch.int64, "slot_mapping must be int64"
    assert k_cache.is_contiguous() and v_cache.is_contiguous(), "KV pool tensors must be contiguous"
    assert v_cache.shape == k_cache.shape
    num_blocks, block_size, num_kv_heads, head_dim = k_cache.shape
    row = (num_kv_heads, head_dim)
    k3 = k_new if k_new.dim() == 3 and k_new.shape[1:] == row else k_new.reshape(-1, num_kv_heads, head_dim)
    v3 = v_new if v_new.dim() == 3 and v_new.shape[1:] == row else v_new.reshape(-1, num_kv_heads, head_dim)
    num_tokens = k3.shape[0]
    assert v3.shape[0] == num_tokens and slot_mapping.numel() == num_tokens, (
        f"k_new/v_new/slot_mapping disagree on the token count ({num_tokens}, {v3.shape[0]}, {slot_mapping.numel()})"
    )
    if num_tokens == 0:
        return
    ks, vs = k3.stride(), v3.stride()
    if ks[2] != 1:
        k3 = k3.contiguous()
        ks = k3.stride()
    if vs[2] != 1:
        v3 = v3.contiguous()
        vs = v3.stride()
    slots = slot_mapping if slot_mapping.dim() == 1 else slot_mapping.reshape(-1)
    if not slots.is_contiguous():
        slots = slots.contiguous()
    rc = _launch(
        k_cache.get_device(), _native.lib().pagedkv_kv_append,
        k_cache.data_ptr(), v_cache.data_ptr(),
        k3.data_ptr(), ks[0], ks[1],
        v3.data_ptr(), vs[0], vs[1],
        slots.data_ptr(), num_tokens, num_kv_heads, head_dim,
        num_blocks, block_size, _DTYPES[k_cache.dtype],
    )
    if rc:
        _native.check(rc, "pagedkv_kv_append")
    if _DEBUG:
        _debug_check(k_cache.device, "kv_append")


# Device arrays of per-layer pool base pointers, keyed by the pointer tuple.
_ptr_tables: dict[tuple, tuple[torch.Tensor, torch.Tensor]] = {}


def _pointer_tables(k_caches: Sequence[torch.Tensor], v_caches: Sequence[torch.Tensor]):
    key = tuple(t.data_ptr() for t in k_caches) + tuple(t.data_ptr() for t in v_caches)
    hit = _ptr_tables.get(key)
    if hit is None:
        dev = k_caches[0].device
        kp = torch.tensor([t.data_ptr() for t in k_caches], dtype=torch.int64).to(dev)
        vp = torch.tensor([t.data_ptr() for t in v_caches], dtype=torch.int64).to(dev)
        if len(_ptr_tables) > 64:
            _ptr_tables.clear()
        hit = (kp, vp)
        _ptr_tables[key] = hit
    return hit


def copy_blocks(
    k_caches: Sequence[torch.Tensor],
    v_caches: Sequence[torch.Tensor],
    block_mapping: torch.Tensor,  # [num_pairs, 2] int64 (src, dst)
) -> None:
    """Copy-on-write block copy: for each (src, dst) pair and every layer,
    ``k_caches[l][dst] = k_caches[l][src]`` and the same for V, in one launch.

    The reference shares blocks by refcount only (block_allocator.py:264-270)
    and asserts it never writes a shared block (integration.py:587-592); this
    is the data copy that lets a writer take a private copy instead.
    Destinations must be distinct and must not be sources in the same call.
    """
    assert len(k_caches) == len(v_caches) and len(k_caches) > 0
    ref = k_caches[0]
    assert ref.is_cuda and block_mapping.is_cuda
    assert block_mapping.dtype == torch.int64 and block_mapping.dim() == 2 and block_mapping.shape[1] == 2
    for t in list(k_caches) + list(v_caches):
        assert t.shape == ref.shape and t.dtype == ref.dtype and t.is_contiguous() and t.device == ref.device
        assert t.data_ptr() % 16 == 0, "pool tensors must start on a 16-byte boundary"
    num_pairs = block_mapping.shape[0]
    if num_pairs == 0:
        return
    mapping = block_mapping if block_mapping.is_contiguous() else block_mapping.contiguous()
    kp, vp = _pointer_tables(k_caches, v_caches)
    block_bytes = ref[0].numel() * ref.element_size()
    rc = _launch(
        ref.get_device(), _native.lib().pagedkv_copy_blocks,
        kp.data_ptr(), vp.data_ptr(), len(k_caches), mapping.data_ptr(), num_pairs,
        block_bytes, ref.shape[0],
    )
    if rc:
        _native.check(rc, "pagedkv_copy_blocks")
    if _DEBUG:
        _debug_check(ref.device, "copy_blocks")


def kv_append_rope(
    q: torch.Tensor,             # [num_tokens, num_q_heads, head_dim]
    k_new: torch.Tensor,         # [num_tokens, num_kv_heads, head_dim]
    v_new: torch.Tensor,         # [num_tokens, num_kv_heads, head_dim]
    cos: torch.Tensor,           # [num_tokens, head_dim] (or [num_tokens, 1, head_dim])
    sin: torch.Tensor,
    k_cache: torch.Tensor,       # [num_blocks, block_size, num_kv_heads, head_dim]
    v_cache: torch.Tensor,
    slot_mapping: torch.Tensor,  # [num_tokens] int64
    q_out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Rotary embedding of q and k fused with the KV append, in one launch.

    Returns ``rope(q)`` (in ``q_out`` when given; it may be ``q`` itself) and
    writes ``rope(k_new)`` / ``v_new`` into the pool slots, with rope(x) =
    ``x * cos + rotate_half(x) * sin`` rounded exactly as transformers'
    ``apply_rotary_pos_emb`` tensor ops (the reference decode forward,
    paged_attention_integration.py:108-109, then the append of :150-160).
    """
    for t in (q, k_new, v_new, cos, sin, k_cache, v_cache, slot_mapping):
        assert t.is_cuda and t.device == k_cache.device
    dt = k_cache.dtype
    assert dt in _DTYPES and v_cache.dtype == dt
    assert q.dtype == dt and k_new.dtype == dt and v_new.dtype == dt and cos.dtype == dt and sin.dtype == dt
    assert slot_mapping.dtype == torch.int64
    assert k_cache.is_contiguous() and v_cache.is_contiguous() and v_cache.shape == k_cache.shape
    num_blocks, block_size, hkv, d = k_cache.shape
    assert d % 16 == 0, "head_dim must be a multiple of 16"
    q3 = q if q.dim() == 3 else q.reshape(q.shape[0], -1, d)
    row = (hkv, d)
    k3 = k_new if k_new.dim() == 3 and k_new.shape[1:] == row else k_new.reshape(-1, hkv, d)
    v3 = v_new if v_new.dim() == 3 and v_new.shape[1:] == row else v_new.reshape(-1, hkv, d)
    n, hq = q3.shape[0], q3.shape[1]
    c2 = cos.reshape(n, d) if cos.dim() != 2 else cos
    s2 = sin.reshape(n, d) if sin.dim() != 2 else sin
    assert k3.shape[0] == n and v3.shape[0] == n and slot_mapping.numel() == n and c2.shape == (n, d)
    if q_out is None:
        q_out = torch.empty((n, hq, d), dtype=dt, device=k_cache.device)
    assert q_out.shape == (n, hq, d) and q_out.dtype == dt and q_out.stride(-1) == 1
    if n == 0:
        return q_out
    fix = lambda t: t if t.stride(-1) == 1 else t.contiguous()
    q3, k3, v3 = fix(q3), fix(k3), fix(v3)
    if c2.stride() != s2.stride() or c2.stride(-1) != 1:
        c2, s2 = c2.contiguous(), s2.contiguous()
    slots = slot_mapping if slot_mapping.dim() == 1 else slot_mapping.reshape(-1)
    if not slots.is_contiguous():
        slots = slots.contiguous()
    qos, qs, ks, vs = q_out.stride(), q3.stride(), k3.stride(), v3.stride()
    rc = _launch(
        k_cache.get_device(), _native.lib().pagedkv_kv_append_rope,
        q_out.data_ptr(), qos[0], qos[1],
        q3.data_ptr(), qs[0], qs[1], hq,
        k_cache.data_ptr(), v_cache.data_ptr(),
        k3.data_ptr(), ks[0], ks[1],
        v3.data_ptr(), vs[0], vs[1],
        c2.data_ptr(), s2.data_ptr(), c2.stride(0),
        slots.data_ptr(), n, hkv, d, num_blocks, block_size, _DTYPES[dt],
    )
    if rc:
        _native.check(rc, "pagedkv_kv_append_rope")
    if _DEBUG:
        _debug_check(k_cache.device, "kv_append_rope")
    return q_out


def kv_write_prefill(
    k_srcs: Sequence[torch.Tensor],
    v_srcs: Sequence[torch.Tensor],
    k_caches: Sequence[torch.Tensor],
    v_caches: Sequence[torch.Tensor],
    block_ids: torch.Tensor,  # [num_write_blocks] int64, on the pools' device
    num_tokens: int,
) -> None:
    """Prefill K/V write into whole blocks, every layer in one launch.

    For layer l, block i and position t: ``k_caches[l][block_ids[i], t] =
    k_srcs[l][i * block_size + t]`` while that index is below ``num_tokens``,
    else zeros (the padded tail of the last block); the same for V. Sources are
    ``[num_tokens, num_kv_heads, head_dim]`` views (any token / head strides,
    last dim contiguous) in the pool dtype or float32 (rounded to nearest even,
    as ``.to()``). Restates ``_copy_prefill_kv``
    (paged_attention_integration.py:278-326: pad + index_copy_ per layer).
    """
    nl = len(k_caches)
    assert nl > 0 and len(v_caches) == nl and len(k_srcs) == nl and len(v_srcs) == nl
    ref = k_caches[0]
    assert ref.is_cuda and ref.dim() == 4, "pools must be CUDA [num_blocks, block_size, kv_heads, head_dim]"
    assert ref.dtype in (torch.float16, torch.bfloat16), "pool dtype must be float16 or bfloat16"
    for t in list(k_caches) + list(v_caches):
        assert t.shape == ref.shape and t.dtype == ref.dtype and t.is_contiguous() and t.device == ref.device
    nb, bs, hkv, d = ref.shape
    src_dtype = k_srcs[0].dtype
    assert src_dtype in (ref.dtype, torch.float32), "source dtype must be the pool dtype or float32"
    ks0, vs0 = k_srcs[0], v_srcs[0]
    for t, t0 in [(t, ks0) for t in k_srcs] + [(t, vs0) for t in v_srcs]:
        assert t.is_cuda and t.device == ref.device and t.dtype == src_dtype
        assert t.dim() == 3 and t.shape[1:] == (hkv, d) and t.shape[0] >= num_tokens
        assert t.stride(2) == 1 and t.stride()[:2] == t0.stride()[:2], "sources share one layout, last dim contiguous"
    assert block_ids.is_cuda and block_ids.device == ref.device and block_ids.dtype == torch.int64 and block_ids.dim() == 1
    nw = block_ids.shape[0]
    assert 0 <= num_tokens <= nw * bs
    if nw == 0:
        return
    ids = block_ids if block_ids.is_contiguous() else block_ids.contiguous()
    arr = ctypes.c_void_p * nl
    kc = arr(*[t.data_ptr() for t in k_caches])
    vc = arr(*[t.data_ptr() for t in v_caches])
    ksrc = arr(*[t.data_ptr() for t in k_srcs])
    vsrc = arr(*[t.data_ptr() for t in v_srcs])
    sd = _native.DTYPE_F32 if src_dtype == torch.float32 else _DTYPES[ref.dtype]
    dev = ref.device
    guard = _device_guard(dev)
    with guard if guard is not None else _NullCtx():
        rc = _native.lib().pagedkv_kv_write_prefill(
            kc, vc, ksrc, vsrc, nl,
            ks0.stride(0), ks0.stride(1), vs0.stride(0), vs0.stride(1), sd,
            ids.data_ptr(), nw, int(num_tokens), hkv, d, nb, bs, _DTYPES[ref.dtype],
            _stream_handle(dev),
        )
    _native.check(rc, "pagedkv_kv_write_prefill")
    _debug_check(dev, "kv_write_prefill")


def _decode_slots(block_tables: torch.Tensor, seq_lens: torch.Tensor, block_size: int) -> torch.Tensor:
    """int64 slot of position len - 1 of every sequence (-1 for length 0),
    computed on the device from the tables and lengths."""
    pos = seq_lens.to(torch.int64) - 1
    p0 = pos.clamp(min=0)
    blk = block_tables.gather(1, (p0 // block_size).view(-1, 1)).view(-1).to(torch.int64)
    return torch.where(pos >= 0, blk * block_size + p0 % block_size, torch.full_like(pos, -1))


def paged_attention_decode_append(
    q: torch.Tensor,             # [num_seqs, num_q_heads, head_dim]
    k_cache: torch.Tensor,       # [num_blocks, block_size, num_kv_heads, head_dim]
    v_cache: torch.Tensor,
    block_tables: torch.Tensor,  # [num_seqs, max_blocks_per_seq] int32
    seq_lens: torch.Tensor,      # [num_seqs] int32, lengths AFTER this step's token
    scale: float,
    k_new: torch.Tensor,         # [num_seqs, num_kv_heads, head_dim]
    v_new: torch.Tensor,
    cos: torch.Tensor | None = None,  # [num_seqs, head_dim] (or [num_seqs, 1, head_dim])
    sin: torch.Tensor | None = None,
    slot_mapping: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """One layer's decode step in ONE launch: the KV append of each sequence's
    new K / V row at position ``seq_len - 1`` of its block table, then batched
    decode attention over the ``seq_len`` tokens (the reference's append,
    paged_attention_integration.py:150-160, followed by its kernel call,
    :164-171). With ``cos`` / ``sin``, q and k are first rotated as
    transformers' ``apply_rotary_pos_emb`` (integration.py:108-109) rounds
    them, as :func:`kv_append_rope` does.

    The pool rows written are bit-identical to :func:`kv_append` /
    :func:`kv_append_rope` at those slots, and the output to
    :func:`paged_attention_decode_batched` on the (rotated) q. Shapes served
    by the CUDA-core kernel (block_size < 8) or unaligned new rows run those
    two operations as separate launches (``slot_mapping``, if given, must be
    the slots of position ``seq_len - 1``; else it is computed on the device).
    ``out`` (optional, [num_seqs, num_q_heads, head_dim] in q's dtype, last
    dimension contiguous) receives the output in place of a new tensor.
    """
    assert q.is_cuda and k_cache.is_cuda and v_cache.is_cuda and block_tables.is_cuda and seq_lens.is_cuda
    assert q.dtype in _DTYPES and k_cache.dtype == q.dtype and v_cache.dtype == q.dtype
    assert k_new.dtype == q.dtype and v_new.dtype == q.dtype
    assert block_tables.dtype == torch.int32 and seq_lens.dtype == torch.int32
    assert k_cache.is_contiguous() and v_cache.is_contiguous() and v_cache.shape == k_cache.shape
    num_seqs, num_q_heads, head_dim = q.shape
    num_blocks, block_size, num_kv_heads, head_dim_k = k_cache.shape
    assert head_dim == head_dim_k, f"Head dimensions must match: {head_dim} vs {head_dim_k}"
    assert num_q_heads % num_kv_heads == 0
    assert block_tables.shape[0] == num_seqs and seq_lens.shape[0] == num_seqs
    row = (num_kv_heads, head_dim)
    k3 = k_new if k_new.dim() == 3 and k_new.shape[1:] == row else k_new.reshape(-1, num_kv_heads, head_dim)
    v3 = v_new if v_new.dim() == 3 and v_new.shape[1:] == row else v_new.reshape(-1, num_kv_heads, head_dim)
    assert k3.shape[0] == num_seqs and v3.shape[0] == num_seqs
    rope = cos is not None
    assert rope == (sin is not None), "pass both cos and sin, or neither"
    if rope:
        c2 = cos.reshape(num_seqs, head_dim) if cos.dim() != 2 else cos
        s2 = sin.reshape(num_seqs, head_dim) if sin.dim() != 2 else sin
        assert c2.dtype == q.dtype and s2.dtype == q.dtype and c2.shape == (num_seqs, head_dim)
        if c2.stride() != s2.stride() or c2.stride(-1) != 1:
            c2, s2 = c2.contiguous(), s2.contiguous()
    if out is None:
        out = torch.empty_like(q)
    else:
        assert out.shape == q.shape and out.dtype == q.dtype and out.device == q.device
    if num_seqs == 0:
        return out
    if block_tables.stride(-1) != 1:
        block_tables = block_tables.contiguous()
    if not seq_lens.is_contiguous():
        seq_lens = seq_lens.contiguous()
    given_out = out
    if not _qo_ok(out):
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    if k3.stride(2) != 1:
        k3 = k3.contiguous()
    if v3.stride(2) != 1:
        v3 = v3.contiguous()
    qq = q if _qo_ok(q) else q.contiguous()
    dtype = _DTYPES[q.dtype]
    max_blocks = block_tables.shape[1]
    idx = q.get_device()
    lib = _native.lib()
    key = (idx, num_seqs, num_q_heads, num_kv_heads, head_dim, block_size, max_blocks, dtype)
    nbytes = _ws_sizes.get(key)
    if nbytes is None:
        nbytes = lib.pagedkv_decode_attention_workspace_size(
            num_seqs, num_q_heads, num_kv_heads, head_dim, block_size, max_blocks, dtype
        )
        _ws_sizes[key] = nbytes
    ws = _workspace(idx, nbytes)
    qs, os_, ks, vs = qq.stride(), out.stride(), k3.stride(), v3.stride()
    rc = _launch(
        idx, lib.pagedkv_decode_attention_append,
        out.data_ptr(), os_[0], os_[1],
        qq.data_ptr(), qs[0], qs[1],
        k_cache.data_ptr(), v_cache.data_ptr(),
        block_tables.data_ptr(), block_tables.stride(0),
        seq_lens.data_ptr(),
        num_seqs, num_q_heads, num_kv_heads, head_dim,
        num_blocks, block_size, max_blocks,
        k3.data_ptr(), ks[0], ks[1],
        v3.data_ptr(), vs[0], vs[1],
        c2.data_ptr() if rope else None, s2.data_ptr() if rope else None, c2.stride(0) if rope else 0,
        float(scale), dtype,
        ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
    )
    if rc == _native.PAGEDKV_ERR_UNSUPPORTED:
        # nothing was launched: the append and the attention as two launches
        slots = slot_mapping if slot_mapping is not None else _decode_slots(block_tables, seq_lens, block_size)
        if rope:
            q_rot = kv_append_rope(q, k3, v3, c2, s2, k_cache, v_cache, slots)
        else:
            kv_append(k3, v3, k_cache, v_cache, slots)
            q_rot = q
        _decode_into(out, q_rot, k_cache, v_cache, block_tables, seq_lens, 0, scale)
    else:
        if rc:
            _native.check(rc, "pagedkv_decode_attention_append")
        if _DEBUG:
            _debug_check(q.device, "paged decode attention + append")
    if out is not given_out:
        given_out.copy_(out)
    return given_out


def last_decode_launch_info() -> tuple[int, str]:
    """(kernel launches, kernel family) of the last decode call on this thread."""
    lib = _native.lib()
    return int(lib.pagedkv_last_decode_launches()), lib.pagedkv_last_decode_kernel().decode()
