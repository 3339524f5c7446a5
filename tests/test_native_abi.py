"""CPU: the C-ABI library loads and exports what include/pagedkv.h declares,
and rejects bad arguments before touching a device."""
import ctypes
import re

import pytest

from pagedkv import _native


def _header_functions() -> list[str]:
    text = _native.HEADER_PATH.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pagedkv_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_header_symbol():
    lib = _native.lib()
    declared = _header_functions()
    assert declared, "no declarations parsed from include/pagedkv.h"
    missing = [name for name in declared if not hasattr(lib, name)]
    assert not missing, f"symbols declared in include/pagedkv.h but not exported: {missing}"
    # the ctypes binding covers exactly the header
    assert sorted(_native.declared_symbols()) == declared


def test_version_string():
    v = _native.lib().pagedkv_version().decode()
    assert v.startswith("pagedkv-b200") and "sm_100a" in v


def _decode(lib, **kw):
    args = dict(
        out=None, os=0, oh=0, q=None, qs=0, qh=0, k=None, v=None, bt=None, bts=0, lens=None, ulen=0,
        n=1, hq=14, hkv=2, d=64, nb=16, bs=16, mb=1, scale=0.125, dtype=0, ws=None, wsb=0, stream=None,
    )
    args.update(kw)
    return lib.pagedkv_decode_attention(*args.values())


def test_decode_rejects_bad_arguments_without_a_device():
    lib = _native.lib()
    assert _decode(lib, n=0) == _native.PAGEDKV_OK  # empty batch is a no-op
    assert _decode(lib, hq=13) == _native.PAGEDKV_ERR_INVALID_ARGUMENT
    assert "multiple of num_kv_heads" in lib.pagedkv_last_error().decode()
    assert _decode(lib, d=80) == _native.PAGEDKV_ERR_UNSUPPORTED
    assert _decode(lib, dtype=7) == _native.PAGEDKV_ERR_UNSUPPORTED
    assert _decode(lib, bs=0) == _native.PAGEDKV_ERR_INVALID_ARGUMENT
    assert _decode(lib) == _native.PAGEDKV_ERR_INVALID_ARGUMENT  # null pointers
    assert _decode(lib, n=-1) == _native.PAGEDKV_ERR_INVALID_ARGUMENT


def test_append_and_copy_reject_bad_arguments_without_a_device():
    lib = _native.lib()
    assert lib.pagedkv_kv_append(None, None, None, 0, 0, None, 0, 0, None, 0, 2, 64, 16, 16, 0, None) == 0
    assert lib.pagedkv_kv_append(None, None, None, 0, 0, None, 0, 0, None, 3, 2, 64, 16, 16, 0, None) == (
        _native.PAGEDKV_ERR_INVALID_ARGUMENT
    )
    assert lib.pagedkv_kv_append(None, None, None, 0, 0, None, 0, 0, None, 3, 2, 64, 16, 16, 5, None) == (
        _native.PAGEDKV_ERR_UNSUPPORTED
    )
    assert lib.pagedkv_copy_blocks(None, None, 1, None, 0, 4096, 8, None) == 0
    assert lib.pagedkv_copy_blocks(None, None, 1, None, 1, 4095, 8, None) == _native.PAGEDKV_ERR_INVALID_ARGUMENT
    assert lib.pagedkv_copy_blocks(None, None, 1, None, 1, 4096, 8, None) == _native.PAGEDKV_ERR_INVALID_ARGUMENT
    assert lib.pagedkv_read_error_flags(None, 0, None) == _native.PAGEDKV_ERR_INVALID_ARGUMENT


def test_append_rope_rejects_bad_arguments_without_a_device():
    lib = _native.lib()
    f = lib.pagedkv_kv_append_rope
    args = [None, 0, 0, None, 0, 0, 14, None, None, None, 0, 0, None, 0, 0, None, None, 0, None]
    assert f(*args, 0, 2, 64, 16, 16, 0, None) == 0  # no tokens
    assert f(*args, 4, 2, 64, 16, 16, 3, None) == _native.PAGEDKV_ERR_UNSUPPORTED  # dtype
    assert f(*args, 4, 2, 72, 16, 16, 0, None) == _native.PAGEDKV_ERR_UNSUPPORTED  # head_dim % 16
    assert f(*args, 4, 2, 64, 16, 16, 0, None) == _native.PAGEDKV_ERR_INVALID_ARGUMENT  # null pointers
    assert f(*args, -1, 2, 64, 16, 16, 0, None) == _native.PAGEDKV_ERR_INVALID_ARGUMENT


def test_prefill_write_rejects_bad_arguments_without_a_device():
    lib = _native.lib()
    f = lib.pagedkv_kv_write_prefill
    # (pool ptrs, srcs, layers, strides, src dtype, ids, blocks, tokens, hkv, d, nb, bs, dtype, stream)
    assert f(None, None, None, None, 0, 0, 0, 0, 0, 0, None, 4, 10, 2, 64, 16, 16, 0, None) == 0  # no layers
    assert f(None, None, None, None, 2, 0, 0, 0, 0, 0, None, 0, 0, 2, 64, 16, 16, 0, None) == 0  # no blocks
    assert f(None, None, None, None, 2, 0, 0, 0, 0, 1, None, 4, 10, 2, 64, 16, 16, 0, None) == (
        _native.PAGEDKV_ERR_UNSUPPORTED  # bf16 source into an f16 pool
    )
    assert f(None, None, None, None, 2, 0, 0, 0, 0, 0, None, 4, 10, 2, 64, 16, 16, 2, None) == (
        _native.PAGEDKV_ERR_UNSUPPORTED  # f32 pool
    )
    assert f(None, None, None, None, 2, 0, 0, 0, 0, 0, None, 2, 33, 2, 64, 16, 16, 0, None) == (
        _native.PAGEDKV_ERR_INVALID_ARGUMENT  # more tokens than the blocks hold
    )
    assert f(None, None, None, None, 2, 0, 0, 0, 0, 0, None, 2, 20, 2, 60, 16, 16, 0, None) == (
        _native.PAGEDKV_ERR_INVALID_ARGUMENT  # head_dim not a multiple of 8
    )
    assert f(None, None, None, None, 2, 0, 0, 0, 0, 2, None, 2, 20, 2, 64, 16, 16, 0, None) == (
        _native.PAGEDKV_ERR_INVALID_ARGUMENT  # null pointers
    )


def test_error_flag_descriptions():
    assert _native.describe_error_flags(0) == "none"
    text = _native.describe_error_flags(_native.EFLAG_BLOCK_ID_RANGE | _native.EFLAG_SLOT_RANGE)
    assert "block-table" in text and "slot" in text


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_native, "_lib", None)
    monkeypatch.setattr(_native, "LIB_PATH", tmp_path / "nope.so")
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _native.lib()


def test_pipeline_timeout_report_rezeroes_the_workspace_flags(monkeypatch):
    """A decode launch that gave up (EFLAG_PIPE_TIMEOUT) may leave cross-CTA
    completion flags set; reading the report zeroes the cached workspace's
    8 KiB flag header and leaves the rest alone (host logic, no device)."""
    import torch

    from pagedkv import paged_attention as pa

    class FakeLib:
        def pagedkv_read_error_flags(self, out_ref, clear, stream):
            out_ref._obj.value = _native.EFLAG_PIPE_TIMEOUT | _native.EFLAG_SLOT_RANGE
            return _native.PAGEDKV_OK

    monkeypatch.setattr(_native, "lib", lambda: FakeLib())
    monkeypatch.setattr(torch.cuda, "current_device", lambda: 0)
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a, **k: None)
    monkeypatch.setattr(pa, "_stream_handle", lambda dev: 0)
    ws = torch.ones(16384, dtype=torch.uint8)
    monkeypatch.setitem(pa._workspaces, 0, ws)
    flags = pa.read_error_flags(0)
    assert flags & _native.EFLAG_PIPE_TIMEOUT and flags & _native.EFLAG_SLOT_RANGE
    assert int(ws[:8192].sum()) == 0 and int(ws[8192:].sum()) == 8192
