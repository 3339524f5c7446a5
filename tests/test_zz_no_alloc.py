"""GPU: the decode-attention entry point that allocates nothing.

Some callers cannot allocate device memory while they decode (a memory budget
fixed at start-up, an allocator owned by someone else, a binding without an
allocator). pagedkv_decode_attention_noalloc serves them from a fixed scratch
array inside the library. This file is collected last on purpose, and each
test must pass both alone in a fresh process and after every other test.
"""
import ctypes
import math

import pytest
import torch

import pagedkv
from oracle import paged_ref
from pagedkv import _native

pytestmark = pytest.mark.gpu

ATOL = 2e-3
RTOL = 2e-3


def _case(seed, n, hq, hkv, d, bs, lens, dev):
    g = torch.Generator().manual_seed(seed)
    need = [max(1, (x + bs - 1) // bs) for x in lens]
    nb = sum(need) + 7
    perm = torch.randperm(nb, generator=g)
    tables = torch.zeros(n, max(need), dtype=torch.int32)
    at = 0
    for i, c in enumerate(need):
        tables[i, :c] = perm[at : at + c].to(torch.int32)
        at += c
    q = torch.randn(n, hq, d, generator=g).half().to(dev)
    k = torch.randn(nb, bs, hkv, d, generator=g).half().to(dev)
    v = torch.randn(nb, bs, hkv, d, generator=g).half().to(dev)
    return q, k, v, tables.to(dev), torch.tensor(lens, dtype=torch.int32, device=dev)


def _noalloc(out, q, k, v, tables, lens, scale):
    lib = _native.lib()
    rc = lib.pagedkv_decode_attention_noalloc(
        out.data_ptr(), out.stride(0), out.stride(1),
        q.data_ptr(), q.stride(0), q.stride(1),
        k.data_ptr(), v.data_ptr(),
        tables.data_ptr(), tables.stride(0),
        lens.data_ptr(), 0,
        q.shape[0], q.shape[1], k.shape[2], q.shape[2],
        k.shape[0], k.shape[1], tables.shape[1],
        ctypes.c_float(scale), _native.DTYPE_F16,
        torch.cuda.current_stream().cuda_stream,
    )
    return rc


@pytest.mark.parametrize(
    "shape",
    [
        (256, 14, 2, 64, 16, "cfg2"),    # tensor-core path, cut segments combined across CTAs
        (6, 56, 8, 128, 16, "varlen"),   # tensor-core path, head_dim 128, ragged lengths
        (5, 8, 4, 64, 4, "simt"),        # CUDA-core split-K path (block_size 4)
    ],
)
def test_noalloc_matches_oracle_and_workspace_entry_point_twice(shape):
    assert torch.cuda.is_available(), "GPU test selected but no CUDA device is visible"
    dev = torch.device("cuda", 0)
    n, hq, hkv, d, bs, kind = shape
    if kind == "cfg2":
        lens = [2048] * n
    elif kind == "varlen":
        lens = [1, 130, 4097, 777, 0, 2600]
    else:
        lens = [3, 700, 1500, 16, 2049]
    q, k, v, tables, lens_t = _case(7, n, hq, hkv, d, bs, lens, dev)
    scale = 1.0 / math.sqrt(d)
    ref = pagedkv.paged_attention_decode_batched(q, k, v, tables, lens_t, scale)
    # the fp32 CPU oracle (the reference's naive_reference_paged_attention restated)
    rows = [tables[i, : (x + bs - 1) // bs].tolist() for i, x in enumerate(lens)]
    expected = paged_ref.paged_attention_ref(q.float().cpu(), k.float().cpu(), v.float().cpu(), rows, lens, scale)
    for _ in range(2):  # the shared scratch keeps the previous call's contents
        out = torch.full_like(q, float("nan"))
        rc = _noalloc(out, q, k, v, tables, lens_t, scale)
        assert rc == _native.PAGEDKV_OK, _native.lib().pagedkv_last_error().decode()
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float().cpu(), ref.float().cpu(), atol=ATOL, rtol=RTOL)
        torch.testing.assert_close(out.float().cpu(), expected, atol=ATOL, rtol=RTOL)
    assert pagedkv.read_error_flags(dev) == 0


def test_noalloc_rejects_shapes_beyond_its_scratch():
    assert torch.cuda.is_available(), "GPU test selected but no CUDA device is visible"
    dev = torch.device("cuda", 0)
    # One long sequence on the CUDA-core split-K path (block_size 4): it is
    # split into ~1200 chunks whose partials need ~9.8 MB, beyond the 4 MiB.
    n, hq, hkv, d, bs, width = 1, 8, 1, 256, 4, 75776
    q = torch.zeros(n, hq, d, dtype=torch.half, device=dev)
    k = torch.zeros(64, bs, hkv, d, dtype=torch.half, device=dev)
    tables = torch.zeros(n, width, dtype=torch.int32, device=dev)
    lens = torch.full((n,), width * bs, dtype=torch.int32, device=dev)
    need = _native.lib().pagedkv_decode_attention_workspace_size(n, hq, hkv, d, bs, width, 0)
    assert need > (4 << 20)
    out = torch.empty_like(q)
    rc = _noalloc(out, q, k, k, tables, lens, 0.1)
    assert rc == _native.PAGEDKV_ERR_WORKSPACE
    assert "more than the fixed" in _native.lib().pagedkv_last_error().decode()
