"""GPU: decode attention with the KV append (and RoPE) fused into one launch.

``pagedkv.paged_attention_decode_append`` (C entry
``pagedkv_decode_attention_append``) writes each sequence's new K / V row at
position seq_len - 1 of its block table inside the tensor-core decode launch,
then attends over the seq_len tokens. It must equal, bit for bit, the two
operations it replaces run as separate launches (``kv_append`` or
``kv_append_rope``, then ``paged_attention_decode_batched``): the same pool
rows and the same output. And against the fp32 oracle (the reference's
naive_reference_paged_attention restated, engine/kernels/paged_attention.py
:30-83, after the reference's append at paged_attention_integration.py
:150-160), the output is within the north star's 2e-3.
"""
from __future__ import annotations

import ctypes
import math
import random

import numpy as np
import pytest
import torch

import pagedkv
from oracle import paged_ref
from pagedkv import _native

pytestmark = pytest.mark.gpu

ATOL = 2e-3
RTOL = 2e-3


def _case(seed, hq, hkv, d, bs, lens, dtype=torch.float16, q_scale=1.0):
    g = torch.Generator().manual_seed(seed)
    need = [max(1, (x + bs - 1) // bs) for x in lens]
    nb = sum(need) + 9
    perm = list(range(nb))
    random.Random(seed).shuffle(perm)
    rows, at = [], 0
    for c in need:
        rows.append(perm[at : at + c])
        at += c
    tables = torch.zeros(len(lens), max(need), dtype=torch.int32)
    for i, r in enumerate(rows):
        tables[i, : len(r)] = torch.tensor(r, dtype=torch.int32)
    n = len(lens)
    q = (torch.randn(n, hq, d, generator=g) * q_scale).to(dtype)
    k = torch.randn(nb, bs, hkv, d, generator=g).to(dtype)
    v = torch.randn(nb, bs, hkv, d, generator=g).to(dtype)
    k_new = torch.randn(n, hkv, d, generator=g).to(dtype)
    v_new = torch.randn(n, hkv, d, generator=g).to(dtype)
    # rotary tables as transformers builds them: cat(freqs, freqs) at each position
    inv = 1.0 / (1000000.0 ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
    pos = torch.tensor([max(0, x - 1) for x in lens], dtype=torch.float32)
    emb = torch.cat([pos[:, None] * inv[None], pos[:, None] * inv[None]], dim=-1)
    cos, sin = emb.cos().to(dtype), emb.sin().to(dtype)
    return dict(q=q, k=k, v=v, tables=tables, rows=rows, lens=lens, k_new=k_new, v_new=v_new, cos=cos, sin=sin)


def _run(c, dev, rope):
    """(fused out, fused pools, unfused out, unfused pools)."""
    lens_d = torch.tensor(c["lens"], dtype=torch.int32, device=dev)
    tables_d = c["tables"].to(dev)
    scale = 1.0 / math.sqrt(c["q"].shape[-1])
    bs = c["k"].shape[1]
    slots = torch.from_numpy(paged_ref.decode_slots(c["rows"], c["lens"], bs)).to(dev)
    q, kn, vn = c["q"].to(dev), c["k_new"].to(dev), c["v_new"].to(dev)
    cos, sin = (c["cos"].to(dev), c["sin"].to(dev)) if rope else (None, None)
    kf, vf = c["k"].to(dev), c["v"].to(dev)
    out_f = pagedkv.paged_attention_decode_append(q, kf, vf, tables_d, lens_d, scale, kn, vn, cos, sin)
    ku, vu = c["k"].to(dev), c["v"].to(dev)
    if rope:
        q_rot = pagedkv.kv_append_rope(q, kn, vn, cos, sin, ku, vu, slots)
    else:
        pagedkv.kv_append(kn, vn, ku, vu, slots)
        q_rot = q
    out_u = pagedkv.paged_attention_decode_batched(q_rot, ku, vu, tables_d, lens_d, scale)
    return out_f, kf, vf, out_u, ku, vu, q_rot, scale


SHAPES = [
    # (hq, hkv, head_dim, block_size, lens)
    (14, 2, 64, 16, [1, 16, 17, 300, 2048, 0, 129]),   # Qwen2.5-0.5B heads, a zero-length sequence
    (8, 8, 128, 16, [5, 128, 4097, 777]),              # config 3 shape, G 1
    (56, 8, 128, 16, [33, 1000, 2600]),                # G 7 at head_dim 128
    (40, 2, 64, 32, [70, 900, 2049]),                  # G 20: query-head chunks re-read one tile row
    (12, 4, 32, 8, [3, 8, 9, 515]),                    # head_dim 32: four kv heads per tile row
    (16, 8, 256, 16, [17, 2048, 1]),                   # head_dim 256: two sub-rows per head
    (14, 2, 64, 64, [63, 64, 65, 1500]),               # 64-token blocks
]


@pytest.mark.parametrize("rope", [False, True])
@pytest.mark.parametrize("shape", SHAPES)
def test_fused_append_equals_separate_launches_and_oracle(cuda_ready, shape, rope):
    hq, hkv, d, bs, lens = shape
    c = _case(hash((hq, hkv, d, bs)) % 10000, hq, hkv, d, bs, lens)
    out_f, kf, vf, out_u, ku, vu, q_rot, scale = _run(c, cuda_ready, rope)
    assert pagedkv.last_decode_launch_info() == (1, "tc")
    torch.cuda.synchronize()
    # bit-identical pools and output
    assert torch.equal(kf, ku) and torch.equal(vf, vu)
    assert torch.equal(out_f, out_u)
    # against the fp32 oracle on the appended pool
    ref = paged_ref.paged_attention_ref(q_rot.float().cpu(), ku.float().cpu(), vu.float().cpu(), c["rows"],
                                        c["lens"], scale)
    torch.testing.assert_close(out_f.float().cpu(), ref, atol=ATOL, rtol=RTOL)
    # the appended rows are the new ones (K rotated when RoPE is on)
    slots = paged_ref.decode_slots(c["rows"], c["lens"], bs)
    kr, vr = c["k"].numpy().copy(), c["v"].numpy().copy()
    k_rows = paged_ref.rope_ref(c["k_new"], c["cos"], c["sin"]).numpy() if rope else c["k_new"].numpy()
    paged_ref.kv_append_ref(kr, vr, k_rows, c["v_new"].numpy(), slots)
    assert np.array_equal(kf.cpu().numpy(), kr) and np.array_equal(vf.cpu().numpy(), vr)
    assert pagedkv.read_error_flags(cuda_ready) == 0


def test_fused_append_bf16(cuda_ready):
    c = _case(5, 14, 2, 64, 16, [40, 700, 2048], dtype=torch.bfloat16)
    out_f, kf, vf, out_u, ku, vu, _, _ = _run(c, cuda_ready, True)
    assert torch.equal(kf, ku) and torch.equal(vf, vu) and torch.equal(out_f, out_u)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(14, 2, 64, 16, [33, 700, 129]), (16, 8, 256, 16, [17, 300])])
def test_fused_rope_rounding_at_extreme_magnitudes(cuda_ready, shape, dtype):
    """Q and the new K row scaled element-wise by powers of two down to the
    16-bit subnormals (and, for bf16, products below fp32's normal range),
    with some cos / sin entries tiny as well: the in-kernel rotation still
    equals transformers' op sequence bit for bit (the pool row against the
    oracle, the output against the separate RoPE + append launches)."""
    hq, hkv, d, bs, lens = shape
    c = _case(11, hq, hkv, d, bs, lens, dtype=dtype)
    g = torch.Generator().manual_seed(12)
    lo_exp = -30 if dtype == torch.float16 else -130

    def spread(x):
        e = torch.randint(lo_exp, 1, x.shape, generator=g).float()
        return (x.float() * torch.pow(2.0, e)).to(dtype)

    c["q"], c["k_new"] = spread(c["q"]), spread(c["k_new"])
    tiny = torch.rand(c["sin"].shape, generator=g) < 0.25
    c["sin"] = torch.where(tiny, spread(c["sin"]), c["sin"])
    c["cos"] = torch.where(~tiny, spread(c["cos"]), c["cos"])
    out_f, kf, vf, out_u, ku, vu, _, _ = _run(c, cuda_ready, True)
    torch.cuda.synchronize()
    assert torch.equal(kf, ku) and torch.equal(vf, vu)
    assert torch.equal(out_f, out_u)
    slots = paged_ref.decode_slots(c["rows"], c["lens"], bs)
    kr, vr = c["k"].clone(), c["v"].clone()
    k_rows = paged_ref.rope_ref(c["k_new"], c["cos"], c["sin"])
    paged_ref.kv_append_ref(kr.view(torch.int16).numpy(), vr.view(torch.int16).numpy(),
                            k_rows.view(torch.int16).numpy(), c["v_new"].view(torch.int16).numpy(), slots)
    assert torch.equal(kf.cpu().view(torch.int16), kr.view(torch.int16))
    assert torch.equal(vf.cpu().view(torch.int16), vr.view(torch.int16))
    assert pagedkv.read_error_flags(cuda_ready) == 0


def test_fused_append_config2_full_size(cuda_ready):
    """256 x 2048 tokens, 40960-block pool, the append of
    the 2048th token fused into the attention."""
    n, hq, hkv, d, bs, ctx = 256, 14, 2, 64, 16, 2048
    g = torch.Generator().manual_seed(22)
    nb = 40960
    perm = list(range(nb))
    random.Random(22).shuffle(perm)
    rows = [perm[i * 128 : (i + 1) * 128] for i in range(n)]
    tables = torch.tensor(rows, dtype=torch.int32)
    q = torch.randn(n, hq, d, generator=g).half()
    k = torch.randn(nb, bs, hkv, d, generator=g).half()
    v = torch.randn(nb, bs, hkv, d, generator=g).half()
    kn = torch.randn(n, hkv, d, generator=g).half()
    vn = torch.randn(n, hkv, d, generator=g).half()
    dev = cuda_ready
    kd, vd = k.to(dev), v.to(dev)
    out = pagedkv.paged_attention_decode_append(q.to(dev), kd, vd, tables.to(dev),
                                                torch.full((n,), ctx, dtype=torch.int32, device=dev), 0.125,
                                                kn.to(dev), vn.to(dev))
    slots = paged_ref.decode_slots(rows, [ctx] * n, bs)
    kr, vr = k.numpy().copy(), v.numpy().copy()
    paged_ref.kv_append_ref(kr, vr, kn.numpy(), vn.numpy(), slots)
    assert np.array_equal(kd.cpu().numpy(), kr) and np.array_equal(vd.cpu().numpy(), vr)
    ref = paged_ref.paged_attention_ref(q.float(), torch.from_numpy(kr).float(), torch.from_numpy(vr).float(),
                                        rows, [ctx] * n, 0.125)
    torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)


def test_cuda_core_shapes_and_unaligned_rows_run_as_two_launches(cuda_ready):
    """block_size 4 runs on the CUDA-core kernel, which has no fused append:
    the C entry refuses before launching anything, and the Python op runs the
    append and the attention separately with the same results. Unaligned new
    rows take the same route."""
    dev = cuda_ready
    c = _case(9, 8, 2, 64, 4, [3, 17, 400])
    lens_d = torch.tensor(c["lens"], dtype=torch.int32, device=dev)
    q, kd, vd = c["q"].to(dev), c["k"].to(dev), c["v"].to(dev)
    kn, vn = c["k_new"].to(dev), c["v_new"].to(dev)
    out = torch.empty_like(q)
    rc = _native.lib().pagedkv_decode_attention_append(
        out.data_ptr(), out.stride(0), out.stride(1), q.data_ptr(), q.stride(0), q.stride(1),
        kd.data_ptr(), vd.data_ptr(), c["tables"].to(dev).data_ptr(), c["tables"].shape[1], lens_d.data_ptr(),
        3, 8, 2, 64, kd.shape[0], 4, c["tables"].shape[1],
        kn.data_ptr(), kn.stride(0), kn.stride(1), vn.data_ptr(), vn.stride(0), vn.stride(1),
        None, None, 0, ctypes.c_float(0.125), _native.DTYPE_F16, None, 0, torch.cuda.current_stream().cuda_stream)
    assert rc == _native.PAGEDKV_ERR_UNSUPPORTED
    assert torch.equal(kd, c["k"].to(dev))  # nothing was written
    for case, rope in ((c, False), (_case(10, 14, 2, 64, 16, [20, 300]), True)):
        if case is not c:
            # new K rows at an odd element offset: not 16-byte aligned
            big = torch.zeros(case["k_new"].numel() + 1, dtype=torch.float16)
            big[1:] = case["k_new"].reshape(-1)
            kn_odd = big.to(dev)[1:].view(case["k_new"].shape)
            assert kn_odd.data_ptr() % 16 != 0
            case = dict(case, k_new=kn_odd)  # stays a device view: .to(dev) keeps it
        out_f, kf, vf, out_u, ku, vu, _, _ = _run(case, dev, rope)
        assert torch.equal(kf, ku) and torch.equal(vf, vu) and torch.equal(out_f, out_u)


@pytest.mark.parametrize("rope", [False, True])
@pytest.mark.parametrize("lens", [[0, 0, 0, 0], [1], [0, 5, 0], [3000]])
def test_fused_append_batches_that_leave_ctas_without_work(cuda_ready, lens, rope):
    """Batches whose tiles do not reach every CTA of the launch (all padding
    rows, one token, a single long sequence): the idle CTAs must read nothing,
    and the result is still the two separate launches'."""
    c = _case(31 + len(lens) + sum(lens), 14, 2, 64, 16, lens)
    out_f, kf, vf, out_u, ku, vu, _, _ = _run(c, cuda_ready, rope)
    torch.cuda.synchronize()
    assert torch.equal(kf, ku) and torch.equal(vf, vu) and torch.equal(out_f, out_u)
    assert pagedkv.read_error_flags(cuda_ready) == 0


def test_fused_append_writes_into_a_given_output(cuda_ready):
    """``out=`` receives the result in place of a new tensor (a row of a
    larger buffer, as a caller batching several layers' outputs passes it)."""
    c = _case(77, 14, 2, 64, 16, [40, 700, 2048])
    dev = cuda_ready
    out_f, _, _, _, _, _, _, _ = _run(c, dev, False)
    buf = torch.full((3,) + tuple(c["q"].shape), float("nan"), dtype=torch.float16, device=dev)
    kf, vf = c["k"].to(dev), c["v"].to(dev)
    got = pagedkv.paged_attention_decode_append(
        c["q"].to(dev), kf, vf, c["tables"].to(dev), torch.tensor(c["lens"], dtype=torch.int32, device=dev),
        1.0 / 8, c["k_new"].to(dev), c["v_new"].to(dev), out=buf[1])
    assert got.data_ptr() == buf[1].data_ptr()
    assert torch.equal(buf[1], out_f)
    assert torch.isnan(buf[0]).all() and torch.isnan(buf[2]).all()
