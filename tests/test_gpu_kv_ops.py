"""GPU parity of the KV append and the copy-on-write block copy (bit-exact)."""
import numpy as np
import pytest
import torch

import cases
import pagedkv
from oracle import paged_ref
from pagedkv import _native

pytestmark = pytest.mark.gpu


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().view(torch.int16).numpy()


@pytest.mark.parametrize("name", list(cases.APPEND_CASES))
def test_append_matches_reference_pool_bit_exact(cuda_ready, golden, name):
    """The pool after kv_append equals, bit for bit, the pool after the
    reference's own decode forward appended the same rows."""
    arrays, manifest = golden
    case = cases.APPEND_CASES[name]
    inp = cases.make_append_inputs(case)
    k_cache = torch.from_numpy(inp["k_cache"]).to(cuda_ready)
    v_cache = torch.from_numpy(inp["v_cache"]).to(cuda_ready)
    slots = torch.from_numpy(paged_ref.decode_slots(inp["tables"], inp["lens"], case["bs"])).to(cuda_ready)
    k_new = torch.from_numpy(arrays[f"{name}__k_new"]).to(cuda_ready)
    v_new = torch.from_numpy(arrays[f"{name}__v_new"]).to(cuda_ready)
    pagedkv.kv_append(k_new, v_new, k_cache, v_cache, slots)
    got = cases.sha256_arrays(k_cache.cpu().numpy(), v_cache.cpu().numpy())
    assert got == manifest["append"][name]["pool_after_sha256"]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(64, 16, 2, 64), (40, 8, 8, 128), (30, 16, 1, 32), (20, 4, 3, 256)])
def test_append_random_vs_oracle(cuda_ready, dtype, shape):
    nb, bs, hkv, d = shape
    g = torch.Generator().manual_seed(sum(shape))
    k_cache = torch.randn(shape, generator=g).to(dtype)
    v_cache = torch.randn(shape, generator=g).to(dtype)
    n = 37
    slots = torch.randperm(nb * bs, generator=g)[:n].to(torch.int64)
    slots[::5] = -1  # padding tokens are skipped
    k_new = torch.randn(n, hkv, d, generator=g).to(dtype)
    v_new = torch.randn(n, hkv, d, generator=g).to(dtype)
    kc, vc = k_cache.to(cuda_ready), v_cache.to(cuda_ready)
    pagedkv.kv_append(k_new.to(cuda_ready), v_new.to(cuda_ready), kc, vc, slots.to(cuda_ready))
    kr, vr = _bits(k_cache).copy(), _bits(v_cache).copy()
    paged_ref.kv_append_ref(kr, vr, _bits(k_new), _bits(v_new), slots.numpy())
    assert np.array_equal(_bits(kc), kr) and np.array_equal(_bits(vc), vr)


def test_append_strided_sources_and_unaligned_head_dim(cuda_ready):
    # k/v rows taken from a fused qkv tensor (strided), and a head_dim (36)
    # whose rows are not 16-byte multiples (scalar path).
    for d in (64, 36):
        nb, bs, hkv = 10, 16, 2
        kc = torch.randn(nb, bs, hkv, d, dtype=torch.float16)
        vc = torch.randn(nb, bs, hkv, d, dtype=torch.float16)
        qkv = torch.randn(9, 14 * d + 2 * hkv * d, dtype=torch.float16)
        k_new = qkv[:, 14 * d : 14 * d + hkv * d].view(9, hkv, d)
        v_new = qkv[:, 14 * d + hkv * d :].view(9, hkv, d)
        slots = torch.tensor([0, 17, 33, 159, 5, 80, 81, 82, -1], dtype=torch.int64)
        kd, vd = kc.to(cuda_ready), vc.to(cuda_ready)
        qkv_d = qkv.to(cuda_ready)
        pagedkv.kv_append(qkv_d[:, 14 * d : 14 * d + hkv * d].view(9, hkv, d),
                          qkv_d[:, 14 * d + hkv * d :].view(9, hkv, d), kd, vd, slots.to(cuda_ready))
        kr, vr = _bits(kc).copy(), _bits(vc).copy()
        paged_ref.kv_append_ref(kr, vr, _bits(k_new.contiguous()), _bits(v_new.contiguous()), slots.numpy())
        assert np.array_equal(_bits(kd), kr) and np.array_equal(_bits(vd), vr)


def test_append_out_of_range_slot_flagged(cuda_ready):
    kc = torch.zeros(4, 16, 2, 64, dtype=torch.float16, device=cuda_ready)
    vc = torch.zeros_like(kc)
    new = torch.ones(2, 2, 64, dtype=torch.float16, device=cuda_ready)
    pagedkv.read_error_flags(cuda_ready, clear=True)
    pagedkv.kv_append(new, new, kc, vc, torch.tensor([3, 4 * 16 + 1], dtype=torch.int64, device=cuda_ready))
    assert pagedkv.read_error_flags(cuda_ready, clear=True) & _native.EFLAG_SLOT_RANGE
    assert kc[0, 3].eq(1).all() and kc.sum().item() == 2 * 64


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_copy_blocks_all_layers_vs_oracle(cuda_ready, dtype):
    layers, nb, bs, hkv, d = 24, 64, 16, 2, 64
    g = torch.Generator().manual_seed(3)
    ks = [torch.randn(nb, bs, hkv, d, generator=g).to(dtype) for _ in range(layers)]
    vs = [torch.randn(nb, bs, hkv, d, generator=g).to(dtype) for _ in range(layers)]
    mapping = torch.tensor([[1, 40], [2, 41], [1, 42], [63, 0], [10, 11]], dtype=torch.int64)
    kd = [t.to(cuda_ready) for t in ks]
    vd = [t.to(cuda_ready) for t in vs]
    pagedkv.copy_blocks(kd, vd, mapping.to(cuda_ready))
    kr = [_bits(t).copy() for t in ks]
    vr = [_bits(t).copy() for t in vs]
    paged_ref.copy_blocks_ref(kr, vr, mapping.numpy())
    for a, b in zip(kd + vd, kr + vr):
        assert np.array_equal(_bits(a), b)


@pytest.mark.parametrize(
    "layers,nb,bs,hkv,d,pairs",
    [
        (3, 32, 3, 1, 8, 7),            # 48-byte blocks: 3 chunks, most lanes idle
        (2, 24, 64, 8, 128, 9),         # 128 KiB blocks: many unrolled rounds per warp
        (1, 8192, 16, 2, 64, 4000),     # more (pair, layer) units than the grid's warps
        (48, 1280, 16, 2, 64, 600),     # 28 800 units over 48 layers
    ],
)
def test_copy_blocks_shapes_and_grid_stride(cuda_ready, layers, nb, bs, hkv, d, pairs):
    g = torch.Generator().manual_seed(layers * 1000 + pairs)
    ks = [torch.randn(nb, bs, hkv, d, generator=g).half() for _ in range(layers)]
    vs = [torch.randn(nb, bs, hkv, d, generator=g).half() for _ in range(layers)]
    perm = torch.randperm(nb, generator=g)
    mapping = torch.stack([perm[:pairs], perm[pairs : 2 * pairs]], dim=1).contiguous()
    kd = [t.to(cuda_ready) for t in ks]
    vd = [t.to(cuda_ready) for t in vs]
    pagedkv.copy_blocks(kd, vd, mapping.to(cuda_ready))
    kr = [_bits(t).copy() for t in ks]
    vr = [_bits(t).copy() for t in vs]
    paged_ref.copy_blocks_ref(kr, vr, mapping.numpy())
    for a, b in zip(kd + vd, kr + vr):
        assert np.array_equal(_bits(a), b)


def test_copy_blocks_out_of_range_flagged(cuda_ready):
    kc = [torch.zeros(4, 16, 2, 64, dtype=torch.float16, device=cuda_ready)]
    vc = [torch.zeros(4, 16, 2, 64, dtype=torch.float16, device=cuda_ready)]
    pagedkv.read_error_flags(cuda_ready, clear=True)
    pagedkv.copy_blocks(kc, vc, torch.tensor([[0, 9]], dtype=torch.int64, device=cuda_ready))
    assert pagedkv.read_error_flags(cuda_ready, clear=True) & _native.EFLAG_COPY_RANGE


def test_copy_blocks_out_of_range_pairs_between_valid_ones(cuda_ready):
    """Out-of-range pairs in the middle of a launch are skipped and flagged;
    every valid pair around them, on every layer, is still copied bit for bit."""
    layers, nb, bs, hkv, d, pairs = 3, 600, 16, 2, 64, 250
    g = torch.Generator().manual_seed(11)
    ks = [torch.randn(nb, bs, hkv, d, generator=g).half() for _ in range(layers)]
    vs = [torch.randn(nb, bs, hkv, d, generator=g).half() for _ in range(layers)]
    perm = torch.randperm(nb, generator=g)
    mapping = torch.stack([perm[:pairs], perm[pairs : 2 * pairs]], dim=1).contiguous()
    bad = [7, 100, 101, 249]
    mapping[7, 0] = nb + 3
    mapping[100, 1] = -2
    mapping[101, 0] = -1
    mapping[249, 1] = nb
    kd = [t.to(cuda_ready) for t in ks]
    vd = [t.to(cuda_ready) for t in vs]
    pagedkv.read_error_flags(cuda_ready, clear=True)
    pagedkv.copy_blocks(kd, vd, mapping.to(cuda_ready))
    assert pagedkv.read_error_flags(cuda_ready, clear=True) & _native.EFLAG_COPY_RANGE
    good = np.array([i for i in range(pairs) if i not in bad])
    kr = [_bits(t).copy() for t in ks]
    vr = [_bits(t).copy() for t in vs]
    paged_ref.copy_blocks_ref(kr, vr, mapping.numpy()[good])
    for a, b in zip(kd + vd, kr + vr):
        assert np.array_equal(_bits(a), b)


def test_pool_larger_than_2gib_uses_64bit_offsets(cuda_ready):
    """A per-layer tensor above 2^31 bytes (config 5 pools are ~1.25 GB per
    tensor; this one is 2.3 GB): append, copy and attend at the far end."""
    nb, bs, hkv, d = 70000, 16, 8, 128  # 32 KiB per block
    kc = torch.zeros(nb, bs, hkv, d, dtype=torch.float16, device=cuda_ready)
    vc = torch.zeros_like(kc)
    assert kc.numel() * 2 > 2**31
    last = nb - 1
    g = torch.Generator(device=cuda_ready).manual_seed(0)
    rows_k = torch.randn(bs, hkv, d, generator=g, device=cuda_ready).half()
    rows_v = torch.randn(bs, hkv, d, generator=g, device=cuda_ready).half()
    slots = torch.arange(last * bs, last * bs + bs, dtype=torch.int64, device=cuda_ready)
    pagedkv.kv_append(rows_k, rows_v, kc, vc, slots)
    assert torch.equal(kc[last], rows_k) and torch.equal(vc[last], rows_v)
    pagedkv.copy_blocks([kc], [vc], torch.tensor([[last, last - 1], [last, 3]], dtype=torch.int64, device=cuda_ready))
    assert torch.equal(kc[last - 1], rows_k) and torch.equal(vc[3], rows_v)
    q = torch.randn(2, 8 * 4, d, generator=g, device=cuda_ready).half()
    tables = torch.tensor([[last - 1, last], [3, last]], dtype=torch.int32, device=cuda_ready)
    lens = torch.tensor([2 * bs, bs + 5], dtype=torch.int32, device=cuda_ready)
    out = pagedkv.paged_attention_decode_batched(q, kc, vc, tables, lens, d ** -0.5)
    k_small = torch.stack([kc[last - 1], kc[last], kc[3]]).cpu().float()
    v_small = torch.stack([vc[last - 1], vc[last], vc[3]]).cpu().float()
    ref = paged_ref.paged_attention_ref(q.cpu().float(), k_small, v_small, [[0, 1], [2, 1]], lens.tolist(), d ** -0.5)
    torch.testing.assert_close(out.float().cpu(), ref, atol=2e-3, rtol=2e-3)
    del kc, vc
    torch.cuda.empty_cache()
