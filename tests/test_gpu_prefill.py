"""GPU parity of the prefill K/V write (bit-exact vs the oracle restatement of
_copy_prefill_kv, which tests/test_oracle_prefill.py pins to the reference)."""
from types import SimpleNamespace

import pytest
import torch

import pagedkv
from oracle import paged_ref
from pagedkv import _native, integration

pytestmark = pytest.mark.gpu


def _pools(num_layers, shape, dtype, g):
    return ([torch.randn(shape, generator=g).to(dtype) for _ in range(num_layers)],
            [torch.randn(shape, generator=g).to(dtype) for _ in range(num_layers)])


def _check(dev, num_layers, shape, dtype, src_dtype, prompt_len, skip, misalign=False, seed=0):
    nb, bs, hkv, d = shape
    g = torch.Generator().manual_seed(seed)
    kc, vc = _pools(num_layers, shape, dtype, g)
    # HF cache layout [1, kv_heads, tokens, head_dim]; the write reads tokens
    # [skip * bs, prompt_len) through a permuted (strided) view
    full_k = [torch.randn(1, hkv, prompt_len + (1 if misalign else 0), d, generator=g).to(src_dtype) for _ in range(num_layers)]
    full_v = [torch.randn(1, hkv, prompt_len + (1 if misalign else 0), d, generator=g).to(src_dtype) for _ in range(num_layers)]
    nblk = (prompt_len + bs - 1) // bs
    ids = torch.randperm(nb, generator=g)[:nblk].tolist()
    start = skip * bs
    sl = slice(start + (1 if misalign else 0), prompt_len + (1 if misalign else 0))
    srcs_k = [t[0, :, sl, :].permute(1, 0, 2) for t in full_k]
    srcs_v = [t[0, :, sl, :].permute(1, 0, 2) for t in full_v]
    exp_k = [t.clone() for t in kc]
    exp_v = [t.clone() for t in vc]
    paged_ref.prefill_write_ref(exp_k, exp_v, srcs_k, srcs_v, ids[skip:nblk], prompt_len - start)
    gk = [t.to(dev) for t in kc]
    gv = [t.to(dev) for t in vc]
    pagedkv.kv_write_prefill([t.to(dev)[0, :, sl, :].permute(1, 0, 2) for t in full_k],
                             [t.to(dev)[0, :, sl, :].permute(1, 0, 2) for t in full_v],
                             gk, gv, torch.tensor(ids[skip:nblk], dtype=torch.int64, device=dev), prompt_len - start)
    for a, b in zip(gk + gv, exp_k + exp_v):
        assert torch.equal(a.cpu().view(torch.int16), b.view(torch.int16))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("src", ["same", "f32"])
@pytest.mark.parametrize("shape,prompt_len,skip", [((24, 16, 2, 64), 37, 0), ((24, 16, 2, 64), 37, 1),
                                                   ((16, 8, 8, 128), 64, 2), ((40, 4, 1, 32), 13, 1)])
def test_prefill_write_vs_oracle(cuda_ready, dtype, src, shape, prompt_len, skip):
    _check(cuda_ready, 3, shape, dtype, dtype if src == "same" else torch.float32, prompt_len, skip,
           seed=prompt_len * 7 + skip)


def test_prefill_write_many_layers_and_unaligned_sources(cuda_ready):
    # 50 layers take two launches; a source view starting one element in is
    # not 16-byte aligned (element-wise path)
    _check(cuda_ready, 50, (12, 16, 2, 64), torch.float16, torch.float16, 40, 0, seed=1)
    _check(cuda_ready, 2, (12, 16, 2, 64), torch.float16, torch.float16, 40, 1, misalign=True, seed=2)
    _check(cuda_ready, 2, (12, 16, 2, 64), torch.bfloat16, torch.float32, 40, 0, misalign=True, seed=3)


def test_prefill_write_flags_bad_block_ids(cuda_ready):
    pagedkv.read_error_flags(cuda_ready, clear=True)
    kc = [torch.zeros(4, 16, 2, 64, dtype=torch.float16, device=cuda_ready)]
    vc = [torch.zeros(4, 16, 2, 64, dtype=torch.float16, device=cuda_ready)]
    src = torch.ones(32, 2, 64, dtype=torch.float16, device=cuda_ready)
    ids = torch.tensor([1, 9], dtype=torch.int64, device=cuda_ready)  # 9 is out of range
    pagedkv.kv_write_prefill([src], [src], kc, vc, ids, 32)
    assert pagedkv.read_error_flags(cuda_ready, clear=True) & _native.EFLAG_BLOCK_ID_RANGE
    assert torch.all(kc[0][1] == 1) and torch.all(kc[0][0] == 0) and torch.all(kc[0][2:] == 0)


def _fake_runner(dev, num_layers, shape, dtype, g):
    kc, vc = _pools(num_layers, shape, dtype, g)
    return SimpleNamespace(block_size=shape[1], pool=SimpleNamespace(k_cache=[t.to(dev) for t in kc],
                                                                     v_cache=[t.to(dev) for t in vc])), kc, vc


@pytest.mark.parametrize("layout", ["tuple", "layers"])
def test_copy_prefill_kv_drop_in(cuda_ready, layout):
    """integration.copy_prefill_kv (the patched _copy_prefill_kv) leaves prefix
    hit blocks alone and writes the owned blocks like the reference method."""
    g = torch.Generator().manual_seed(11)
    shape = (10, 16, 2, 64)
    runner, kc, vc = _fake_runner(cuda_ready, 2, shape, torch.float16, g)
    prompt_len, skip = 45, 1
    keys = [torch.randn(1, 2, prompt_len, 64, generator=g).half() for _ in range(2)]
    vals = [torch.randn(1, 2, prompt_len, 64, generator=g).half() for _ in range(2)]
    dk = [t.to(cuda_ready) for t in keys]
    dv = [t.to(cuda_ready) for t in vals]
    if layout == "tuple":
        pkv = tuple(zip(dk, dv))
    else:
        pkv = SimpleNamespace(layers=[SimpleNamespace(keys=k, values=v) for k, v in zip(dk, dv)])
    table = SimpleNamespace(physical_block_ids=[7, 2, 5], num_tokens=prompt_len)
    integration.copy_prefill_kv(runner, pkv, table, prompt_len, skip_blocks=skip)
    exp_k = [t.clone() for t in kc]
    exp_v = [t.clone() for t in vc]
    paged_ref.prefill_write_ref(exp_k, exp_v, [t[0, :, 16:, :].permute(1, 0, 2) for t in keys],
                                [t[0, :, 16:, :].permute(1, 0, 2) for t in vals], [2, 5], prompt_len - 16)
    for a, b in zip(runner.pool.k_cache + runner.pool.v_cache, exp_k + exp_v):
        assert torch.equal(a.cpu().view(torch.int16), b.view(torch.int16))
    assert torch.equal(runner.pool.k_cache[0][7].cpu(), kc[0][7])  # the hit block is untouched
