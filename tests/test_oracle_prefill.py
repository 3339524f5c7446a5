"""CPU: the prefill-write restatement in oracle/ against the reference's own
KernelPagedManualDecode._copy_prefill_kv (paged_attention_integration.py:278-326),
run here on CPU with a fake model's cache (the reference's prefix-cache test uses
the same construction). Pins the oracle the GPU prefill-write tests check against."""
import sys
from types import SimpleNamespace

import pytest
import torch

from oracle import paged_ref

import refpath

refpath.ensure_on_path()


def _runner_and_cache(num_layers, hkv, d, bs, nb, prompt_len, dtype, src_dtype, seed):
    from engine.kernels.paged_attention_integration import KernelPagedManualDecode

    model = SimpleNamespace(config=SimpleNamespace(num_hidden_layers=num_layers, num_key_value_heads=hkv, head_dim=d))
    runner = KernelPagedManualDecode(model=model, tokenizer=None, block_size=bs, num_blocks=nb, device="cpu", dtype=dtype)
    g = torch.Generator().manual_seed(seed)
    for l in range(num_layers):
        runner.pool.k_cache[l].copy_(torch.randn(runner.pool.k_cache[l].shape, generator=g).to(dtype))
        runner.pool.v_cache[l].copy_(torch.randn(runner.pool.v_cache[l].shape, generator=g).to(dtype))
    pkv = tuple(
        (torch.randn(1, hkv, prompt_len, d, generator=g).to(src_dtype), torch.randn(1, hkv, prompt_len, d, generator=g).to(src_dtype))
        for _ in range(num_layers)
    )
    return runner, pkv


@refpath.requires_reference
@pytest.mark.parametrize(
    "num_layers,hkv,d,bs,nb,prompt_len,skip,dtype,src_dtype",
    [
        (2, 2, 64, 16, 12, 37, 0, torch.float16, torch.float16),
        (3, 2, 64, 16, 12, 37, 1, torch.float16, torch.float32),
        (2, 1, 8, 4, 10, 13, 2, torch.bfloat16, torch.float32),
        (1, 8, 128, 16, 6, 48, 0, torch.bfloat16, torch.bfloat16),
        (2, 2, 64, 16, 8, 16, 1, torch.float16, torch.float16),  # every block a hit: no write
    ],
)
def test_prefill_write_oracle_matches_reference(num_layers, hkv, d, bs, nb, prompt_len, skip, dtype, src_dtype):
    from engine.memory.block_allocator import BlockTable

    runner, pkv = _runner_and_cache(num_layers, hkv, d, bs, nb, prompt_len, dtype, src_dtype, seed=prompt_len + skip)
    nblk = (prompt_len + bs - 1) // bs
    ids = list(range(nb))[::-1][:nblk]  # non-contiguous physical blocks
    table = BlockTable(seq_id=0, block_size=bs, physical_block_ids=ids, num_tokens=prompt_len)
    ours_k = [t.clone() for t in runner.pool.k_cache]
    ours_v = [t.clone() for t in runner.pool.v_cache]
    runner._copy_prefill_kv(pkv, table, prompt_len, skip_blocks=skip)
    start = skip * bs
    if start < prompt_len:
        srcs_k = [pkv[l][0][0, :, start:prompt_len, :].permute(1, 0, 2) for l in range(num_layers)]
        srcs_v = [pkv[l][1][0, :, start:prompt_len, :].permute(1, 0, 2) for l in range(num_layers)]
        paged_ref.prefill_write_ref(ours_k, ours_v, srcs_k, srcs_v, ids[skip:nblk], prompt_len - start)
    for l in range(num_layers):
        assert torch.equal(ours_k[l].view(torch.int16), runner.pool.k_cache[l].view(torch.int16))
        assert torch.equal(ours_v[l].view(torch.int16), runner.pool.v_cache[l].view(torch.int16))
