"""GPU parity at the BASELINE configurations that share or skew K/V.

* Config 3 at its full batch: 128 sequences, head_dim 128, 8 kv heads, GQA
  G in {1, 2, 4, 7}, lengths log-uniform in [16, 8192], q x30 (large scores).
* Config 4 as stated: 512 sequences in 8 groups of 64; each group's tables
  share one 1024-token prefix (the same 64 block ids, ref count 64), then 256
  tokens of the sequence's own; one decode step = KV append of the 1280th token
  + attention over 1280 tokens.
* Config 4 with copy-on-write: each group's last block is shared and partially
  filled (15 of 16 rows, ref count 64 in the reference's BlockAllocator) when
  the step starts; the step runs copy-on-write bookkeeping
  (pagedkv.integration.prepare_copy_on_write) -> one copy_blocks launch over
  24 layers -> KV append -> attention, and is checked against the oracle
  running the same three operations on the CPU (pool bit-exact, attention
  within 2e-3).

The attention bar is the north star's: fp16 output within 2e-3 abs + 2e-3 rel
of the fp32 oracle (oracle/paged_ref.py, pinned to the reference's
naive_reference_paged_attention, engine/kernels/paged_attention.py:30-83).
The mirrored reference case for batched shared tables is
tests/test_paged_attention_reference.py:540-643.
"""
from __future__ import annotations

import math
import random

import numpy as np
import pytest
import torch

import pagedkv
import refpath
from oracle import paged_ref

pytestmark = pytest.mark.gpu

ATOL = 2e-3
RTOL = 2e-3


def _oracle_check(out, q, k, v, rows, lens, scale):
    ref = paged_ref.paged_attention_ref(q.float(), k.float(), v.float(), rows, lens, scale)
    torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("gqa", [1, 2, 4, 7])
def test_config3_full_batch_vs_oracle(cuda_ready, gqa):
    n, hkv, d, bs = 128, 8, 128, 16
    hq = hkv * gqa
    rng = np.random.default_rng(3000 + gqa)
    lens = [int(round(math.exp(x))) for x in rng.uniform(math.log(16), math.log(8192), n)]
    need = [(x + bs - 1) // bs for x in lens]
    nb = sum(need) + 64
    perm = list(range(nb))
    random.Random(43 + gqa).shuffle(perm)
    rows, at = [], 0
    for c in need:
        rows.append(perm[at : at + c])
        at += c
    tables = torch.zeros(n, max(need), dtype=torch.int32)
    for i, r in enumerate(rows):
        tables[i, : len(r)] = torch.tensor(r, dtype=torch.int32)
    g = torch.Generator().manual_seed(1100 + gqa)
    q = (torch.randn(n, hq, d, generator=g) * 30.0).half()
    k = torch.randn(nb, bs, hkv, d, generator=g).half()
    v = torch.randn(nb, bs, hkv, d, generator=g).half()
    dev = cuda_ready
    out = pagedkv.paged_attention_decode_batched(q.to(dev), k.to(dev), v.to(dev), tables.to(dev),
                                                 torch.tensor(lens, dtype=torch.int32, device=dev), 1 / math.sqrt(d))
    _oracle_check(out, q, k, v, rows, lens, 1 / math.sqrt(d))
    assert pagedkv.read_error_flags(dev) == 0


def _config4_tables(seed, groups=8, per_group=64, prefix_blocks=64, own_blocks=16, spare=64):
    """Block lists of config 4: group g's sequences share ``prefix_blocks``
    block ids, then own ``own_blocks`` blocks each. Returns (rows, num_blocks)."""
    n = groups * per_group
    nb = groups * prefix_blocks + n * own_blocks + spare
    perm = list(range(nb))
    random.Random(seed).shuffle(perm)
    at = 0
    prefixes = []
    for _ in range(groups):
        prefixes.append(perm[at : at + prefix_blocks])
        at += prefix_blocks
    rows = []
    for s in range(n):
        rows.append(prefixes[s // per_group] + perm[at : at + own_blocks])
        at += own_blocks
    return rows, nb, perm[at:]


def test_config4_shared_prefix_append_and_attention_vs_oracle(cuda_ready):
    hq, hkv, d, bs, ctx = 14, 2, 64, 16, 1280
    rows, nb, _ = _config4_tables(44)
    n = len(rows)
    assert n == 512 and all(len(r) == 80 for r in rows)
    assert len({tuple(r[:64]) for r in rows}) == 8  # 8 prefixes, each shared by 64 tables
    g = torch.Generator().manual_seed(1200)
    q = torch.randn(n, hq, d, generator=g).half()
    k_new = torch.randn(n, hkv, d, generator=g).half()
    v_new = torch.randn(n, hkv, d, generator=g).half()
    k = torch.randn(nb, bs, hkv, d, generator=g).half()
    v = torch.randn(nb, bs, hkv, d, generator=g).half()
    lens = [ctx] * n
    slots = paged_ref.decode_slots(rows, lens, bs)
    dev = cuda_ready
    kd, vd = k.to(dev), v.to(dev)
    tables = pagedkv.pad_block_tables(rows, device=dev)
    pagedkv.kv_append(k_new.to(dev), v_new.to(dev), kd, vd, torch.from_numpy(slots).to(dev))
    out = pagedkv.paged_attention_decode_batched(q.to(dev), kd, vd, tables,
                                                 torch.tensor(lens, dtype=torch.int32, device=dev), 1 / math.sqrt(d))
    kr, vr = k.numpy().copy(), v.numpy().copy()
    paged_ref.kv_append_ref(kr, vr, k_new.numpy(), v_new.numpy(), slots)
    assert np.array_equal(kd.cpu().numpy(), kr) and np.array_equal(vd.cpu().numpy(), vr)
    _oracle_check(out, q, torch.from_numpy(kr), torch.from_numpy(vr), rows, lens, 1 / math.sqrt(d))
    assert pagedkv.read_error_flags(dev) == 0


@refpath.requires_reference
def test_config4_copy_on_write_append_attention_vs_oracle(cuda_ready):
    """Config 4 with every group's last block shared and partial (15 rows,
    ref count 64): copy-on-write bookkeeping on the reference's
    BlockAllocator, one copy_blocks launch over 24 layers, the append, then
    attention; the same three steps on the CPU oracle."""
    refpath.ensure_on_path()
    from engine.memory.block_allocator import BlockAllocator, BlockTable
    from pagedkv import integration

    groups, per_group, layers = 8, 64, 24
    hq, hkv, d, bs = 14, 2, 64, 16
    n = groups * per_group
    prefix_blocks, own_blocks = 64, 15  # + the shared partial block = 80 blocks, 1280 tokens after the append
    nb = groups * (prefix_blocks + 1) + n * (own_blocks + 1) + 64
    alloc = BlockAllocator(num_blocks=nb)
    tables = []
    for gi in range(groups):
        prefix = [alloc.allocate() for _ in range(prefix_blocks)]
        fork = alloc.allocate()
        for s in range(per_group):
            shared = list(prefix) + [fork] if s == 0 else [alloc.fork(b) for b in prefix] + [alloc.fork(fork)]
            own = [alloc.allocate() for _ in range(own_blocks)]
            ids = shared[:prefix_blocks] + own + shared[prefix_blocks:]
            tables.append(BlockTable(seq_id=gi * per_group + s, block_size=bs, physical_block_ids=ids,
                                     num_tokens=1279))
    forks = {t.physical_block_ids[-1] for t in tables}
    assert len(forks) == groups and all(alloc.ref_counts[f] == per_group for f in forks)
    pairs = integration.prepare_copy_on_write(tables, alloc, bs)
    # every sharer but the last one of each group takes a copy
    assert len(pairs) == groups * (per_group - 1)
    assert all(alloc.ref_counts[f] == 1 for f in forks)
    alloc.check_invariants()

    g = torch.Generator().manual_seed(1201)
    kc = [torch.randn(nb, bs, hkv, d, generator=g).half() for _ in range(layers)]
    vc = [torch.randn(nb, bs, hkv, d, generator=g).half() for _ in range(layers)]
    q = torch.randn(n, hq, d, generator=g).half()
    k_new = torch.randn(n, hkv, d, generator=g).half()
    v_new = torch.randn(n, hkv, d, generator=g).half()
    rows = [list(t.physical_block_ids) for t in tables]
    lens = [t.num_tokens + 1 for t in tables]
    slots = paged_ref.decode_slots(rows, lens, bs)
    mapping = np.asarray(pairs, dtype=np.int64)

    dev = cuda_ready
    kd = [t.to(dev) for t in kc]
    vd = [t.to(dev) for t in vc]
    pagedkv.copy_blocks(kd, vd, torch.from_numpy(mapping).to(dev))
    layer = 5  # the layer whose decode step runs here
    pagedkv.kv_append(k_new.to(dev), v_new.to(dev), kd[layer], vd[layer], torch.from_numpy(slots).to(dev))
    out = pagedkv.paged_attention_decode_batched(q.to(dev), kd[layer], vd[layer],
                                                 pagedkv.pad_block_tables(rows, device=dev),
                                                 torch.tensor(lens, dtype=torch.int32, device=dev), 1 / math.sqrt(d))

    kr = [t.numpy().copy() for t in kc]
    vr = [t.numpy().copy() for t in vc]
    paged_ref.copy_blocks_ref(kr, vr, mapping)
    paged_ref.kv_append_ref(kr[layer], vr[layer], k_new.numpy(), v_new.numpy(), slots)
    for l in range(layers):
        assert np.array_equal(kd[l].cpu().numpy(), kr[l]) and np.array_equal(vd[l].cpu().numpy(), vr[l]), l
    _oracle_check(out, q, torch.from_numpy(kr[layer]), torch.from_numpy(vr[layer]), rows, lens, 1 / math.sqrt(d))
    assert pagedkv.read_error_flags(dev) == 0
