"""CPU: host-side logic of the drop-in integration (no kernel launches)."""
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest
import torch

import cases
from oracle import paged_ref
from pagedkv import integration, prefix_index

REFERENCE = Path("/root/reference")


def test_decode_metadata_matches_oracle_slots():
    inp = cases.make_append_inputs(cases.APPEND_CASES["append_qwen_shape"])
    bs = cases.APPEND_CASES["append_qwen_shape"]["bs"]
    tables, lens, slots = integration.build_decode_metadata(inp["tables"], inp["lens"], bs, "cpu")
    assert tables.dtype == torch.int32 and lens.dtype == torch.int32 and slots.dtype == torch.int64
    assert lens.tolist() == inp["lens"]
    for i, row in enumerate(inp["tables"]):
        assert tables[i, : len(row)].tolist() == row
        assert not tables[i, len(row):].any()
    assert np.array_equal(slots.numpy(), paged_ref.decode_slots(inp["tables"], inp["lens"], bs))


def test_decode_metadata_zero_length_and_empty_tables():
    tables, lens, slots = integration.build_decode_metadata([[], [5, 6]], [0, 17], 16, "cpu")
    assert tables.shape == (2, 2) and slots.tolist() == [-1, 6 * 16 + 0]
    tables, lens, slots = integration.build_decode_metadata([[]], [0], 16, "cpu")
    assert tables.shape == (1, 1) and slots.tolist() == [-1]


class _FakeAllocator:
    """Minimal allocator with the reference's refcount API."""

    def __init__(self, n):
        self.free_ids = list(range(n))
        self.ref_counts = {}

    def allocate(self):
        b = self.free_ids.pop()
        self.ref_counts[b] = 1
        return b

    def fork(self, b):
        self.ref_counts[b] += 1
        return b

    def release(self, b):
        self.ref_counts[b] -= 1
        if self.ref_counts[b] == 0:
            del self.ref_counts[b]
            self.free_ids.append(b)


def test_prepare_copy_on_write_with_fake_allocator():
    alloc = _FakeAllocator(16)
    shared = alloc.allocate()
    a = SimpleNamespace(physical_block_ids=[alloc.allocate(), shared], num_tokens=20)
    b = SimpleNamespace(physical_block_ids=[a.physical_block_ids[0], alloc.fork(shared)], num_tokens=20)
    alloc.fork(a.physical_block_ids[0])
    c = SimpleNamespace(physical_block_ids=[alloc.allocate()], num_tokens=3)  # private write block
    pairs = integration.prepare_copy_on_write([a, b, c], alloc, 16)
    # a's write block (index 1) was shared by b: a gets a copy; then b is the sole owner
    assert len(pairs) == 1 and pairs[0][0] == shared
    assert a.physical_block_ids[1] == pairs[0][1] and b.physical_block_ids[1] == shared
    assert alloc.ref_counts[shared] == 1 and alloc.ref_counts[pairs[0][1]] == 1


@pytest.mark.skipif(not (REFERENCE / "engine").exists(), reason="reference checkout not present")
def test_prepare_copy_on_write_with_reference_allocator():
    sys.path.insert(0, str(REFERENCE))
    from engine.memory.block_allocator import BlockAllocator, BlockTable

    alloc = BlockAllocator(num_blocks=32)
    prefix = [alloc.allocate() for _ in range(2)]
    tables = []
    for i in range(4):
        ids = [alloc.fork(b) for b in prefix] if i else list(prefix)
        tables.append(BlockTable(seq_id=i, block_size=16, physical_block_ids=ids, num_tokens=24))
    pairs = integration.prepare_copy_on_write(tables, alloc, 16)
    assert len(pairs) == 3  # the last table to be visited owns the block alone
    assert sorted(set(p[0] for p in pairs)) == [prefix[1]]
    assert len({t.physical_block_ids[1] for t in tables}) == 4
    alloc.check_invariants()


@pytest.mark.skipif(not (REFERENCE / "engine").exists(), reason="reference checkout not present")
def test_install_replaces_reference_symbols_and_uninstall_restores():
    sys.path.insert(0, str(REFERENCE))
    import engine.kernels.paged_attention as pa
    import engine.kernels.paged_attention_integration as integ

    before = (pa.paged_attention_decode_batched, integ.paged_attention_decode_batched, integ.PagedAttentionContext)
    saved = integration.install(pa, integ)
    try:
        import pagedkv

        assert pa.paged_attention_decode_batched is pagedkv.paged_attention_decode_batched
        assert integ.paged_attention_decode_batched is pagedkv.paged_attention_decode_batched
        assert integ.PagedAttentionContext is integration.PagedAttentionContext
        assert integ.paged_decode_attention_forward is integration.paged_decode_attention_forward
        assert pa.naive_reference_paged_attention.__module__ == "engine.kernels.paged_attention"
        assert integ.KernelPagedManualDecode._copy_prefill_kv is integration.copy_prefill_kv
        from engine.memory.block_allocator import BlockAllocator

        assert BlockAllocator.lookup_prefix is prefix_index.lookup_prefix
    finally:
        integration.uninstall(saved)
    assert integ.KernelPagedManualDecode._copy_prefill_kv is not integration.copy_prefill_kv
    from engine.memory.block_allocator import BlockAllocator

    assert BlockAllocator.lookup_prefix is not prefix_index.lookup_prefix
    assert (pa.paged_attention_decode_batched, integ.paged_attention_decode_batched, integ.PagedAttentionContext) == before
