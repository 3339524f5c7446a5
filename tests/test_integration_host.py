"""CPU: host-side logic of the drop-in integration (no kernel launches)."""
import sys
from types import SimpleNamespace

import numpy as np
import pytest
import torch

import cases
import refpath
from oracle import paged_ref
from pagedkv import integration, prefix_index



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


@refpath.requires_reference
def test_prepare_copy_on_write_with_reference_allocator():
    refpath.ensure_on_path()
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


@refpath.requires_reference
def test_install_replaces_reference_symbols_and_uninstall_restores():
    refpath.ensure_on_path()
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
        assert integ.KernelPagedManualDecode.decode_step is integration.decode_step
        from engine.memory.block_allocator import BlockAllocator

        assert BlockAllocator.lookup_prefix is prefix_index.lookup_prefix
    finally:
        integration.uninstall(saved)
    assert integ.KernelPagedManualDecode._copy_prefill_kv is not integration.copy_prefill_kv
    assert integ.KernelPagedManualDecode.decode_step is not integration.decode_step
    from engine.memory.block_allocator import BlockAllocator

    assert BlockAllocator.lookup_prefix is not prefix_index.lookup_prefix
    assert (pa.paged_attention_decode_batched, integ.paged_attention_decode_batched, integ.PagedAttentionContext) == before


def _decode_step_fixture(dtype):
    """Sequences of every kind the reference's decode_step accepts, a fake
    model whose logits depend on the input ids only, and a fake runner."""

    class BT:
        def __init__(self, ids, n):
            self.physical_block_ids = list(ids)
            self.num_tokens = n

    class NoDiag:  # no last_logits attribute: no diagnostics stored
        def __init__(self, bt, gen):
            self.block_table = bt
            self.generated_ids = gen

    seqs = [
        SimpleNamespace(seq_id=0, block_table=BT([3, 4], 17), last_token_id=11, last_logits=None,
                        last_logit_margin=None),
        {"seq_id": 1, "block_table": BT([7], 5), "last_token_id": 42},
        NoDiag(BT([9, 10, 12], 40), [5, 77]),
        SimpleNamespace(seq_id=3, block_table=BT([1], 15), last_token_id=3, last_logits=None,
                        last_logit_margin=None),
    ]
    vocab = 257

    class FakeModel:
        def __call__(self, input_ids, position_ids, use_cache):
            rows = []
            for tok, pos in zip(input_ids[:, 0].tolist(), position_ids[:, 0].tolist()):
                g = torch.Generator().manual_seed(tok * 1000 + pos)
                rows.append((torch.randn(vocab, generator=g) * 4).to(dtype))
            return SimpleNamespace(logits=torch.stack(rows)[:, None, :])

    runner = SimpleNamespace(block_size=16, device=torch.device("cpu"), pool=SimpleNamespace(device="cpu"),
                             model=FakeModel(), allocator=SimpleNamespace(ref_counts={3: 1, 4: 1, 7: 1}))
    return seqs, runner


class _NullPatch:
    def __init__(self, *a, **k):
        pass

    def __enter__(self):
        return None

    def __exit__(self, *exc):
        return False


@refpath.requires_reference
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_decode_step_matches_the_reference_with_batched_syncs(monkeypatch, dtype):
    """integration.decode_step against the reference's own
    KernelPagedManualDecode.decode_step on the same sequences and logits: the
    same next tokens, length bumps, last_logits and logit margins (the model
    forward is a fake; the kernels are covered by the GPU tests)."""
    refpath.ensure_on_path()
    import engine.kernels.paged_attention_integration as integ

    seqs_ref, runner_ref = _decode_step_fixture(dtype)
    seqs_new, runner_new = _decode_step_fixture(dtype)
    for mod in (integ, integration):
        monkeypatch.setattr(mod, "patch_paged_attention", _NullPatch)
        monkeypatch.setattr(mod, "PagedAttentionContext", lambda **k: None)
    want = integ.KernelPagedManualDecode.decode_step(runner_ref, seqs_ref, None)
    got = integration.decode_step(runner_new, seqs_new, None)
    assert got == want
    for a, b in zip(seqs_ref, seqs_new):
        f = (lambda s, k: s[k]) if isinstance(a, dict) else getattr
        assert f(a, "block_table").num_tokens == f(b, "block_table").num_tokens
        if isinstance(a, dict) or hasattr(a, "last_logits"):
            assert torch.equal(f(a, "last_logits"), f(b, "last_logits"))
            assert f(a, "last_logit_margin") == f(b, "last_logit_margin")
        else:
            assert not hasattr(b, "last_logits")


def test_decode_step_refuses_missing_and_shared_write_blocks():
    seqs, runner = _decode_step_fixture(torch.float16)
    seqs[0].block_table.num_tokens = 32  # write block index 2: not allocated
    with pytest.raises(AssertionError, match="no allocated block"):
        integration.decode_step(runner, seqs[:1], None)
    seqs, runner = _decode_step_fixture(torch.float16)
    runner.allocator.ref_counts[4] = 3  # seq 0 writes into block 4, now shared
    with pytest.raises(AssertionError, match="shared"):
        integration.decode_step(runner, seqs[:1], None)


class _FakeAttention(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.q_proj = self.k_proj = self.v_proj = self.o_proj = torch.nn.Identity()

    def forward(self, hidden_states, position_embeddings=None, attention_mask=None, past_key_values=None, **kw):
        return ("original", hidden_states)


def test_patch_paged_attention_binds_once_and_only_swaps_the_context():
    """The attention modules are bound to the paged forward on first use and
    never rebound; entering / leaving a decode block only swaps the context,
    and with no decode context a module runs its original forward."""
    model = torch.nn.Sequential(_FakeAttention(), torch.nn.Sequential(_FakeAttention()))
    attn = [m for m in model.modules() if isinstance(m, _FakeAttention)]
    not_decode = SimpleNamespace(is_decode=False)
    with integration.patch_paged_attention(model, not_decode):
        bound = [m.__dict__["forward"] for m in attn]
        assert model._pagedkv_context_holder.ctx is not_decode
        assert attn[0](hidden_states=5, position_embeddings=None) == ("original", 5)
    assert model._pagedkv_context_holder.ctx is None
    for _ in range(3):
        with integration.patch_paged_attention(model, not_decode):
            assert all(m.__dict__["forward"] is b for m, b in zip(attn, bound))
    assert attn[1](hidden_states=7, position_embeddings=None) == ("original", 7)  # outside a step: original forward
    integration.detach_paged_attention(model)
    assert all("forward" not in m.__dict__ and "_pagedkv_context_holder" not in m.__dict__ for m in attn)
    assert "_pagedkv_context_holder" not in model.__dict__


def test_install_options_are_set_on_the_runner_class_and_removed():
    class Runner:
        def decode_step(self):
            pass

        def _copy_prefill_kv(self):
            pass

    pa, integ = SimpleNamespace(), SimpleNamespace(KernelPagedManualDecode=Runner)
    saved = integration.install(pa, integ, SimpleNamespace(), copy_on_write=True, cuda_graphs=False)
    assert Runner._pagedkv_copy_on_write is True and Runner._pagedkv_cuda_graphs is False
    assert Runner.decode_step is integration.decode_step
    integration.uninstall(saved)
    assert "_pagedkv_copy_on_write" not in Runner.__dict__ and "_pagedkv_cuda_graphs" not in Runner.__dict__
    assert Runner.decode_step is not integration.decode_step


def test_decode_step_copy_on_write_replaces_the_shared_block_assert(monkeypatch):
    """With copy-on-write on, a shared write block is given to the sequence as
    a fresh copy (one copy_blocks call for all layers) instead of raising."""
    seqs, runner = _decode_step_fixture(torch.float16)
    alloc = _FakeAllocator(64)
    for b in range(16):
        alloc.ref_counts[b] = 1
    alloc.free_ids = [i for i in alloc.free_ids if i >= 16]
    alloc.ref_counts[4] = 2  # seq 0 writes into block 4, shared
    runner.allocator = alloc
    runner._pagedkv_copy_on_write = True
    calls = []
    monkeypatch.setattr(integration, "copy_on_write", lambda pool, pairs: calls.append(list(pairs)))
    monkeypatch.setattr(integration, "patch_paged_attention", _NullPatch)
    monkeypatch.setattr(integration, "PagedAttentionContext", lambda **k: None)
    seqs[0].block_table.num_tokens = 17
    out = integration.decode_step(runner, seqs[:1], None)
    assert len(out) == 1 and len(calls) == 1 and calls[0][0][0] == 4
    new_block = seqs[0].block_table.physical_block_ids[1]
    assert new_block != 4 and alloc.ref_counts[4] == 1 and alloc.ref_counts[new_block] == 1
