"""GPU: the reference's own serving stack running on the installed B200 path.

``pagedkv.integration.install()`` puts the kernels, the decode forward, the
runner's prefill write and decode step and the prefix index into the
reference's modules. These tests then drive the reference's OWN code on the
B200 (found through ``refpath``):

* the reference's Triton-gated kernel tests
  (tests/test_paged_attention_reference.py:267-643 of the reference), run
  unmodified against the installed kernels;
* the reference's ``Scheduler.step`` -> ``KernelPagedManualDecode.prefill`` /
  ``decode_step`` -> ``Scheduler.post_step`` loop (the loop of
  engine/serving/async_engine.py:106-121 and :160-200, the scheduler of
  engine/scheduler/continuous_batching.py:337-476, the runner of
  engine/kernels/paged_attention_integration.py:518-653) on a random-init
  Qwen2 model, compared with the same loop on the uninstalled reference with
  its naive paged attention (paged_attention.py:30-83, fp32) in place of its
  Triton kernel;
* the installed decode step's CUDA-graph path against its eager path, with
  the attention modules bound once (nothing rebound per step);
* copy-on-write inside the installed decode step for a partial block shared
  between two sequences of the reference's ``BlockAllocator``.
"""
from __future__ import annotations

import importlib
import importlib.util

import pytest
import torch

import refpath

pytestmark = [pytest.mark.gpu, refpath.requires_reference]

refpath.ensure_on_path()

TRITON_TESTS = [
    "test_triton_paged_attention_decode_v1_matches_reference",
    "test_triton_paged_attention_decode_v2_matches_v1_and_reference",
    "test_triton_paged_attention_long_sequence_2048_tokens",
    "test_triton_paged_attention_large_magnitude_scores_no_overflow",
    "test_triton_paged_attention_decode_batched_variable_lengths",
]

# Logit tolerance between the B200 path (fp16 attention output, fp32
# accumulation) and the naive reference (fp32 attention) after two decoder
# layers: the two greedy streams must agree token for token until a step whose
# top-1 / top-2 logit margin is within this noise.
LOGIT_ATOL = 0.25


def _modules():
    pa = importlib.import_module("engine.kernels.paged_attention")
    integ = importlib.import_module("engine.kernels.paged_attention_integration")
    alloc = importlib.import_module("engine.memory.block_allocator")
    sched = importlib.import_module("engine.scheduler.continuous_batching")
    return pa, integ, alloc, sched


@pytest.fixture
def installed(cuda_ready):
    from pagedkv import integration

    pa, integ, alloc, _ = _modules()
    saved = integration.install(pa, integ, alloc)
    try:
        yield saved
    finally:
        integration.uninstall(saved)


@pytest.mark.parametrize("name", TRITON_TESTS)
def test_reference_kernel_tests_on_installed_kernels(installed, name):
    """The reference's own GPU kernel tests, loaded after install() so their
    ``from engine.kernels.paged_attention import ...`` binds the B200 kernels."""
    import pagedkv

    path = refpath.reference_test_file("test_paged_attention_reference.py")
    assert path is not None
    spec = importlib.util.spec_from_file_location(f"ref_kernel_tests_{name}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert mod.paged_attention_decode_batched is pagedkv.paged_attention_decode_batched
    assert mod.paged_attention_decode_v2 is pagedkv.paged_attention_decode_v2
    getattr(mod, name)()
    launches, family = pagedkv.last_decode_launch_info()
    assert launches >= 1 and family in ("tc", "simt")


def _small_qwen2(dev, layers=2, seed=0):
    """Random-init Qwen2 with the Qwen2.5-0.5B attention shape (14 / 2 heads,
    head_dim 64), a small MLP and vocabulary, fp16; the output projection is
    scaled so greedy margins stand well above fp16 noise."""
    from transformers import Qwen2Config, Qwen2ForCausalLM

    torch.manual_seed(seed)
    cfg = Qwen2Config(hidden_size=896, intermediate_size=1024, num_hidden_layers=layers, num_attention_heads=14,
                      num_key_value_heads=2, vocab_size=2048, tie_word_embeddings=False,
                      max_position_embeddings=4096, rope_theta=1000000.0, rms_norm_eps=1e-6)
    with torch.device(dev):
        model = Qwen2ForCausalLM(cfg).to(torch.float16)
    with torch.no_grad():
        model.lm_head.weight.mul_(16.0)
    return model.eval()


def _naive_batched(pa):
    """The reference's naive paged attention (fp32) behind the batched
    kernel's signature: the oracle arm of the loop comparison."""

    def fn(q, k_cache, v_cache, block_tables, seq_lens, scale):
        lens = [int(x) for x in seq_lens.tolist()]
        bs = k_cache.shape[1]
        tables = [row[: (n + bs - 1) // bs] for row, n in zip(block_tables.tolist(), lens)]
        out = pa.naive_reference_paged_attention(q.float(), k_cache.float(), v_cache.float(), tables, lens, scale)
        return out.to(q.dtype)

    return fn


def _run_loop(model, requests, *, num_blocks, prefix_mode, max_batch, install_opts=None, max_new=24):
    """Drive the reference's scheduler and runner over ``requests`` (lists of
    prompt token ids). With ``install_opts`` the B200 path is installed for the
    run; without, the reference runs with its naive attention in place of the
    Triton kernel. Returns ({request index: [(token, margin, logits)]}, runner)."""
    from pagedkv import integration

    pa, integ, alloc_mod, sched_mod = _modules()
    saved = None
    orig_kernel = integ.paged_attention_decode_batched
    if install_opts is not None:
        saved = integration.install(pa, integ, alloc_mod, **install_opts)
    else:
        integ.paged_attention_decode_batched = _naive_batched(pa)
    try:
        share = prefix_mode != "off"
        allocator = alloc_mod.BlockAllocator(num_blocks=num_blocks, enable_prefix_cache=share)
        runner = integ.KernelPagedManualDecode(model=model, tokenizer=None, block_size=16, num_blocks=num_blocks,
                                               device="cuda", dtype=torch.float16, prefix_mode=prefix_mode)
        scheduler = sched_mod.Scheduler(allocator, block_size=16, max_batch_size=max_batch,
                                        prefix_mode=prefix_mode, debug_invariants=True)
        index = {}
        for i, ids in enumerate(requests):
            seq = scheduler.add_request(prompt="", max_new_tokens=max_new, prompt_token_ids=list(ids),
                                        ignore_eos=True)
            index[seq.seq_id] = i
        record = {i: [] for i in range(len(requests))}
        steps = 0
        while scheduler.has_unfinished_requests():
            batch = scheduler.step()
            if batch is None or batch.is_empty:
                continue
            if batch.batch_type == sched_mod.BatchType.PREFILL:
                toks = [runner.prefill(batch.sequences[0], allocator=allocator)]
            else:
                toks = runner.decode_step(batch.sequences, allocator=allocator)
            for seq, t in zip(batch.sequences, toks):
                record[index[seq.seq_id]].append((int(t), float(seq.last_logit_margin), seq.last_logits.float()))
            scheduler.post_step(batch, toks)
            steps += 1
            assert steps < 10000
        allocator.check_invariants()
        return record, runner
    finally:
        if saved is not None:
            integration.uninstall(saved)
        else:
            integ.paged_attention_decode_batched = orig_kernel


def _compare(rec_new, rec_ref):
    """Token streams equal until a near-tie; logits close while they agree."""
    diverged, worst = 0, 0.0
    for i in rec_ref:
        a, b = rec_new[i], rec_ref[i]
        assert len(a) == len(b)
        for (ta, ma, la), (tb, mb, lb) in zip(a, b):
            diff = float((la - lb).abs().max())
            worst = max(worst, diff)
            assert diff <= LOGIT_ATOL, f"request {i}: logits differ by {diff}"
            if ta != tb:
                # a flip is only acceptable where the reference's own margin is noise-sized
                assert mb <= 2 * LOGIT_ATOL, f"request {i}: token {ta} vs {tb} at margin {mb}"
                diverged += 1
                break
    assert diverged <= max(1, len(rec_ref) // 2), f"{diverged} of {len(rec_ref)} streams diverged"
    return worst


def _requests(seed, n, lo, hi, shared_prefix=0):
    g = torch.Generator().manual_seed(seed)
    prefix = torch.randint(0, 2048, (shared_prefix,), generator=g).tolist()
    out = []
    for _ in range(n):
        length = int(torch.randint(lo, hi + 1, (1,), generator=g))
        out.append(prefix + torch.randint(0, 2048, (length,), generator=g).tolist())
    return out


@pytest.mark.parametrize(
    "prefix_mode,num_blocks,shared",
    [
        ("off", 40, 0),     # a pool small enough that the scheduler preempts and re-prefills
        ("share", 256, 48),  # prefix cache: blocks of a 48-token shared prefix are reused
    ],
)
def test_reference_scheduler_loop_matches_naive_reference(cuda_ready, prefix_mode, num_blocks, shared):
    model = _small_qwen2(cuda_ready)
    reqs = _requests(11, 6, 20, 120, shared_prefix=shared)
    rec_ref, _ = _run_loop(model, reqs, num_blocks=num_blocks, prefix_mode=prefix_mode, max_batch=8)
    rec_new, runner = _run_loop(model, reqs, num_blocks=num_blocks, prefix_mode=prefix_mode, max_batch=8,
                                install_opts={})
    assert runner.__dict__.get("_pagedkv_graphs") is not None and runner._pagedkv_graphs.graphs
    _compare(rec_new, rec_ref)


def test_installed_graphs_match_eager_and_bind_once(cuda_ready):
    """The CUDA-graph decode step against the eager one (attention modules
    bound once and never rebound), both on the installed path."""
    from pagedkv import integration

    model = _small_qwen2(cuda_ready, seed=3)
    reqs = _requests(5, 5, 10, 90)
    rec_graph, runner_g = _run_loop(model, reqs, num_blocks=256, prefix_mode="off", max_batch=8,
                                    install_opts={"cuda_graphs": True})
    attn = [m for m in model.modules() if hasattr(m, "q_proj")]
    assert all("forward" not in m.__dict__ for m in attn)  # the graph path never patches

    # eager path: wrap the runner's step to observe the bound forwards between steps
    pa, integ, alloc_mod, _ = _modules()
    seen = []
    orig_step = integration.decode_step

    def spying_step(self, seqs, allocator=None):
        out = orig_step(self, seqs, allocator)
        seen.append([m.__dict__.get("forward") for m in attn])
        return out

    integration_decode = integration.decode_step
    try:
        integration.decode_step = spying_step
        rec_eager, _ = _run_loop(model, reqs, num_blocks=256, prefix_mode="off", max_batch=8,
                                 install_opts={"cuda_graphs": False})
    finally:
        integration.decode_step = integration_decode
    assert len(seen) > 3
    assert all(f is not None for f in seen[0])
    for later in seen[1:]:
        assert all(a is b for a, b in zip(later, seen[0])), "a decode step rebound an attention forward"
    # uninstall restored the modules
    assert all("forward" not in m.__dict__ for m in attn)
    for i in rec_graph:
        assert [t for t, _, _ in rec_graph[i]] == [t for t, _, _ in rec_eager[i]]
        for (_, _, la), (_, _, lb) in zip(rec_graph[i], rec_eager[i]):
            assert float((la - lb).abs().max()) <= 0.05


def _fork_pair(runner, allocator, sched_mod, prompt, second_token_offset=1):
    """Prefill ``prompt`` for sequence A and fork it into B: B's table holds
    the same blocks (ref count 2), the last one partially filled."""
    seq_a = sched_mod.Sequence(seq_id=0, prompt="", max_new_tokens=8, prompt_token_ids=list(prompt))
    seq_a.block_table = importlib.import_module("engine.memory.block_allocator").BlockTable(seq_id=0, block_size=16)
    for _ in range((len(prompt) + 15) // 16):
        seq_a.block_table.physical_block_ids.append(allocator.allocate())
    seq_a.block_table.num_tokens = len(prompt)
    first = runner.prefill(seq_a, allocator=allocator)
    bt_b = importlib.import_module("engine.memory.block_allocator").BlockTable(
        seq_id=1, block_size=16, physical_block_ids=[allocator.fork(b) for b in seq_a.block_table.physical_block_ids],
        num_tokens=len(prompt))
    seq_b = sched_mod.Sequence(seq_id=1, prompt="", max_new_tokens=8, prompt_token_ids=list(prompt), block_table=bt_b)
    seq_a.last_token_id = first
    seq_b.last_token_id = (first + second_token_offset) % 2048
    return seq_a, seq_b


def test_copy_on_write_decode_step_on_shared_partial_block(cuda_ready):
    """Two sequences of the reference BlockAllocator share every block,
    the last one partial (ref count 2). The installed decode step with
    copy-on-write gives A a private copy of that block before the append, B
    keeps the original; both then step like two unshared sequences of the
    naive reference. Without copy-on-write the reference's assert fires."""
    from pagedkv import integration

    pa, integ, alloc_mod, sched_mod = _modules()
    model = _small_qwen2(cuda_ready, seed=7)
    prompt = torch.randint(0, 2048, (40,), generator=torch.Generator().manual_seed(3)).tolist()

    # default: the reference's shared-block assert
    saved = integration.install(pa, integ, alloc_mod)
    try:
        allocator = alloc_mod.BlockAllocator(num_blocks=64)
        runner = integ.KernelPagedManualDecode(model=model, tokenizer=None, block_size=16, num_blocks=64,
                                               device="cuda", dtype=torch.float16)
        a, b = _fork_pair(runner, allocator, sched_mod, prompt)
        with pytest.raises(AssertionError, match="shared"):
            runner.decode_step([a, b], allocator=allocator)
    finally:
        integration.uninstall(saved)

    # copy-on-write
    saved = integration.install(pa, integ, alloc_mod, copy_on_write=True)
    try:
        allocator = alloc_mod.BlockAllocator(num_blocks=64)
        runner = integ.KernelPagedManualDecode(model=model, tokenizer=None, block_size=16, num_blocks=64,
                                               device="cuda", dtype=torch.float16)
        a, b = _fork_pair(runner, allocator, sched_mod, prompt)
        shared = a.block_table.physical_block_ids[2]
        before = [runner.pool.k_cache[l][shared].clone() for l in range(2)]
        got = {0: [], 1: []}
        for step in range(20):  # crosses into the next block at token 48
            for s in (a, b):
                bt = s.block_table
                if bt.num_tokens % 16 == 0:
                    bt.physical_block_ids.append(allocator.allocate())
            toks = runner.decode_step([a, b], allocator=allocator)
            for i, (s, t) in enumerate(zip((a, b), toks)):
                got[i].append((t, float(s.last_logit_margin), s.last_logits.float()))
                s.last_token_id = t
            if step == 0:
                copy = a.block_table.physical_block_ids[2]
                assert copy != shared and b.block_table.physical_block_ids[2] == shared
                assert allocator.ref_counts[shared] == 1 and allocator.ref_counts[copy] == 1
                for l in range(2):
                    ka, kb = runner.pool.k_cache[l][copy], runner.pool.k_cache[l][shared]
                    assert torch.equal(ka[:8], before[l][:8]) and torch.equal(kb[:8], before[l][:8])
                    assert not torch.equal(ka[8], kb[8])  # each sequence appended its own token
        allocator.check_invariants()
    finally:
        integration.uninstall(saved)

    # oracle: the uninstalled reference with naive attention on two separately
    # prefilled (unshared) sequences fed the same first tokens
    orig = integ.paged_attention_decode_batched
    integ.paged_attention_decode_batched = _naive_batched(pa)
    try:
        allocator = alloc_mod.BlockAllocator(num_blocks=64)
        runner = integ.KernelPagedManualDecode(model=model, tokenizer=None, block_size=16, num_blocks=64,
                                               device="cuda", dtype=torch.float16)
        seqs = []
        for sid, off in ((0, 0), (1, 1)):
            s = sched_mod.Sequence(seq_id=sid, prompt="", max_new_tokens=8, prompt_token_ids=list(prompt))
            s.block_table = alloc_mod.BlockTable(seq_id=sid, block_size=16)
            for _ in range(3):
                s.block_table.physical_block_ids.append(allocator.allocate())
            s.block_table.num_tokens = 40
            first = runner.prefill(s, allocator=allocator)
            s.last_token_id = (first + off) % 2048
            seqs.append(s)
        want = {0: [], 1: []}
        for step in range(20):
            for s in seqs:
                if s.block_table.num_tokens % 16 == 0:
                    s.block_table.physical_block_ids.append(allocator.allocate())
            toks = runner.decode_step(seqs, allocator=allocator)
            for i, (s, t) in enumerate(zip(seqs, toks)):
                want[i].append((t, float(s.last_logit_margin), s.last_logits.float()))
                s.last_token_id = t
    finally:
        integ.paged_attention_decode_batched = orig
    _compare(got, want)
