"""CPU: the indexed prefix-cache lookup against the reference allocator.

The reference's own randomized state-machine test
(tests/test_block_allocator.py:145-240 of the reference) runs against the
patched class, and a second randomized run compares the indexed lookup with
the reference's scanning lookup on caches with several key lengths and deep
chains."""
import importlib.util
import random
import sys
import time

import pytest

import refpath  # noqa: E402

pytestmark = refpath.requires_reference
refpath.ensure_on_path()

from pagedkv import prefix_index  # noqa: E402


@pytest.fixture
def patched():
    from engine.memory.block_allocator import BlockAllocator

    saved = prefix_index.install(BlockAllocator)
    try:
        yield BlockAllocator
    finally:
        prefix_index.uninstall(saved)


@pytest.mark.parametrize("seed", [7, 19, 2025, 65537])
def test_reference_state_machine_on_patched_allocator(patched, seed):
    spec = importlib.util.spec_from_file_location("ref_test_block_allocator", refpath.reference_test_file("test_block_allocator.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert mod.BlockAllocator is patched and patched.lookup_prefix is prefix_index.lookup_prefix
    mod.test_prefix_cache_randomized_state_machine(seed)


def test_indexed_lookup_equals_scan_with_mixed_key_lengths(patched):
    from engine.memory.block_allocator import BlockAllocator

    rng = random.Random(3)
    for trial in range(40):
        alloc = BlockAllocator(num_blocks=64, enable_prefix_cache=True)
        keys = [None]
        for _ in range(rng.randrange(5, 60)):
            if not (alloc.free_block_ids or alloc.cached_free):
                break
            bid = alloc.allocate()
            parent = rng.choice(keys)
            tokens = tuple(rng.randrange(4) for _ in range(rng.choice([1, 2, 2, 3])))
            key = (parent, tokens)
            if key in alloc.cache:
                alloc.release(bid)
                continue
            alloc.register(bid, key)
            keys.append(key)
            if rng.random() < 0.4:
                alloc.release(bid)  # cached-free: later allocations may evict it
        for _ in range(60):
            q = [rng.randrange(4) for _ in range(rng.randrange(0, 12))]
            got = alloc.lookup_prefix(q)
            assert got == _scan(alloc, q), (trial, q)


def _scan(alloc, token_ids):
    """The reference algorithm (block_allocator.py:236-252), restated."""
    result, offset, parent = [], 0, None
    while offset < len(token_ids):
        matches = [(key, b) for key, b in alloc.cache.items()
                   if key[0] == parent and tuple(token_ids[offset: offset + len(key[1])]) == key[1]]
        if not matches:
            break
        key, b = max(matches, key=lambda item: len(item[0][1]))
        result.append(b)
        offset += len(key[1])
        parent = key
    return result


def test_index_survives_uninstall_and_reinstall():
    from engine.memory.block_allocator import BlockAllocator

    saved = prefix_index.install(BlockAllocator)
    alloc = BlockAllocator(num_blocks=8, enable_prefix_cache=True)
    b0 = alloc.allocate()
    alloc.register(b0, (None, (1, 2)))
    assert alloc.lookup_prefix([1, 2, 3]) == [b0]
    prefix_index.uninstall(saved)
    b1 = alloc.allocate()
    alloc.register(b1, ((None, (1, 2)), (3,)))  # registered through the reference's own method
    saved = prefix_index.install(BlockAllocator)
    try:
        assert alloc.lookup_prefix([1, 2, 3]) == [b0, b1]  # stale index rebuilt
    finally:
        prefix_index.uninstall(saved)


def test_indexed_lookup_is_faster_on_a_large_cache(patched):
    from engine.memory.block_allocator import BlockAllocator

    alloc = BlockAllocator(num_blocks=4096, enable_prefix_cache=True)
    parent = None
    chain = []
    for i in range(4096):
        bid = alloc.allocate()
        tokens = tuple(range(16 * i, 16 * i + 16))
        alloc.register(bid, (parent, tokens))
        parent = (parent, tokens)
        chain.append(bid)
    prompt = list(range(16 * 64))  # a 64-block prompt
    t0 = time.perf_counter()
    got = alloc.lookup_prefix(prompt)
    fast = time.perf_counter() - t0
    t0 = time.perf_counter()
    want = _scan(alloc, prompt)
    slow = time.perf_counter() - t0
    assert got == want == chain[:64]
    assert fast * 20 < slow, (fast, slow)
