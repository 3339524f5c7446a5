"""Indexed prefix-cache lookup for the reference's ``BlockAllocator``.

``BlockAllocator.lookup_prefix`` (engine/memory/block_allocator.py:231-252)
walks the chain of cached full blocks matching a prompt, and at every step
scans the WHOLE cache for keys whose parent is the current chain key and whose
tokens match the prompt at the current offset, taking the longest: O(cache)
per block of the prompt. The same chain-key semantics with a per-parent index
``{parent_key: {token_count: {tokens: block_id}}}`` cost one dict lookup per
distinct key length per step.

:func:`install` patches ``lookup_prefix`` and the two methods that change the
cache (``register`` adds a key, ``allocate`` evicts the oldest cached-free
block's key) on the allocator class, so every instance keeps its index in step;
an instance whose index predates an :func:`uninstall` rebuilds it from its
``cache`` on first use. Everything else (``cache``, ``block_key``,
``cached_free``, the ref counts, errors) is the reference's own code.
"""
from __future__ import annotations

from typing import Any, Dict, Hashable, List, Tuple

_generation = 0  # bumped by uninstall(): indexes built before it are stale

Index = Dict[Any, Dict[int, Dict[Tuple[int, ...], int]]]


def _build(alloc: Any) -> Index:
    by_parent: Index = {}
    for (parent, tokens), block_id in alloc.cache.items():
        by_parent.setdefault(parent, {}).setdefault(len(tokens), {})[tokens] = block_id
    alloc.__dict__["_pagedkv_prefix_index"] = (by_parent, _generation)
    return by_parent


def _index(alloc: Any) -> Index:
    held = alloc.__dict__.get("_pagedkv_prefix_index")
    if held is None or held[1] != _generation:
        return _build(alloc)
    return held[0]


def lookup_prefix(self: Any, token_ids: List[int]) -> List[int]:
    """Longest cached block chain matching ``token_ids`` (same result as the
    reference's scan: at each step the longest key under the current parent
    whose tokens match the prompt at the offset)."""
    if not self.enable_prefix_cache:
        return []
    by_parent = _index(self)
    result: List[int] = []
    offset = 0
    parent: Hashable | None = None
    n = len(token_ids)
    while offset < n:
        by_len = by_parent.get(parent)
        if not by_len:
            break
        hit = None
        for length in sorted(by_len, reverse=True):
            if offset + length > n:
                continue
            tokens = tuple(token_ids[offset : offset + length])
            block_id = by_len[length].get(tokens)
            if block_id is not None:
                hit = (tokens, block_id)
                break
        if hit is None:
            break
        tokens, block_id = hit
        result.append(block_id)
        offset += len(tokens)
        parent = (parent, tokens)
    return result


def _patched_register(orig):
    def register(self: Any, block_id: int, key: Tuple[Hashable | None, Tuple[int, ...]]) -> None:
        orig(self, block_id, key)  # validation and the cache entry, unchanged
        parent, tokens = key[0], tuple(key[1])
        _index(self).setdefault(parent, {}).setdefault(len(tokens), {})[tokens] = block_id

    register.__doc__ = orig.__doc__
    return register


def _patched_allocate(orig):
    def allocate(self: Any) -> int:
        evicted = None
        if not self.free_block_ids and self.enable_prefix_cache and self.cached_free:
            evicted = self.block_key.get(next(iter(self.cached_free)))
        block_id = orig(self)
        if evicted is not None:
            parent, tokens = evicted
            by_len = _index(self).get(parent)
            if by_len is not None and len(tokens) in by_len:
                by_len[len(tokens)].pop(tokens, None)
                if not by_len[len(tokens)]:
                    del by_len[len(tokens)]
                if not by_len:
                    del _index(self)[parent]
        return block_id

    allocate.__doc__ = orig.__doc__
    return allocate


def install(allocator_cls: Any) -> dict:
    """Patch ``allocator_cls`` (the reference's ``BlockAllocator``); returns
    what :func:`uninstall` restores."""
    saved = {name: allocator_cls.__dict__[name] for name in ("lookup_prefix", "register", "allocate")}
    allocator_cls.lookup_prefix = lookup_prefix
    allocator_cls.register = _patched_register(saved["register"])
    allocator_cls.allocate = _patched_allocate(saved["allocate"])
    return {(allocator_cls, name): fn for name, fn in saved.items()}


def uninstall(saved: dict) -> None:
    global _generation
    for (cls, name), fn in saved.items():
        setattr(cls, name, fn)
    _generation += 1
