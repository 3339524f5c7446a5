"""CPU oracle for the paged KV-cache decode path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` may import this module, and only as the checker / the timed CPU
reference. The product (``pagedkv``) never imports it and has no CPU path.

Pinned: ``tests/test_oracle_golden.py`` checks every function here against
golden vectors produced by running the reference implementation itself
(``tests/golden/make_golden.py`` imports the reference's
``naive_reference_paged_attention`` and its ``paged_decode_attention_forward``
append and stores their outputs).

Restated from XVX-016/vLLM-inference-engine:

* ``paged_attention_ref`` — ``naive_reference_paged_attention``,
  engine/kernels/paged_attention.py:30-83: per sequence, take the first
  ``seq_len`` tokens of the blocks listed in its table (:58-69), map query
  head h to kv head h // G (:74-76), softmax(scale * q.K) @ V (:78-80).
  Output starts as zeros_like(q) (:52). Math in the input dtype (fp32 here).
* ``decode_slots`` — the write position of the decode append,
  engine/kernels/paged_attention_integration.py:150-155 (and :120-126):
  pos = seq_len - 1; slot = table[pos // BS] * BS + pos % BS.
* ``kv_append_ref`` — the assignment at integration.py:159-160:
  k_cache[phys, off] = k_new[b] (bit-exact copy).
* ``copy_blocks_ref`` — the copy-on-write data copy the reference does not
  have (fork only bumps a refcount, engine/memory/block_allocator.py:264-270):
  pool[l][dst] = pool[l][src] for all layers, K and V.
"""
from __future__ import annotations

from typing import Sequence

import numpy as np
import torch


def paged_attention_ref(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: Sequence[Sequence[int]],
    seq_lens: Sequence[int],
    scale: float,
) -> torch.Tensor:
    """softmax(scale * q K^T) V per sequence over its paged K/V, on CPU.

    q: [N, Hq, D]; k_cache/v_cache: [NB, BS, Hkv, D]; computed in q's dtype
    (pass fp32 tensors for the fp32 oracle). Returns [N, Hq, D].
    """
    num_seqs, num_q_heads, head_dim = q.shape
    num_blocks, block_size, num_kv_heads, _ = k_cache.shape
    assert num_q_heads % num_kv_heads == 0
    group = num_q_heads // num_kv_heads
    k_flat = k_cache.reshape(num_blocks * block_size, num_kv_heads, head_dim)
    v_flat = v_cache.reshape(num_blocks * block_size, num_kv_heads, head_dim)
    out = torch.zeros_like(q)
    for s in range(num_seqs):
        n = int(seq_lens[s])
        if n <= 0:
            continue
        blocks = torch.as_tensor(list(block_tables[s])[: (n + block_size - 1) // block_size], dtype=torch.int64)
        slots = (blocks[:, None] * block_size + torch.arange(block_size)[None, :]).reshape(-1)[:n]
        k = k_flat.index_select(0, slots)  # [n, Hkv, D]
        v = v_flat.index_select(0, slots)
        qs = q[s].reshape(num_kv_heads, group, head_dim)
        scores = torch.einsum("kgd,nkd->kgn", qs, k) * scale
        probs = torch.softmax(scores, dim=-1)
        out[s] = torch.einsum("kgn,nkd->kgd", probs, v).reshape(num_q_heads, head_dim)
    return out


def paged_attention_ref_f64(
    q: np.ndarray,
    k_cache: np.ndarray,
    v_cache: np.ndarray,
    block_tables: Sequence[Sequence[int]],
    seq_lens: Sequence[int],
    scale: float,
) -> np.ndarray:
    """The same function in float64 numpy: an independent high-precision
    cross-check of ``paged_attention_ref`` (max-subtracted softmax)."""
    q = np.asarray(q, dtype=np.float64)
    k_cache = np.asarray(k_cache, dtype=np.float64)
    v_cache = np.asarray(v_cache, dtype=np.float64)
    num_seqs, num_q_heads, head_dim = q.shape
    num_blocks, block_size, num_kv_heads, _ = k_cache.shape
    group = num_q_heads // num_kv_heads
    out = np.zeros_like(q)
    for s in range(num_seqs):
        n = int(seq_lens[s])
        if n <= 0:
            continue
        tok = np.arange(n)
        blocks = np.asarray(block_tables[s], dtype=np.int64)[tok // block_size]
        k = k_cache[blocks, tok % block_size]  # [n, Hkv, D]
        v = v_cache[blocks, tok % block_size]
        for h in range(num_q_heads):
            kh = h // group
            sc = (k[:, kh, :] @ q[s, h]) * scale
            sc -= sc.max()
            p = np.exp(sc)
            out[s, h] = (p @ v[:, kh, :]) / p.sum()
    return out


def decode_slots(block_tables: Sequence[Sequence[int]], seq_lens: Sequence[int], block_size: int) -> np.ndarray:
    """Slot of the token a decode step writes for each sequence, whose
    ``seq_len`` already counts that token (integration.py:150-155); -1 (no
    write) for a sequence of length 0, which holds no token (the reference's
    decode step never sees one: it bumps the length before the write)."""
    slots = np.empty(len(seq_lens), dtype=np.int64)
    for b, n in enumerate(seq_lens):
        pos = int(n) - 1
        if pos < 0:
            slots[b] = -1
            continue
        slots[b] = int(block_tables[b][pos // block_size]) * block_size + pos % block_size
    return slots


def kv_append_ref(
    k_cache: np.ndarray,
    v_cache: np.ndarray,
    k_new: np.ndarray,
    v_new: np.ndarray,
    slot_mapping: np.ndarray,
) -> None:
    """In place: k_cache[slot // BS, slot % BS] = k_new[i] (and V) for every
    token with slot >= 0 (integration.py:159-160). Arrays are numpy views of
    the pool; 16-bit payloads are copied as raw bits."""
    block_size = k_cache.shape[1]
    for i, slot in enumerate(np.asarray(slot_mapping, dtype=np.int64)):
        if slot < 0:
            continue
        k_cache[slot // block_size, slot % block_size] = k_new[i]
        v_cache[slot // block_size, slot % block_size] = v_new[i]


def copy_blocks_ref(
    k_caches: Sequence[np.ndarray],
    v_caches: Sequence[np.ndarray],
    block_mapping: np.ndarray,
) -> None:
    """In place: pool[l][dst] = pool[l][src] for every (src, dst) pair and
    every layer, K and V."""
    for src, dst in np.asarray(block_mapping, dtype=np.int64).reshape(-1, 2):
        for kc, vc in zip(k_caches, v_caches):
            kc[dst] = kc[src]
            vc[dst] = vc[src]


def rope_ref(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotary embedding as transformers' apply_rotary_pos_emb computes it for
    one decode token (used at paged_attention_integration.py:108-109):
    ``x * cos + rotate_half(x) * sin`` with rotate_half(x) = cat(-x2, x1), as
    16-bit tensor ops (each product and the sum rounded to the dtype).
    x: [tokens, heads, D]; cos / sin: [tokens, D]."""
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return (x * cos[:, None, :]) + (rot * sin[:, None, :])


def prefill_write_ref(
    k_caches: Sequence[torch.Tensor],
    v_caches: Sequence[torch.Tensor],
    k_srcs: Sequence[torch.Tensor],
    v_srcs: Sequence[torch.Tensor],
    block_ids: Sequence[int],
    num_tokens: int,
) -> None:
    """In place, restating KernelPagedManualDecode._copy_prefill_kv
    (paged_attention_integration.py:305-326): the [num_tokens, Hkv, D] source
    rows are zero-padded to whole blocks (:315-317), converted to the pool
    dtype (:319-320, torch .to: round to nearest even) and index_copy_'d into
    blocks ``block_ids`` of every layer's K and V pool (:322-323)."""
    bs, hkv, d = k_caches[0].shape[1:]
    nw = len(block_ids)
    pad = nw * bs - num_tokens
    ids = torch.tensor(list(block_ids), dtype=torch.long, device=k_caches[0].device)
    for kc, vc, ks, vs in zip(k_caches, v_caches, k_srcs, v_srcs):
        k_src, v_src = ks[:num_tokens], vs[:num_tokens]
        if pad > 0:
            k_src = torch.nn.functional.pad(k_src, (0, 0, 0, 0, 0, pad))
            v_src = torch.nn.functional.pad(v_src, (0, 0, 0, 0, 0, pad))
        kc.index_copy_(0, ids, k_src.reshape(nw, bs, hkv, d).to(kc.dtype))
        vc.index_copy_(0, ids, v_src.reshape(nw, bs, hkv, d).to(vc.dtype))


def time_paged_attention_cpu(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: Sequence[Sequence[int]],
    seq_lens: Sequence[int],
    scale: float,
    threads: int,
) -> float:
    """Seconds for one ``paged_attention_ref`` call on ``threads`` host threads
    (the CPU baseline of the benchmark)."""
    import time

    prev = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        t0 = time.perf_counter()
        paged_attention_ref(q, k_cache, v_cache, block_tables, seq_lens, scale)
        return time.perf_counter() - t0
    finally:
        torch.set_num_threads(prev)
