"""Host-side drop-in for the reference engine's decode path.

The reference imports its kernels by name (engine/kernels/
paged_attention_integration.py:19-23) and runs one Python loop per sequence
per layer for the KV append, with a device->host ``.item()`` sync in each
iteration (:150-160). This module provides:

* :func:`install` — put the B200 kernels in place of the reference's symbols
  in ``engine.kernels.paged_attention`` and
  ``engine.kernels.paged_attention_integration`` (and their batched decode
  forward / context), so ``KernelPagedManualDecode``, the continuous-batching
  scheduler, ``AsyncEngine`` and the HTTP server run unchanged on top;
* :class:`PagedAttentionContext` — same constructor as the reference's
  (:29-62); additionally builds the int64 ``slot_mapping`` of the token each
  sequence writes this step, with ONE host->device copy for tables, lengths
  and slots together;
* :func:`paged_decode_attention_forward` — the reference's decode forward
  (:65-176) with the append done by :func:`pagedkv.kv_append` (one launch per
  layer, no host sync) and attention by the sm_100a kernel;
* :func:`prepare_copy_on_write` — the block bookkeeping of a copy-on-write
  append (fresh block for every sequence whose write block is shared), whose
  data copy :func:`pagedkv.copy_blocks` performs for all layers at once;
* :func:`decode_step` — the runner's batched decode step with its
  per-sequence host syncs batched (installed over
  ``KernelPagedManualDecode.decode_step``).
"""
from __future__ import annotations

import math
import weakref
from contextlib import contextmanager
from typing import Any, Dict, Iterable, List, Optional, Sequence, Tuple, Union

import torch

from . import prefix_index
from .paged_attention import (
    copy_blocks,
    paged_attention_decode_append,
    kv_append_rope,
    kv_write_prefill,
    pad_block_tables,
    paged_attention_decode,
    paged_attention_decode_batched,
    paged_attention_decode_v1,
    paged_attention_decode_v2,
)


def _block_ids(bt: Any) -> List[int]:
    return list(bt.physical_block_ids) if hasattr(bt, "physical_block_ids") else list(bt)


def build_decode_metadata(
    block_tables: Sequence[Any],
    seq_lens: Sequence[int],
    block_size: int,
    device: Union[torch.device, str],
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Padded int32 tables [N, max(1, W)], int32 seq_lens [N] and int64
    slot_mapping [N] on ``device`` from one pinned host buffer.

    The slot of sequence b is the position its decode step writes,
    ``table[(len - 1) // BS] * BS + (len - 1) % BS`` (reference
    integration.py:151-155); a sequence of length 0 gets slot -1 (skipped).
    """
    n = len(block_tables)
    rows = [_block_ids(bt) for bt in block_tables]
    width = max(1, max((len(r) for r in rows), default=0))
    # int64 host image: [tables (n*width) | lens (n) | slots (n)]
    host = torch.zeros(n * width + 2 * n, dtype=torch.int64)
    tab = host[: n * width].view(n, width)
    for i, r in enumerate(rows):
        if r:
            tab[i, : len(r)] = torch.tensor(r, dtype=torch.int64)
    lens = torch.tensor([int(x) for x in seq_lens], dtype=torch.int64)
    host[n * width : n * width + n] = lens
    pos = lens - 1
    slots = torch.full((n,), -1, dtype=torch.int64)
    has = pos >= 0
    if bool(has.any()):
        idx = torch.nonzero(has).view(-1)
        blk = tab[idx, pos[idx] // block_size]
        slots[idx] = blk * block_size + pos[idx] % block_size
    host[n * width + n :] = slots
    dev = torch.device(device)
    if dev.type == "cuda":
        d = host.pin_memory().to(dev, non_blocking=True)
    else:
        d = host.to(dev)
    tables_d = d[: n * width].view(n, width).to(torch.int32)
    lens_d = d[n * width : n * width + n].to(torch.int32)
    slots_d = d[n * width + n :]
    return tables_d, lens_d, slots_d


class PagedAttentionContext:
    """Per-step context passed to the patched attention modules.

    Constructor and attributes as the reference's (integration.py:29-62):
    ``pool``, ``block_size``, ``is_decode``, ``is_batched``; batched:
    ``block_table_list``, ``padded_block_tables``, ``seq_lens_tensor``;
    single: ``single_block_table``, ``single_seq_len``, ``block_table_tensor``.
    Added: ``slot_mapping`` (int64 [N]) for the one-launch append.
    """

    def __init__(
        self,
        pool: Any,
        block_tables: Any,
        seq_lens: Union[int, List[int], torch.Tensor],
        block_size: int = 16,
        is_decode: bool = True,
    ):
        self.pool = pool
        self.block_size = block_size
        self.is_decode = is_decode
        device = pool.device
        if hasattr(block_tables, "physical_block_ids") and not isinstance(block_tables, (list, tuple)):
            self.is_batched = False
            self.single_block_table = block_tables
            self.single_seq_len = int(seq_lens)
            tables, lens, slots = build_decode_metadata([block_tables], [self.single_seq_len], block_size, device)
            self.block_table_tensor = tables[0, : max(1, len(block_tables.physical_block_ids))]
            self.padded_block_tables = tables
            self.seq_lens_tensor = lens
            self.slot_mapping = slots
        else:
            self.is_batched = True
            self.block_table_list = block_tables
            if isinstance(seq_lens, torch.Tensor):
                seq_lens = [int(x) for x in seq_lens.tolist()]
            tables, lens, slots = build_decode_metadata(block_tables, list(seq_lens), block_size, device)
            self.padded_block_tables = tables
            self.seq_lens_tensor = lens
            self.slot_mapping = slots


def paged_decode_attention_forward(
    self: torch.nn.Module,
    hidden_states: torch.Tensor,
    position_embeddings: Tuple[torch.Tensor, torch.Tensor],
    attention_mask: Optional[torch.Tensor] = None,
    past_key_values: Any = None,
    **kwargs: Any,
) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Decode-step replacement for ``Qwen2Attention.forward`` (reference
    integration.py:65-176): projections, RoPE fused with the KV append through
    the slot mapping (one launch per layer), batched paged attention, o_proj."""
    ctx = getattr(self, "_paged_attention_context", None)
    if ctx is None:
        holder = getattr(self, "_pagedkv_context_holder", None)
        ctx = holder.ctx if holder is not None else None
    if ctx is None or not ctx.is_decode:
        orig_forward = getattr(self, "_orig_attention_forward", None)
        if orig_forward is not None:
            return orig_forward(
                hidden_states=hidden_states,
                position_embeddings=position_embeddings,
                attention_mask=attention_mask,
                past_key_values=past_key_values,
                **kwargs,
            )
        raise RuntimeError("No fallback forward method found on attention module.")

    layer_idx = self.layer_idx
    input_shape = hidden_states.shape[:-1]
    hidden_shape = (*input_shape, -1, self.head_dim)
    # [B, 1, H * D] -> [B, H, D] views (one decode token per sequence)
    query_states = self.q_proj(hidden_states).view(hidden_shape)[:, 0]
    key_states = self.k_proj(hidden_states).view(hidden_shape)[:, 0]
    value_states = self.v_proj(hidden_states).view(hidden_shape)[:, 0]
    cos, sin = position_embeddings  # [B, 1, D]
    scale = self.scaling if hasattr(self, "scaling") else 1.0 / math.sqrt(self.head_dim)

    pool = ctx.pool
    k_cache = pool.k_cache[layer_idx]
    v_cache = pool.v_cache[layer_idx]
    # RoPE on q and k and the append of k and v fused into the attention
    # launch: one kernel instead of the rotary tensor ops, the append loop and
    # the attention kernel.
    bsz = query_states.shape[0]
    cos2 = cos.reshape(-1, cos.shape[-1])  # [B, 1, D] (or a broadcast [1, 1, D]) -> rows
    sin2 = sin.reshape(-1, sin.shape[-1])
    if cos2.shape[0] != bsz:
        cos2, sin2 = cos2.expand(bsz, -1), sin2.expand(bsz, -1)
    attn_output = paged_attention_decode_append(
        query_states, k_cache, v_cache, ctx.padded_block_tables, ctx.seq_lens_tensor, scale,
        key_states, value_states, cos2, sin2, slot_mapping=ctx.slot_mapping,
    )
    attn_output = attn_output.reshape(*input_shape, -1).contiguous()
    attn_output = self.o_proj(attn_output)
    return attn_output, None


class _ContextHolder:
    """The decode context every patched attention module of one model reads;
    ``None`` outside a decode step (the modules then run their own forward)."""

    __slots__ = ("ctx",)

    def __init__(self) -> None:
        self.ctx: Optional[PagedAttentionContext] = None


# Models whose attention modules are routed through the paged forward.
_attached: "weakref.WeakSet[torch.nn.Module]" = weakref.WeakSet()


def _is_attention(module: torch.nn.Module) -> bool:
    return all(hasattr(module, a) for a in ("q_proj", "k_proj", "v_proj", "o_proj"))


def attach_paged_attention(model: torch.nn.Module) -> _ContextHolder:
    """Route every decoder attention module of ``model`` through
    :func:`paged_decode_attention_forward`, once per model, and return the
    holder whose ``ctx`` selects the paged path.

    The reference rebinds ``forward`` on every attention module at every
    decode step and restores it afterwards (integration.py:179-208, used at
    :629-634). Here the binding is made on first use and kept: a step only
    stores its context in the holder (one assignment), and with no context
    the modules fall back to their original forward (prefill, generation
    outside the runner), as the reference's patched forward does."""
    holder = getattr(model, "_pagedkv_context_holder", None)
    if holder is not None:
        return holder
    holder = _ContextHolder()
    for module in model.modules():
        if _is_attention(module) and not hasattr(module, "_pagedkv_context_holder"):
            module._orig_attention_forward = module.forward
            module._pagedkv_own_forward = "forward" in module.__dict__
            module._pagedkv_context_holder = holder
            module.forward = paged_decode_attention_forward.__get__(module, module.__class__)
    model._pagedkv_context_holder = holder
    _attached.add(model)
    return holder


def detach_paged_attention(model: torch.nn.Module) -> None:
    """Undo :func:`attach_paged_attention` (restore every module's forward)."""
    for module in model.modules():
        if module is not model and getattr(module, "_pagedkv_context_holder", None) is not None:
            if module.__dict__.get("_pagedkv_own_forward"):
                module.forward = module._orig_attention_forward
            else:
                del module.__dict__["forward"]
            for attr in ("_orig_attention_forward", "_pagedkv_context_holder", "_pagedkv_own_forward"):
                if attr in module.__dict__:
                    delattr(module, attr)
    if "_pagedkv_context_holder" in model.__dict__:
        delattr(model, "_pagedkv_context_holder")
    _attached.discard(model)


@contextmanager
def patch_paged_attention(model: torch.nn.Module, context: PagedAttentionContext):
    """Route the decoder attention modules of ``model`` through
    :func:`paged_decode_attention_forward` with ``context`` for the duration
    of the block (reference integration.py:179-208). The modules are bound
    once (:func:`attach_paged_attention`); entering and leaving the block only
    swaps the context."""
    holder = attach_paged_attention(model)
    prev = holder.ctx
    holder.ctx = context
    try:
        yield context
    finally:
        holder.ctx = prev


def _seq_field(seq: Any, name: str, default: Any = None) -> Any:
    if hasattr(seq, name):
        return getattr(seq, name)
    if isinstance(seq, dict):
        return seq.get(name, default)
    return default


def _bucket(n: int, cap: Optional[int] = None) -> int:
    b = 1
    while b < n:
        b *= 2
    return b if cap is None else min(b, cap)


def _graphable(model: Any) -> bool:
    """The decode forward can be replayed layer by layer from a CUDA graph:
    a Qwen2-architecture causal LM (embed / rotary / layers / norm / lm_head,
    attention with q/k/v/o projections) on a CUDA device."""
    cfg = getattr(model, "config", None)
    inner = getattr(model, "model", None)
    if cfg is None or inner is None or getattr(cfg, "model_type", None) != "qwen2":
        return False
    if not all(hasattr(inner, a) for a in ("embed_tokens", "rotary_emb", "layers", "norm")):
        return False
    if not hasattr(model, "lm_head"):
        return False
    try:
        dev = next(model.parameters()).device
    except StopIteration:
        return False
    return dev.type == "cuda"


class DecodeGraphs:
    """CUDA graphs of one runner's decode forward, one per (padded batch,
    padded table width).

    The forward is the one the reference runs through the patched model
    (integration.py:621-640): embedding, rotary table, and per layer input
    norm, q/k/v projections, RoPE fused with the KV append through the slot
    mapping, batched paged attention, o_proj and residual, post-attention norm,
    MLP and residual; then the final norm, ``lm_head``, the greedy token and
    the top-2 logit margin. The same module calls in the same order as the HF
    decoder layer, so the logits are those of the patched forward. Inputs live
    in two static device buffers per graph (int64 [B, 3]: token, position,
    slot; int32 [B, 1 + W]: length, block table) filled by one host-to-device
    copy each per step; padding rows have length 0 and slot -1 (no write,
    zero attention output)."""

    def __init__(self, model: Any, pool: Any) -> None:
        self.model = model
        self.pool = pool
        self.dev = next(model.parameters()).device
        self.graphs: Dict[Tuple[int, int], tuple] = {}
        self.mempool = torch.cuda.graph_pool_handle()

    def _forward(self, m64: torch.Tensor, m32: torch.Tensor):
        m = self.model.model
        ids, pos, slots = m64[:, 0], m64[:, 1], m64[:, 2]
        lens, tables = m32[:, 0], m32[:, 1:]
        b = ids.shape[0]
        x = m.embed_tokens(ids[:, None])
        cos, sin = m.rotary_emb(x, pos[:, None])
        cos2, sin2 = cos[:, 0], sin[:, 0]
        k_caches, v_caches = self.pool.k_cache, self.pool.v_cache
        for li, layer in enumerate(m.layers):
            attn = layer.self_attn
            residual = x
            h = layer.input_layernorm(x)
            q = attn.q_proj(h).view(b, -1, attn.head_dim)
            k = attn.k_proj(h).view(b, -1, attn.head_dim)
            v = attn.v_proj(h).view(b, -1, attn.head_dim)
            scale = attn.scaling if hasattr(attn, "scaling") else 1.0 / math.sqrt(attn.head_dim)
            li_pool = attn.layer_idx if hasattr(attn, "layer_idx") else li
            o = paged_attention_decode_append(q, k_caches[li_pool], v_caches[li_pool], tables, lens, scale, k, v,
                                              cos2, sin2, slot_mapping=slots)
            x = residual + attn.o_proj(o.reshape(b, 1, -1).contiguous())
            residual = x
            x = residual + layer.mlp(layer.post_attention_layernorm(x))
        x = m.norm(x)
        logits = self.model.lm_head(x[:, -1, :])
        top2 = torch.topk(logits, k=2, dim=-1).values
        return logits, torch.argmax(logits, dim=-1), top2[:, 0] - top2[:, 1]

    def get(self, bsz: int, width: int) -> tuple:
        key = (bsz, width)
        hit = self.graphs.get(key)
        if hit is None:
            m64 = torch.zeros(bsz, 3, dtype=torch.int64, device=self.dev)
            m64[:, 2] = -1
            m32 = torch.zeros(bsz, 1 + width, dtype=torch.int32, device=self.dev)
            h64 = torch.zeros(bsz, 3, dtype=torch.int64).pin_memory()
            h32 = torch.zeros(bsz, 1 + width, dtype=torch.int32).pin_memory()
            # Every row is padding here (length 0, slot -1): the warm-up and the
            # capture write nothing into the pool. The warm-up runs size the
            # kernels' cached workspace before capture.
            for _ in range(2):
                self._forward(m64, m32)
            torch.cuda.synchronize(self.dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=self.mempool):
                outs = self._forward(m64, m32)
            hit = (g, m64, m32, h64, h32, outs)
            self.graphs[key] = hit
        return hit


@torch.inference_mode()
def decode_step(self: Any, seqs: List[Any], allocator: Any = None) -> List[int]:
    """``KernelPagedManualDecode.decode_step`` (integration.py:519-651) with the
    same bookkeeping, asserts and results, its host synchronisation batched
    and, for a Qwen2 model on a CUDA device, its forward replayed from a CUDA
    graph per padded batch size and table width.

    Per sequence, as the reference: the write slot is block
    ``num_tokens // block_size`` of its table, which must exist and must not be
    shared (ref count > 1); ``num_tokens`` is bumped by one; the input token is
    ``last_token_id`` (else the last of ``generated_ids``). One forward through
    the paged attention gives the greedy next tokens. The diagnostics the
    reference stores per sequence (``last_logits`` on the host and
    ``last_logit_margin`` = top-1 minus top-2 logit, in the logits' dtype) come
    from one top-2 over the batch and two device-to-host copies in all, instead
    of a ``.cpu()``, a ``topk`` and an ``.item()`` sync per sequence; each
    ``last_logits`` is a row of one host tensor of the batch's logits.

    With copy-on-write enabled (``install(copy_on_write=True)``, or the
    runner attribute ``_pagedkv_copy_on_write``), a write block shared with
    another sequence is first copied to a fresh block for this sequence
    (:func:`prepare_copy_on_write` + one :func:`pagedkv.copy_blocks` launch for
    all layers) instead of failing the reference's shared-block assert.
    """
    n = len(seqs)
    if n == 0:
        return []
    allocator = allocator or self.allocator
    tables_bt: List[Any] = []
    for seq in seqs:
        bt = _seq_field(seq, "block_table")
        if bt is None:
            raise ValueError("Sequence must provide a block_table attribute or dict key.")
        tables_bt.append(bt)
    if getattr(self, "_pagedkv_copy_on_write", False):
        copy_on_write(self.pool, prepare_copy_on_write(tables_bt, allocator, self.block_size))
    seq_lens: List[int] = []
    last_tokens: List[int] = []
    for seq, bt in zip(seqs, tables_bt):
        write_idx = bt.num_tokens // self.block_size
        if write_idx >= len(bt.physical_block_ids):
            raise AssertionError(
                f"Decode write for seq {_seq_field(seq, 'seq_id', '?')} has no allocated block "
                f"at logical index {write_idx}."
            )
        write_block = bt.physical_block_ids[write_idx]
        if allocator.ref_counts.get(write_block, 0) > 1:
            raise AssertionError(
                f"Decode write for seq {_seq_field(seq, 'seq_id', '?')} would modify shared "
                f"block {write_block} with ref_count {allocator.ref_counts[write_block]}."
            )
        bt.num_tokens += 1
        seq_lens.append(bt.num_tokens)
        tok = _seq_field(seq, "last_token_id")
        if tok is None:
            gen = _seq_field(seq, "generated_ids")
            if not gen:
                raise ValueError("Sequence must provide last_token_id or non-empty generated_ids.")
            tok = gen[-1]
        last_tokens.append(int(tok))

    use_graphs = getattr(self, "_pagedkv_cuda_graphs", False) and _graphable(self.model)
    if use_graphs:
        graphs = self.__dict__.get("_pagedkv_graphs")
        if graphs is None or graphs.model is not self.model or graphs.pool is not self.pool:
            graphs = DecodeGraphs(self.model, self.pool)
            self._pagedkv_graphs = graphs
        width = max(len(bt.physical_block_ids) for bt in tables_bt)
        g, m64, m32, h64, h32, (logits_s, next_s, margin_s) = graphs.get(_bucket(n), _bucket(max(1, width)))
        bs = self.block_size
        h64.zero_()
        h32.zero_()
        h64[:, 2] = -1
        a64, a32 = h64.numpy(), h32.numpy()
        for i, (bt, L, tok) in enumerate(zip(tables_bt, seq_lens, last_tokens)):
            ids = bt.physical_block_ids
            a64[i, 0] = tok
            a64[i, 1] = L - 1
            a64[i, 2] = ids[(L - 1) // bs] * bs + (L - 1) % bs
            a32[i, 0] = L
            a32[i, 1 : 1 + len(ids)] = ids
        m64.copy_(h64, non_blocking=True)
        m32.copy_(h32, non_blocking=True)
        g.replay()
        logits, next_t, margin = logits_s[:n], next_s[:n], margin_s[:n]
    else:
        # token ids and positions in one host->device copy
        host = torch.tensor([last_tokens, [s - 1 for s in seq_lens]], dtype=torch.long)
        if torch.device(self.device).type == "cuda":
            host = host.pin_memory()
        dev_ids = host.to(self.device, non_blocking=True)
        input_ids, position_ids = dev_ids[0].unsqueeze(1), dev_ids[1].unsqueeze(1)
        ctx = PagedAttentionContext(pool=self.pool, block_tables=tables_bt, seq_lens=seq_lens,
                                    block_size=self.block_size, is_decode=True)
        with patch_paged_attention(self.model, ctx):
            step_out = self.model(input_ids=input_ids, position_ids=position_ids, use_cache=False)
        logits = step_out.logits[:, -1, :]
        next_t = torch.argmax(logits, dim=-1)
        margin = None
    want = [i for i, s in enumerate(seqs) if hasattr(s, "last_logits") or isinstance(s, dict)]
    if not want:
        return next_t.tolist()
    if margin is None:
        top2 = torch.topk(logits, k=2, dim=-1).values
        margin = top2[:, 0] - top2[:, 1]  # in the logits' dtype, as the reference's per-row difference
    # float64 holds every token id and every 16/32-bit margin exactly
    packed = torch.cat([next_t.to(torch.float64), margin.to(torch.float64)]).tolist()
    host_logits = logits.detach().cpu()
    for i in want:
        seq = seqs[i]
        if hasattr(seq, "last_logits"):
            seq.last_logits = host_logits[i]
            seq.last_logit_margin = float(packed[n + i])
        else:
            seq["last_logits"] = host_logits[i]
            seq["last_logit_margin"] = float(packed[n + i])
    return [int(x) for x in packed[:n]]


def prepare_copy_on_write(
    block_tables: Iterable[Any],
    allocator: Any,
    block_size: int,
) -> List[Tuple[int, int]]:
    """Give every sequence whose next write lands in a shared block a private
    copy of that block; return the (src, dst) pairs for :func:`copy_blocks`.

    For each table (an object with ``physical_block_ids`` and ``num_tokens``,
    as the reference's ``BlockTable``), the write block is
    ``num_tokens // block_size`` (reference integration.py:580). If the
    allocator's ``ref_counts`` for it is above 1, a fresh block is allocated,
    the table is pointed at it and one reference on the shared block is
    dropped (``release`` when the allocator has it, else ``free``, as the
    reference allocator's API at block_allocator.py:216-270). The data copy
    itself must then run before the step's append.
    """
    pairs: List[Tuple[int, int]] = []
    release = getattr(allocator, "release", None) or allocator.free
    for bt in block_tables:
        idx = bt.num_tokens // block_size
        if idx >= len(bt.physical_block_ids):
            continue
        src = bt.physical_block_ids[idx]
        if allocator.ref_counts.get(src, 0) > 1:
            dst = allocator.allocate()
            bt.physical_block_ids[idx] = dst
            release(src)
            pairs.append((src, dst))
    return pairs


def copy_on_write(pool: Any, pairs: Sequence[Tuple[int, int]]) -> None:
    """Run the data copies of :func:`prepare_copy_on_write` for every layer of
    ``pool`` (an object with ``k_cache`` / ``v_cache`` lists) in one launch."""
    if not pairs:
        return
    dev = pool.k_cache[0].device
    mapping = torch.tensor(list(pairs), dtype=torch.int64).to(dev)
    copy_blocks(pool.k_cache, pool.v_cache, mapping)


def _layer_kv(pkv: Any, layer: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """(keys, values) [batch, kv_heads, tokens, head_dim] of one layer of a
    prefill cache, in either layout the reference reads (integration.py:308-313)."""
    if hasattr(pkv, "layers"):
        return pkv.layers[layer].keys, pkv.layers[layer].values
    return pkv[layer][0], pkv[layer][1]


def copy_prefill_kv(self: Any, pkv: Any, block_table: Any, prompt_len: int, skip_blocks: int = 0) -> None:
    """Drop-in for ``KernelPagedManualDecode._copy_prefill_kv``
    (integration.py:278-326): write the prompt's K/V from token
    ``skip_blocks * block_size`` on into blocks ``[skip_blocks,
    ceil(prompt_len / block_size))`` of the sequence's table, zero-padding the
    last block's tail, for every layer in ONE launch (the reference pads and
    runs two ``index_copy_`` per layer). Blocks before ``skip_blocks`` (prefix
    cache hits) are not touched; nothing is allocated here."""
    bs = self.block_size
    start_token = skip_blocks * bs
    if start_token >= prompt_len:
        return
    total_blocks = (prompt_len + bs - 1) // bs
    blocks_to_write = total_blocks - skip_blocks
    if blocks_to_write <= 0:
        return
    k_caches, v_caches = self.pool.k_cache, self.pool.v_cache
    dev = k_caches[0].device
    ids = torch.tensor(block_table.physical_block_ids[skip_blocks:total_blocks], dtype=torch.int64).to(dev)
    k_srcs, v_srcs = [], []
    for layer in range(len(k_caches)):
        keys, values = _layer_kv(pkv, layer)
        k = keys[0, :, start_token:prompt_len, :].permute(1, 0, 2)
        v = values[0, :, start_token:prompt_len, :].permute(1, 0, 2)
        if k.dtype not in (k_caches[0].dtype, torch.float32):
            k, v = k.to(k_caches[0].dtype), v.to(k_caches[0].dtype)
        if k.stride(2) != 1 or v.stride() != k.stride():
            k, v = k.contiguous(), v.contiguous()
        k_srcs.append(k)
        v_srcs.append(v)
    kv_write_prefill(k_srcs, v_srcs, k_caches, v_caches, ids, prompt_len - start_token)


_INSTALL_NAMES_KERNELS = (
    "paged_attention_decode_batched",
    "paged_attention_decode_v1",
    "paged_attention_decode_v2",
    "paged_attention_decode",
    "pad_block_tables",
)


_MISSING = object()


def install(paged_attention_module: Any = None, integration_module: Any = None,
            allocator_module: Any = None, *, copy_on_write: bool = False,
            cuda_graphs: bool = True) -> dict:
    """Install the B200 path into the reference's modules.

    ``paged_attention_module`` defaults to ``engine.kernels.paged_attention``,
    ``integration_module`` to ``engine.kernels.paged_attention_integration`` and
    ``allocator_module`` to ``engine.memory.block_allocator`` (imported if not
    given; the allocator is skipped when it cannot be imported). Returns the
    replaced symbols for :func:`uninstall`. The reference's
    ``naive_reference_paged_attention`` is left untouched.

    ``copy_on_write``: the installed ``decode_step`` copies a shared write
    block to a fresh block (for all layers, one launch) instead of raising the
    reference's shared-block ``AssertionError`` (integration.py:587-592); off
    by default, which keeps the reference's behaviour. ``cuda_graphs``: the
    installed ``decode_step`` replays its forward from a CUDA graph per padded
    batch size and table width when the runner's model is a Qwen2 causal LM on
    a CUDA device (:class:`DecodeGraphs`); otherwise, or when off, it runs the
    model eagerly with the attention modules bound once
    (:func:`attach_paged_attention`).
    """
    if paged_attention_module is None:
        import importlib

        paged_attention_module = importlib.import_module("engine.kernels.paged_attention")
    if integration_module is None:
        import importlib

        integration_module = importlib.import_module("engine.kernels.paged_attention_integration")
    ours = {
        "paged_attention_decode_batched": paged_attention_decode_batched,
        "paged_attention_decode_v1": paged_attention_decode_v1,
        "paged_attention_decode_v2": paged_attention_decode_v2,
        "paged_attention_decode": paged_attention_decode,
        "pad_block_tables": pad_block_tables,
        "PagedAttentionContext": PagedAttentionContext,
        "paged_decode_attention_forward": paged_decode_attention_forward,
        "patch_paged_attention": patch_paged_attention,
    }
    saved: dict = {}
    for mod in (paged_attention_module, integration_module):
        for name, fn in ours.items():
            if hasattr(mod, name):
                saved[(mod, name)] = getattr(mod, name)
                setattr(mod, name, fn)
    # The runner's prefill write and decode step (methods, patched on the class).
    runner_cls = getattr(integration_module, "KernelPagedManualDecode", None)
    for name, fn in (("_copy_prefill_kv", copy_prefill_kv), ("decode_step", decode_step)):
        if runner_cls is not None and hasattr(runner_cls, name):
            saved[(runner_cls, name)] = runner_cls.__dict__.get(name, getattr(runner_cls, name))
            setattr(runner_cls, name, fn)
    if runner_cls is not None:
        for name, value in (("_pagedkv_copy_on_write", bool(copy_on_write)),
                            ("_pagedkv_cuda_graphs", bool(cuda_graphs))):
            saved[(runner_cls, name)] = runner_cls.__dict__.get(name, _MISSING)
            setattr(runner_cls, name, value)
    # The allocator's prefix lookup: a per-parent index instead of a full scan
    # of the cache per block (block_allocator.py:231-252).
    if allocator_module is None:
        try:
            import importlib

            allocator_module = importlib.import_module("engine.memory.block_allocator")
        except ImportError:
            allocator_module = None
    alloc_cls = getattr(allocator_module, "BlockAllocator", None)
    if alloc_cls is not None and "lookup_prefix" in alloc_cls.__dict__:
        saved[("prefix_index", alloc_cls)] = prefix_index.install(alloc_cls)
    return saved


def uninstall(saved: dict) -> None:
    """Undo :func:`install`."""
    for (mod, name), fn in saved.items():
        if mod == "prefix_index":
            prefix_index.uninstall(fn)
        elif fn is _MISSING:
            if name in getattr(mod, "__dict__", {}):
                delattr(mod, name)
        else:
            setattr(mod, name, fn)
    for model in list(_attached):
        detach_paged_attention(model)
