"""Continuous-batching decode runner for a Qwen2-architecture model on the paged path.

The caller of the hot path at model level (the role of the reference's
``KernelPagedManualDecode`` + scheduler, engine/kernels/paged_attention_integration.py
and engine/scheduler/continuous_batching.py, reduced to what a decode benchmark
needs): a per-layer paged K/V pool, a free-list block allocator, prefill through
the Hugging Face model followed by ONE prefill-write launch for all layers
(:func:`pagedkv.kv_write_prefill`), and decode steps in which every layer runs
the fused RoPE + append (:func:`pagedkv.kv_append_rope`) and the batched paged
attention (:func:`pagedkv.paged_attention_decode_batched`) around the model's own
projections, norms and MLP. A decode step for a padded batch size is captured
once as a CUDA graph and replayed; padding rows have length 0 (zero output) and
slot -1 (no write).

Greedy sampling; every request owns ``ceil((prompt + max_new) / block_size)``
blocks from admission to completion (no preemption). Prompts run right-padded
to a multiple of ``prefill_bucket`` tokens (causal attention: the padding never
reaches the real tokens' K/V or the last real token's logits), so the model
sees a handful of prefill shapes instead of one per prompt length.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

from .paged_attention import kv_write_prefill, paged_attention_decode_append


@dataclass
class Sequence_:
    """One request in flight: its block table, length and generated tokens."""

    seq_id: int
    prompt_len: int
    max_new_tokens: int
    blocks: List[int]
    num_tokens: int            # tokens whose K/V are in the pool
    last_token: int            # token to feed to the next decode step
    generated: List[int] = field(default_factory=list)
    block_row: Optional[np.ndarray] = None  # blocks, zero-padded to the table width

    @property
    def done(self) -> bool:
        return len(self.generated) >= self.max_new_tokens


def _bucket(n: int, max_batch: int) -> int:
    b = 1
    while b < n:
        b *= 2
    return min(b, max_batch)


class PagedDecodeRunner:
    """Decode runner over a Hugging Face ``Qwen2ForCausalLM`` (fp16/bf16, CUDA)."""

    def __init__(self, model: torch.nn.Module, num_blocks: int, block_size: int = 16,
                 max_batch: int = 256, max_seq_len: int = 2048, use_graphs: bool = True,
                 prefill_bucket: int = 64):
        cfg = model.config
        self.model = model
        self.dev = next(model.parameters()).device
        self.dtype = next(model.parameters()).dtype
        assert self.dev.type == "cuda" and self.dtype in (torch.float16, torch.bfloat16)
        self.num_layers = cfg.num_hidden_layers
        self.hq = cfg.num_attention_heads
        self.hkv = cfg.num_key_value_heads
        self.head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        self.block_size = block_size
        self.num_blocks = num_blocks
        self.max_batch = max_batch
        self.max_blocks_per_seq = (max_seq_len + block_size - 1) // block_size
        shape = (num_blocks, block_size, self.hkv, self.head_dim)
        self.k_cache = [torch.empty(shape, dtype=self.dtype, device=self.dev) for _ in range(self.num_layers)]
        self.v_cache = [torch.empty(shape, dtype=self.dtype, device=self.dev) for _ in range(self.num_layers)]
        self.free: List[int] = list(range(num_blocks - 1, -1, -1))
        self.use_graphs = use_graphs
        self.prefill_bucket = max(1, prefill_bucket)
        self._graphs: Dict[int, tuple] = {}
        self._host: Dict[int, tuple] = {}
        self._next_id = 0
        # When a list: (start, end) CUDA events around every decode-graph replay.
        self.timing: Optional[list] = None

    # ---- allocator -------------------------------------------------------------
    def can_admit(self, prompt_len: int, max_new_tokens: int) -> bool:
        need = (prompt_len + max_new_tokens + self.block_size - 1) // self.block_size
        return need <= len(self.free) and need <= self.max_blocks_per_seq

    def _allocate(self, n: int) -> List[int]:
        assert n <= len(self.free), "KV pool exhausted"
        return [self.free.pop() for _ in range(n)]

    def release(self, seq: Sequence_) -> None:
        self.free.extend(reversed(seq.blocks))
        seq.blocks = []

    # ---- prefill ---------------------------------------------------------------
    @torch.inference_mode()
    @torch.cuda.nvtx.range("pagedkv.prefill")
    def prefill(self, prompt_ids: Sequence[int], max_new_tokens: int) -> Sequence_:
        """Run the prompt through the model, write its K/V into freshly
        allocated blocks of every layer (one launch) and sample the first token."""
        p = len(prompt_ids)
        need = (p + max_new_tokens + self.block_size - 1) // self.block_size
        blocks = self._allocate(need)
        padded = (p + self.prefill_bucket - 1) // self.prefill_bucket * self.prefill_bucket
        ids = torch.zeros((1, padded), dtype=torch.long)
        ids[0, :p] = torch.tensor(list(prompt_ids), dtype=torch.long)
        out = self.model(input_ids=ids.to(self.dev, non_blocking=True), use_cache=True,
                         logits_to_keep=torch.tensor([p - 1], device=self.dev))
        pkv = out.past_key_values
        nblk = (p + self.block_size - 1) // self.block_size
        k_srcs, v_srcs = [], []
        for layer in range(self.num_layers):
            lk = pkv.layers[layer].keys if hasattr(pkv, "layers") else pkv[layer][0]
            lv = pkv.layers[layer].values if hasattr(pkv, "layers") else pkv[layer][1]
            k_srcs.append(lk[0, :, :p, :].permute(1, 0, 2))
            v_srcs.append(lv[0, :, :p, :].permute(1, 0, 2))
        block_ids = torch.tensor(blocks[:nblk], dtype=torch.int64, device=self.dev)
        kv_write_prefill(k_srcs, v_srcs, self.k_cache, self.v_cache, block_ids, p)
        first = int(out.logits[0, -1].argmax())
        row = np.zeros(self.max_blocks_per_seq, dtype=np.int64)
        row[: len(blocks)] = blocks
        seq = Sequence_(self._next_id, p, max_new_tokens, blocks, p, first, [first], row)
        self._next_id += 1
        return seq

    @torch.inference_mode()
    @torch.cuda.nvtx.range("pagedkv.prefill_many")
    def prefill_many(self, prompts: Sequence[Sequence[int]], max_new_tokens: int) -> List[Sequence_]:
        """Prefill several prompts in one forward: right-padded to one bucketed
        length (causal attention keeps padding out of every real token), the
        batch padded to a power of two with empty rows, then one prefill-write
        launch per prompt and the first token of each from one device-to-host
        copy. Same sequences as :meth:`prefill` on each prompt (up to the
        rounding of a differently shaped forward)."""
        b = len(prompts)
        assert b >= 1
        lens = [len(x) for x in prompts]
        need = [(p + max_new_tokens + self.block_size - 1) // self.block_size for p in lens]
        assert sum(need) <= len(self.free), "KV pool exhausted"
        padded = (max(lens) + self.prefill_bucket - 1) // self.prefill_bucket * self.prefill_bucket
        rows = 1
        while rows < b:
            rows *= 2
        ids = torch.zeros((rows, padded), dtype=torch.long)
        for i, x in enumerate(prompts):
            ids[i, : lens[i]] = torch.tensor(list(x), dtype=torch.long)
        keep = torch.tensor(lens + [1] * (rows - b), dtype=torch.long) - 1
        out = self.model(input_ids=ids.to(self.dev, non_blocking=True), use_cache=True,
                         logits_to_keep=keep.to(self.dev, non_blocking=True))
        # row i's logits at its own last prompt position: the diagonal of [rows, rows, vocab]
        diag = torch.arange(b, device=self.dev)
        first_t = out.logits[diag, diag].argmax(-1)
        pkv = out.past_key_values
        seqs: List[Sequence_] = []
        for i in range(b):
            p = lens[i]
            blocks = self._allocate(need[i])
            nblk = (p + self.block_size - 1) // self.block_size
            k_srcs, v_srcs = [], []
            for layer in range(self.num_layers):
                lk = pkv.layers[layer].keys if hasattr(pkv, "layers") else pkv[layer][0]
                lv = pkv.layers[layer].values if hasattr(pkv, "layers") else pkv[layer][1]
                k_srcs.append(lk[i, :, :p, :].permute(1, 0, 2))
                v_srcs.append(lv[i, :, :p, :].permute(1, 0, 2))
            block_ids = torch.tensor(blocks[:nblk], dtype=torch.int64, device=self.dev)
            kv_write_prefill(k_srcs, v_srcs, self.k_cache, self.v_cache, block_ids, p)
            row = np.zeros(self.max_blocks_per_seq, dtype=np.int64)
            row[: len(blocks)] = blocks
            seqs.append(Sequence_(self._next_id, p, max_new_tokens, blocks, p, -1, [], row))
            self._next_id += 1
        for seq, tok in zip(seqs, first_t.tolist()):
            seq.last_token = tok
            seq.generated = [tok]
        return seqs

    # ---- decode ----------------------------------------------------------------
    def _logits(self, ids: torch.Tensor, pos: torch.Tensor, tables: torch.Tensor, lens: torch.Tensor,
                slots: torch.Tensor) -> torch.Tensor:
        """One decode token per row through every layer; returns [B, vocab] logits."""
        m = self.model.model
        b = ids.shape[0]
        x = m.embed_tokens(ids[:, None])                      # [B, 1, hidden]
        cos, sin = m.rotary_emb(x, pos[:, None])               # [B, 1, D]
        cos2, sin2 = cos[:, 0], sin[:, 0]
        for li, layer in enumerate(m.layers):
            attn = layer.self_attn
            h = layer.input_layernorm(x)
            q = attn.q_proj(h).view(b, self.hq, self.head_dim)
            k = attn.k_proj(h).view(b, self.hkv, self.head_dim)
            v = attn.v_proj(h).view(b, self.hkv, self.head_dim)
            # RoPE of q and k, the append of k and v and the attention: one launch
            o = paged_attention_decode_append(q, self.k_cache[li], self.v_cache[li], tables, lens, attn.scaling,
                                              k, v, cos2, sin2, slot_mapping=slots)
            x = x + attn.o_proj(o.reshape(b, 1, -1))
            x = x + layer.mlp(layer.post_attention_layernorm(x))
        x = m.norm(x)
        return self.model.lm_head(x[:, 0])

    def _forward(self, ids, pos, tables, lens, slots) -> torch.Tensor:
        return self._logits(ids, pos, tables, lens, slots).argmax(-1)

    def _static(self, bsz: int) -> tuple:
        # int64 [bsz, 3]: token id, position, slot; int32 [bsz, 1 + width]: length, block table
        m64 = torch.zeros(bsz, 3, dtype=torch.int64, device=self.dev)
        m32 = torch.zeros(bsz, 1 + self.max_blocks_per_seq, dtype=torch.int32, device=self.dev)
        m64[:, 2] = -1
        return m64, m32

    def _views(self, m64: torch.Tensor, m32: torch.Tensor) -> tuple:
        return m64[:, 0], m64[:, 1], m32[:, 1:], m32[:, 0], m64[:, 2]

    def _graph_for(self, bsz: int) -> tuple:
        if bsz not in self._graphs:
            m64, m32 = self._static(bsz)
            with torch.inference_mode():
                for _ in range(2):  # warm the kernels and the workspace outside capture
                    self._forward(*self._views(m64, m32))
                torch.cuda.synchronize(self.dev)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    out = self._forward(*self._views(m64, m32))
            self._graphs[bsz] = (g, m64, m32, out)
        return self._graphs[bsz]

    def _host_for(self, bsz: int) -> tuple:
        if bsz not in self._host:
            h64 = torch.zeros(bsz, 3, dtype=torch.int64).pin_memory()
            h32 = torch.zeros(bsz, 1 + self.max_blocks_per_seq, dtype=torch.int32).pin_memory()
            self._host[bsz] = (h64, h32, h64.numpy(), h32.numpy())
        return self._host[bsz]

    @torch.inference_mode()
    @torch.cuda.nvtx.range("pagedkv.decode_step")
    def decode_step(self, seqs: List[Sequence_], return_logits: bool = False) -> Optional[torch.Tensor]:
        """Append each sequence's last token and sample the next one. With
        ``return_logits`` the step runs eagerly on the padded batch and also
        returns the [n, vocab] logits."""
        n = len(seqs)
        if n == 0:
            return None
        bsz = _bucket(n, self.max_batch) if self.use_graphs else n
        assert n <= bsz
        h64, h32, a64, a32 = self._host_for(bsz)
        bs = self.block_size
        pos = np.fromiter((s.num_tokens for s in seqs), dtype=np.int64, count=n)
        rows = np.stack([s.block_row for s in seqs])
        a64[:n, 0] = np.fromiter((s.last_token for s in seqs), dtype=np.int64, count=n)
        a64[:n, 1] = pos
        a64[:n, 2] = rows[np.arange(n), pos // bs] * bs + pos % bs
        a64[n:] = 0
        a64[n:, 2] = -1  # padding rows: no write, length 0
        a32[:n, 0] = pos + 1
        a32[:n, 1:] = rows
        a32[n:] = 0
        logits = None
        if return_logits:
            m64, m32 = self._static(bsz)
            m64.copy_(h64, non_blocking=True)
            m32.copy_(h32, non_blocking=True)
            logits = self._logits(*self._views(m64, m32))
            out = logits.argmax(-1)
            logits = logits[:n]
        elif self.use_graphs:
            g, m64, m32, out = self._graph_for(bsz)
            m64.copy_(h64, non_blocking=True)
            m32.copy_(h32, non_blocking=True)
            if self.timing is not None:
                ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                ev[0].record()
                g.replay()
                ev[1].record()
                self.timing.append(ev)
            else:
                g.replay()
        else:
            m64, m32 = self._static(bsz)
            m64.copy_(h64, non_blocking=True)
            m32.copy_(h32, non_blocking=True)
            out = self._forward(*self._views(m64, m32))
        nxt = out[:n].tolist()  # synchronises: the host buffers are free again
        for s, t in zip(seqs, nxt):
            s.num_tokens += 1
            s.last_token = int(t)
            s.generated.append(int(t))
        return logits

    def warm_prefill(self, max_prompt: int, batches: Sequence[int] = ()) -> None:
        """Run one prefill per bucket length up to ``max_prompt``, and one
        :meth:`prefill_many` per length and batch size in ``batches`` (kernel
        selection for each shape happens here, not inside a timed trace)."""
        for L in range(self.prefill_bucket, max_prompt + self.prefill_bucket, self.prefill_bucket):
            seq = self.prefill([1] * min(L, max_prompt), 1)
            self.release(seq)
            for nb in batches:
                for s_ in self.prefill_many([[1] * min(L, max_prompt)] * nb, 1):
                    self.release(s_)


def random_qwen2(num_layers: int = 24, hidden: int = 896, intermediate: int = 4864, heads: int = 14,
                 kv_heads: int = 2, vocab: int = 151936, dtype: torch.dtype = torch.float16,
                 device: str | torch.device = "cuda", seed: int = 0) -> torch.nn.Module:
    """A random-init Qwen2.5-0.5B-architecture model (tied embeddings)."""
    from transformers import Qwen2Config, Qwen2ForCausalLM

    torch.manual_seed(seed)
    cfg = Qwen2Config(hidden_size=hidden, intermediate_size=intermediate, num_hidden_layers=num_layers,
                      num_attention_heads=heads, num_key_value_heads=kv_heads, vocab_size=vocab,
                      tie_word_embeddings=True, max_position_embeddings=32768, rope_theta=1000000.0,
                      rms_norm_eps=1e-6)
    with torch.device(device):
        model = Qwen2ForCausalLM(cfg).to(dtype)
    return model.eval()
