"""GPU: the drop-in decode forward against the reference's own layer output.

The golden append cases were produced by running the reference's
paged_decode_attention_forward (fp16, CPU). Here the same module weights and
inputs go through pagedkv.integration.paged_decode_attention_forward on the
B200: the attention-layer output must match the reference's, and the pool
must hold exactly the rows this forward computed, at the reference's slots,
with every other row untouched.
"""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

import cases
import pagedkv
from oracle import paged_ref
from pagedkv import integration

pytestmark = pytest.mark.gpu


def _module(inp, case, dev):
    hq, hkv, d = case["hq"], case["hkv"], case["d"]
    hidden = inp["hidden"]
    m = torch.nn.Module()
    m.layer_idx = 0
    m.head_dim = d
    m.scaling = d ** -0.5
    m.q_proj = torch.nn.Linear(hidden, hq * d, bias=True, dtype=torch.float16)
    m.k_proj = torch.nn.Linear(hidden, hkv * d, bias=True, dtype=torch.float16)
    m.v_proj = torch.nn.Linear(hidden, hkv * d, bias=True, dtype=torch.float16)
    m.o_proj = torch.nn.Linear(hq * d, hidden, bias=False, dtype=torch.float16)
    with torch.no_grad():
        for lin, w, b in ((m.q_proj, "w_q", "b_q"), (m.k_proj, "w_k", "b_k"), (m.v_proj, "w_v", "b_v")):
            lin.weight.copy_(torch.from_numpy(inp[w]))
            lin.bias.copy_(torch.from_numpy(inp[b]))
        m.o_proj.weight.copy_(torch.from_numpy(inp["w_o"]))
    return m.to(dev)


@pytest.mark.parametrize("name", list(cases.APPEND_CASES))
def test_decode_forward_matches_reference_layer(cuda_ready, golden, name):
    from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb

    arrays, _ = golden
    dev = cuda_ready
    case = cases.APPEND_CASES[name]
    inp = cases.make_append_inputs(case)
    bs, d = case["bs"], case["d"]
    pool = SimpleNamespace(
        k_cache=[torch.from_numpy(inp["k_cache"]).to(dev)],
        v_cache=[torch.from_numpy(inp["v_cache"]).to(dev)],
        device=dev,
    )
    tables = [SimpleNamespace(physical_block_ids=list(t)) for t in inp["tables"]]
    ctx = integration.PagedAttentionContext(pool=pool, block_tables=tables, seq_lens=list(inp["lens"]), block_size=bs)
    mod = _module(inp, case, dev)
    mod._paged_attention_context = ctx
    cos, sin = cases.rope_cos_sin(np.asarray(inp["lens"]) - 1, d)
    cos_t = torch.from_numpy(cos).to(dev, torch.float16)
    sin_t = torch.from_numpy(sin).to(dev, torch.float16)
    h = torch.from_numpy(inp["h"]).to(dev)
    with torch.inference_mode():
        out, _ = integration.paged_decode_attention_forward(mod, h, (cos_t, sin_t))
        bsz = h.shape[0]
        k = mod.k_proj(h).view(bsz, 1, -1, d).transpose(1, 2)
        q = mod.q_proj(h).view(bsz, 1, -1, d).transpose(1, 2)
        v = mod.v_proj(h).view(bsz, 1, -1, d).transpose(1, 2)
        q, k = apply_rotary_pos_emb(q, k, cos_t, sin_t)
    torch.cuda.synchronize()
    # layer output vs the reference's (fp16 GEMMs on CPU there, on the GPU here)
    torch.testing.assert_close(out.float().cpu(), torch.from_numpy(arrays[f"{name}__attn_out"]), atol=1e-2, rtol=1e-2)
    # the append: rows this forward computed, at the reference's slots, nothing else touched
    slots = paged_ref.decode_slots(inp["tables"], inp["lens"], bs)
    kr = inp["k_cache"].copy()
    vr = inp["v_cache"].copy()
    paged_ref.kv_append_ref(kr, vr, k.squeeze(2).cpu().numpy(), v.squeeze(2).cpu().numpy(), slots)
    assert np.array_equal(pool.k_cache[0].cpu().numpy().view(np.int16), kr.view(np.int16))
    assert np.array_equal(pool.v_cache[0].cpu().numpy().view(np.int16), vr.view(np.int16))
    assert pagedkv.read_error_flags(dev) == 0


def test_copy_on_write_then_append_keeps_the_shared_block(cuda_ready):
    """A shared, partially filled block is copied for the writer before its
    append, so the other sequences still see the original rows."""
    dev = cuda_ready
    layers, nb, bs, hkv, d = 3, 16, 16, 2, 64
    g = torch.Generator().manual_seed(0)
    pool = SimpleNamespace(
        k_cache=[torch.randn(nb, bs, hkv, d, generator=g).half().to(dev) for _ in range(layers)],
        v_cache=[torch.randn(nb, bs, hkv, d, generator=g).half().to(dev) for _ in range(layers)],
        device=dev,
    )
    k0 = [t.clone() for t in pool.k_cache]

    class Alloc:
        def __init__(self):
            self.free_ids = [15, 14, 13]
            self.ref_counts = {2: 2, 7: 1}

        def allocate(self):
            b = self.free_ids.pop(0)
            self.ref_counts[b] = 1
            return b

        def release(self, b):
            self.ref_counts[b] -= 1

    writer = SimpleNamespace(physical_block_ids=[7, 2], num_tokens=16 + 5)
    pairs = integration.prepare_copy_on_write([writer], Alloc(), bs)
    assert pairs == [(2, 15)] and writer.physical_block_ids == [7, 15]
    integration.copy_on_write(pool, pairs)
    new = torch.ones(1, hkv, d, dtype=torch.float16, device=dev)
    slots = torch.tensor([15 * bs + 5], dtype=torch.int64, device=dev)
    for layer in range(layers):
        pagedkv.kv_append(new, new, pool.k_cache[layer], pool.v_cache[layer], slots)
    torch.cuda.synchronize()
    for layer in range(layers):
        assert torch.equal(pool.k_cache[layer][2], k0[layer][2])  # shared block untouched
        assert torch.equal(pool.k_cache[layer][15][:5], k0[layer][2][:5])  # copied prefix
        assert torch.equal(pool.k_cache[layer][15][5], new[0])  # appended row


def test_runner_decode_step_batched_syncs_match_per_sequence_results(cuda_ready):
    """integration.decode_step (installed over the reference runner's
    decode_step) on a 2-layer random-init Qwen2 model: next tokens, pool
    writes, host logits and logit margins equal those of the same forward
    followed by the reference's per-sequence diagnostics."""
    from pagedkv.decode_runner import random_qwen2

    dev = cuda_ready
    model = random_qwen2(num_layers=2, device=dev, seed=3)
    cfg = model.config
    hkv, d, bs, nb = cfg.num_key_value_heads, cfg.hidden_size // cfg.num_attention_heads, 16, 64
    g = torch.Generator(device=dev).manual_seed(4)
    kc = [torch.randn(nb, bs, hkv, d, generator=g, device=dev).half() for _ in range(2)]
    vc = [torch.randn(nb, bs, hkv, d, generator=g, device=dev).half() for _ in range(2)]

    def state():
        pool = SimpleNamespace(k_cache=[t.clone() for t in kc], v_cache=[t.clone() for t in vc], device=dev)
        seqs = [
            SimpleNamespace(seq_id=0, block_table=SimpleNamespace(physical_block_ids=[5, 9], num_tokens=20),
                            last_token_id=101, last_logits=None, last_logit_margin=None),
            SimpleNamespace(seq_id=1, block_table=SimpleNamespace(physical_block_ids=[2], num_tokens=7),
                            last_token_id=7, last_logits=None, last_logit_margin=None),
            SimpleNamespace(seq_id=2, block_table=SimpleNamespace(physical_block_ids=[30, 31, 40], num_tokens=33),
                            last_token_id=150000, last_logits=None, last_logit_margin=None),
        ]
        runner = SimpleNamespace(block_size=bs, device=dev, pool=pool, model=model,
                                 allocator=SimpleNamespace(ref_counts={}))
        return seqs, runner

    seqs, runner = state()
    got = integration.decode_step(runner, seqs, None)

    seqs_e, runner_e = state()
    with torch.inference_mode():
        lens = []
        for s in seqs_e:
            s.block_table.num_tokens += 1
            lens.append(s.block_table.num_tokens)
        ids = torch.tensor([[s.last_token_id] for s in seqs_e], device=dev)
        pos = torch.tensor([[n - 1] for n in lens], device=dev)
        ctx = integration.PagedAttentionContext(pool=runner_e.pool, block_tables=[s.block_table for s in seqs_e],
                                                seq_lens=lens, block_size=bs, is_decode=True)
        with integration.patch_paged_attention(model, ctx):
            logits = model(input_ids=ids, position_ids=pos, use_cache=False).logits[:, -1, :]
        want = torch.argmax(logits, dim=-1).tolist()
    assert got == want
    for i, (a, b) in enumerate(zip(seqs, seqs_e)):
        assert a.block_table.num_tokens == b.block_table.num_tokens
        assert torch.equal(a.last_logits, logits[i].cpu())
        top2 = torch.topk(logits[i], k=2).values
        assert a.last_logit_margin == float((top2[0] - top2[1]).item())
    for x, y in zip(runner.pool.k_cache + runner.pool.v_cache, runner_e.pool.k_cache + runner_e.pool.v_cache):
        assert torch.equal(x, y)
