"""GPU: the model-level decode runner (config 5's caller of the paged path)
against the Hugging Face model itself: prefill K/V land bit-exact in the pool,
and each decode step's logits match HF's own cached decode of the same tokens."""
import pytest
import torch

from pagedkv.decode_runner import PagedDecodeRunner, random_qwen2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small_model(cuda_ready):
    # head_dim 64, GQA 2: the tensor-core decode kernel
    return random_qwen2(num_layers=3, hidden=256, intermediate=512, heads=4, kv_heads=2, vocab=512,
                        dtype=torch.float16, device=cuda_ready, seed=3)


def _hf_decode_logits(model, prompt, tokens, dev):
    """HF's own forward with its DynamicCache: logits for each fed token."""
    with torch.inference_mode():
        out = model(input_ids=torch.tensor([prompt], device=dev), use_cache=True)
        cache = out.past_key_values
        logits = []
        for t in tokens:
            out = model(input_ids=torch.tensor([[t]], device=dev), past_key_values=cache, use_cache=True)
            cache = out.past_key_values
            logits.append(out.logits[0, -1].float())
    return logits


def test_prefill_rows_match_hf_cache(cuda_ready, small_model):
    # prefill_bucket=1: the prompt runs unpadded, so its rows are HF's bit for bit
    runner = PagedDecodeRunner(small_model, num_blocks=64, block_size=16, max_batch=4, max_seq_len=256,
                               prefill_bucket=1)
    prompt = list(range(7, 7 + 37))
    seq = runner.prefill(prompt, max_new_tokens=8)
    with torch.inference_mode():
        cache = small_model(input_ids=torch.tensor([prompt], device=cuda_ready), use_cache=True).past_key_values
    for layer in range(small_model.config.num_hidden_layers):
        hf_k = cache.layers[layer].keys[0].permute(1, 0, 2)  # [tokens, kv_heads, D]
        hf_v = cache.layers[layer].values[0].permute(1, 0, 2)
        for t in range(len(prompt)):
            b, o = seq.blocks[t // 16], t % 16
            assert torch.equal(runner.k_cache[layer][b, o], hf_k[t])
            assert torch.equal(runner.v_cache[layer][b, o], hf_v[t])


def test_decode_logits_match_hf(cuda_ready, small_model):
    runner = PagedDecodeRunner(small_model, num_blocks=128, block_size=16, max_batch=4, max_seq_len=256)
    prompts = [list(range(3, 3 + n)) for n in (5, 40, 77)]
    seqs = [runner.prefill(p, max_new_tokens=6) for p in prompts]
    fed = [[s.last_token] for s in seqs]
    ours = [[] for _ in seqs]
    for _ in range(5):
        logits = runner.decode_step(seqs, return_logits=True)
        for i, s in enumerate(seqs):
            ours[i].append(logits[i].float())
            fed[i].append(s.last_token)
    for i, p in enumerate(prompts):
        ref = _hf_decode_logits(small_model, p, fed[i][:5], cuda_ready)
        for a, b in zip(ours[i], ref):
            scale = b.abs().max().item()
            assert (a - b).abs().max().item() <= 2e-2 * max(scale, 1.0), (i, (a - b).abs().max().item(), scale)


def test_graph_steps_match_eager_steps(cuda_ready, small_model):
    """Captured (padded to the bucket) and eager steps give the same tokens."""
    def run(use_graphs):
        r = PagedDecodeRunner(small_model, num_blocks=128, block_size=16, max_batch=4, max_seq_len=256,
                              use_graphs=use_graphs)
        seqs = [r.prefill(list(range(11, 11 + n)), max_new_tokens=8) for n in (9, 33, 50, 64)]
        for _ in range(7):
            r.decode_step(seqs)
        return [s.generated for s in seqs]

    assert run(True) == run(False)


def test_padded_prefill_keeps_rows_and_first_token(cuda_ready, small_model):
    """Right-padding the prompt to the bucket changes neither the first token
    nor (beyond GEMM rounding) the prompt's K/V rows."""
    prompt = list(range(5, 5 + 45))
    a = PagedDecodeRunner(small_model, num_blocks=16, block_size=16, max_batch=1, max_seq_len=128, prefill_bucket=1)
    b = PagedDecodeRunner(small_model, num_blocks=16, block_size=16, max_batch=1, max_seq_len=128, prefill_bucket=64)
    sa, sb = a.prefill(prompt, 4), b.prefill(prompt, 4)
    assert sa.last_token == sb.last_token
    for layer in range(small_model.config.num_hidden_layers):
        for t in range(len(prompt)):
            ra = a.k_cache[layer][sa.blocks[t // 16], t % 16].float()
            rb = b.k_cache[layer][sb.blocks[t // 16], t % 16].float()
            assert (ra - rb).abs().max().item() <= 1e-2 * max(1.0, ra.abs().max().item())


def test_batched_prefill_matches_one_prompt_at_a_time(cuda_ready, small_model):
    """prefill_many on prompts of different lengths (batch padded to 4 rows):
    the same first tokens and, within GEMM rounding, the same K/V rows as
    prefill() of each prompt alone; then decoding continues from both."""
    prompts = [list(range(7, 7 + 45)), list(range(100, 100 + 130)), list(range(300, 300 + 3))]
    a = PagedDecodeRunner(small_model, num_blocks=64, block_size=16, max_batch=4, max_seq_len=256)
    b = PagedDecodeRunner(small_model, num_blocks=64, block_size=16, max_batch=4, max_seq_len=256)
    one = [a.prefill(p, 4) for p in prompts]
    many = b.prefill_many(prompts, 4)
    assert [s.last_token for s in one] == [s.last_token for s in many]
    assert [s.generated for s in many] == [[s.last_token] for s in many]
    for sa, sb, p in zip(one, many, prompts):
        assert sb.prompt_len == len(p) and sb.num_tokens == len(p)
        for layer in range(small_model.config.num_hidden_layers):
            for t in range(len(p)):
                for pool_a, pool_b in ((a.k_cache, b.k_cache), (a.v_cache, b.v_cache)):
                    ra = pool_a[layer][sa.blocks[t // 16], t % 16].float()
                    rb = pool_b[layer][sb.blocks[t // 16], t % 16].float()
                    assert (ra - rb).abs().max().item() <= 1e-2 * max(1.0, ra.abs().max().item())
    a.decode_step(one)
    b.decode_step(many)
    assert [s.last_token for s in one] == [s.last_token for s in many]
