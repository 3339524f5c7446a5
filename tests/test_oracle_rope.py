"""CPU: the rotary restatement in oracle/ is bit-identical to transformers'
apply_rotary_pos_emb (the function the reference decode forward calls,
paged_attention_integration.py:108-109) for fp16 and bf16."""
import pytest
import torch

from oracle import paged_ref


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("hq,hkv,d", [(14, 2, 64), (8, 8, 128), (4, 1, 32)])
def test_rope_oracle_matches_transformers(dtype, hq, hkv, d):
    from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb

    g = torch.Generator().manual_seed(hq * 1000 + d)
    n = 9
    q = (torch.randn(n, hq, d, generator=g) * 3).to(dtype)
    k = (torch.randn(n, hkv, d, generator=g) * 3).to(dtype)
    pos = torch.randint(0, 8192, (n,), generator=g).float()
    inv = 1.0 / (1e6 ** (torch.arange(0, d, 2).float() / d))
    freqs = pos[:, None] * inv[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    cos, sin = emb.cos().to(dtype), emb.sin().to(dtype)
    # transformers' layout: q/k [B, H, 1, D], cos/sin [B, 1, D]
    rq, rk = apply_rotary_pos_emb(q[:, :, None, :], k[:, :, None, :], cos[:, None, :], sin[:, None, :])
    assert torch.equal(paged_ref.rope_ref(q, cos, sin).view(torch.int16), rq[:, :, 0, :].view(torch.int16))
    assert torch.equal(paged_ref.rope_ref(k, cos, sin).view(torch.int16), rk[:, :, 0, :].view(torch.int16))
