"""GPU: seeded random batches through the one-launch decode step (KV append,
optionally RoPE, then the tensor-core attention).

Each draw mixes what the stream-K work split and each CTA's first ring fill
(issued straight from the range prologue) have to get right: lengths 0 and 1,
lengths on and next to tile boundaries, short and long sequences in one batch
(so CTA ranges start in the middle of segments and first pieces are shorter
than the ring), block sizes 8 to 128, head_dim 32 to 256, GQA groups 1 to 8,
fp16 and bf16. Every batch must equal the separate append (or RoPE + append)
and attention launches bit for bit, pools and output, and the fp32 oracle
(the reference's naive_reference_paged_attention restated,
engine/kernels/paged_attention.py:30-83) within the attention tests'
tolerance (2e-3 for fp16, 8e-3 for bf16 outputs).
"""
from __future__ import annotations

import random

import pytest
import torch

import pagedkv
from oracle import paged_ref

from test_gpu_fused_append import ATOL, RTOL, _case, _run

pytestmark = pytest.mark.gpu

# Bound on sum(lens) * kv_heads * head_dim, so that the fp32 CPU oracle of a
# draw takes about a second.
_ORACLE_ELEMS = 24_000_000
# bf16 output rounding alone is 2^-9 relative (the bf16 attention test's bound).
_TOL = {torch.float16: (ATOL, RTOL), torch.bfloat16: (8e-3, 8e-3)}


def _draw(seed: int):
    r = random.Random(seed)
    d = r.choice([32, 64, 64, 128, 128, 256])
    hkv = r.choice([1, 2, 2, 4, 8])
    g = r.choice([1, 2, 4, 7, 8])
    bs = r.choice([8, 16, 16, 32, 64, 128])
    n = r.choice([1, 3, 17, 64, 150, 300])
    edges = [0, 1, 2, 127, 128, 129, 255, 256, 257, 1000, 2048, 3000]
    lens = [r.choice(edges) if r.random() < 0.5 else r.randint(0, 3000) for _ in range(n)]
    while len(lens) > 1 and sum(lens) * hkv * d > _ORACLE_ELEMS:
        lens.pop()
    dtype = r.choice([torch.float16, torch.bfloat16])
    rope = r.random() < 0.5
    return d, hkv, g, bs, lens, dtype, rope


@pytest.mark.parametrize("seed", range(24))
def test_random_batches_fused_equal_separate_launches_and_oracle(cuda_ready, seed):
    d, hkv, g, bs, lens, dtype, rope = _draw(seed)
    c = _case(1000 + seed, hkv * g, hkv, d, bs, lens, dtype=dtype)
    out_f, kf, vf, out_u, ku, vu, q_rot, scale = _run(c, cuda_ready, rope)
    torch.cuda.synchronize()
    assert torch.equal(kf, ku) and torch.equal(vf, vu)
    assert torch.equal(out_f, out_u)
    ref = paged_ref.paged_attention_ref(q_rot.float().cpu(), ku.float().cpu(), vu.float().cpu(), c["rows"],
                                        c["lens"], scale)
    atol, rtol = _TOL[dtype]
    torch.testing.assert_close(out_f.float().cpu(), ref, atol=atol, rtol=rtol)
    assert pagedkv.read_error_flags(cuda_ready) == 0
