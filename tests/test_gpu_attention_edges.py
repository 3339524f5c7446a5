"""GPU: edge shapes of the tensor-core decode kernel's stream-K machinery,
against the fp32 oracle (tolerance as the other attention tests)."""
import math

import numpy as np
import pytest
import torch

import pagedkv
from oracle import paged_ref

from test_gpu_attention import ATOL, RTOL, _check_vs_oracle, _random_case

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("ctx", [64 * 1024, 300 * 128 + 17])
def test_one_sequence_spanning_every_cta(cuda_ready, ctx):
    """One (sequence, head group) segment cut into ~148 pieces: middle pieces in
    every CTA and a combine over all of them."""
    q, k, v, tables, lists, lens = _random_case(ctx, 1, 14, 2, 64, 16, [ctx])
    _check_vs_oracle(cuda_ready, q, k, v, tables, lists, lens, 0.125)
    assert pagedkv.last_decode_launch_info()[1] == "tc"
    assert pagedkv.read_error_flags(cuda_ready) == 0


def test_two_long_sequences_and_short_ones(cuda_ready):
    lens = [40000, 3, 129, 25000, 128, 256, 1]
    q, k, v, tables, lists, lens_t = _random_case(9, len(lens), 16, 8, 128, 16, lens, q_scale=10.0)
    _check_vs_oracle(cuda_ready, q, k, v, tables, lists, lens_t, 1 / math.sqrt(128))


@pytest.mark.parametrize("hkv", [1, 3, 5])
@pytest.mark.parametrize("g", [1, 7, 16])
def test_odd_kv_heads_at_head_dim_64(cuda_ready, hkv, g):
    """head_dim 64 pairs two kv heads per segment; an odd count leaves the last
    pair half empty."""
    lens = [1, 127, 128, 129, 700]
    q, k, v, tables, lists, lens_t = _random_case(hkv * 100 + g, len(lens), hkv * g, hkv, 64, 16, lens)
    _check_vs_oracle(cuda_ready, q, k, v, tables, lists, lens_t, 0.125)


@pytest.mark.parametrize("bs", [8, 128])
def test_tensor_core_block_size_limits(cuda_ready, bs):
    lens = [1, bs - 1, bs, bs + 1, 128, 129, 5 * bs + 3, 3000]
    q, k, v, tables, lists, lens_t = _random_case(bs + 1, len(lens), 14, 2, 64, bs, lens)
    _check_vs_oracle(cuda_ready, q, k, v, tables, lists, lens_t, 0.125)
    assert pagedkv.last_decode_launch_info()[1] == "tc"


def test_fewer_tiles_than_sms(cuda_ready):
    for lens in ([1], [200], [5, 7], [129, 1, 3]):
        q, k, v, tables, lists, lens_t = _random_case(len(lens) + lens[0], len(lens), 8, 2, 128, 16, lens)
        _check_vs_oracle(cuda_ready, q, k, v, tables, lists, lens_t, 1 / math.sqrt(128))


def test_many_short_sequences(cuda_ready):
    """4096 sequences: the prologue scan walks several sequences per thread."""
    rng = np.random.default_rng(4)
    lens = rng.integers(0, 300, 4096).tolist()
    q, k, v, tables, lists, lens_t = _random_case(41, len(lens), 14, 2, 64, 16, lens)
    out = _check_vs_oracle(cuda_ready, q, k, v, tables, lists, lens_t, 0.125)
    zero = [i for i, n in enumerate(lens) if n == 0]
    assert torch.count_nonzero(out[zero]) == 0


def test_back_to_back_launches_of_changing_shapes(cuda_ready):
    """The cross-CTA flags must be back at zero after every launch: alternate
    shapes whose segments are cut at different places, 60 launches, and check
    every result."""
    cases = []
    for i, lens in enumerate(([2048] * 40, [5000, 17, 3000], [700] * 90, [20000], [129] * 300)):
        cases.append(_random_case(500 + i, len(lens), 14, 2, 64, 16, lens))
    dev = cuda_ready
    dcases = [tuple(t.to(dev) if torch.is_tensor(t) else t for t in c) for c in cases]
    refs = [paged_ref.paged_attention_ref(c[0].float(), c[1].float(), c[2].float(), c[4], c[5].tolist(), 0.125)
            for c in cases]
    for it in range(60):
        i = it % len(cases)
        q, k, v, tables, _, lens = dcases[i]
        out = pagedkv.paged_attention_decode_batched(q, k, v, tables, lens, 0.125)
        torch.testing.assert_close(out.float().cpu(), refs[i], atol=ATOL, rtol=RTOL)
    assert pagedkv.read_error_flags(dev) == 0


@pytest.mark.parametrize("d,g", [(128, 17), (128, 24), (128, 32), (32, 1), (32, 5), (32, 8), (64, 16)])
def test_wide_groups_and_head_dim_32_on_tensor_cores(cuda_ready, d, g):
    """GQA groups up to 32 at head_dim 128 (one kv head per tile, 32 query
    columns) and head_dim 32 (four kv heads per tile, block-diagonal Q)."""
    hkv = 3 if d == 32 else 2  # head_dim 32: a group of four kv heads, the last one partly empty
    lens = [1, 100, 128, 129, 1500]
    q, k, v, tables, lists, lens_t = _random_case(d * 100 + g, len(lens), g * hkv, hkv, d, 16, lens, q_scale=4.0)
    _check_vs_oracle(cuda_ready, q, k, v, tables, lists, lens_t, 1 / math.sqrt(d))
    assert pagedkv.last_decode_launch_info()[1] == "tc"


@pytest.mark.parametrize(
    "d,g,hkv,dtype",
    [
        (128, 40, 2, torch.float16),   # 32 + 8 query heads per kv head
        (128, 64, 1, torch.float16),   # two full chunks of 32
        (64, 71, 1, torch.float16),    # MQA with 71 query heads: chunks 16,16,16,16,7
        (64, 20, 3, torch.bfloat16),   # odd kv heads (a half-empty tile row) and 16 + 4
        (32, 12, 5, torch.float16),    # four kv heads per tile row, 8 + 4
        (32, 9, 4, torch.float16),
    ],
)
def test_groups_wider_than_a_tile_run_in_chunks(cuda_ready, d, g, hkv, dtype):
    """GQA groups above 32 / 16 / 8 query heads per kv head (head_dim 128 / 64
    / 32) run on the tensor cores in chunks of that many heads, one segment per
    chunk; long and short sequences, so chunk segments are also cut across CTAs
    and combined."""
    lens = [1, 100, 129, 3000, 20000]
    q, k, v, tables, lists, lens_t = _random_case(d * 1000 + g, len(lens), g * hkv, hkv, d, 16, lens,
                                                  q_scale=4.0, dtype=dtype)
    tol = dict(atol=8e-3, rtol=8e-3) if dtype == torch.bfloat16 else {}
    _check_vs_oracle(cuda_ready, q, k, v, tables, lists, lens_t, 1 / math.sqrt(d), **tol)
    assert pagedkv.last_decode_launch_info()[1] == "tc"
    assert pagedkv.read_error_flags(cuda_ready) == 0


@pytest.mark.parametrize(
    "g,hkv,bs,dtype",
    [
        (1, 2, 16, torch.float16),
        (2, 8, 16, torch.float16),    # Gemma-2-9B-like: 16 query / 8 kv heads
        (7, 1, 8, torch.float16),
        (16, 2, 16, torch.bfloat16),
        (20, 1, 128, torch.float16),  # chunks of 16 + 4 query heads
        (32, 2, 16, torch.float16),   # two full chunks
    ],
)
def test_head_dim_256_on_tensor_cores(cuda_ready, g, hkv, bs, dtype):
    """head_dim 256: each head is two 128-element sub-rows (two K and two V ring
    stages per tile, S summed over both, one O accumulator each); partial last
    blocks, short and long sequences cut across CTAs."""
    lens = [1, 37, 128, 129, 2000, 9000]
    q, k, v, tables, lists, lens_t = _random_case(256 * 100 + g, len(lens), g * hkv, hkv, 256, bs, lens,
                                                  q_scale=4.0, dtype=dtype)
    tol = dict(atol=8e-3, rtol=8e-3) if dtype == torch.bfloat16 else {}
    _check_vs_oracle(cuda_ready, q, k, v, tables, lists, lens_t, 1 / 16.0, **tol)
    assert pagedkv.last_decode_launch_info()[1] == "tc"
    assert pagedkv.read_error_flags(cuda_ready) == 0
