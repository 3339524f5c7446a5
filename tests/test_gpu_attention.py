"""GPU parity of the paged decode attention kernels (through the C ABI).

Bar (north star): fp16 output within 2e-3 abs / 2e-3 rel of the reference's
fp32 result on identical inputs, checked against (a) the golden outputs of
the reference implementation itself and (b) the pinned CPU oracle.
"""
import math
import random

import numpy as np
import pytest
import torch

import cases
import pagedkv
from oracle import paged_ref
from pagedkv import _native

pytestmark = pytest.mark.gpu

ATOL = 2e-3
RTOL = 2e-3
GPU_CASES = [n for n, c in cases.ATTENTION_CASES.items() if c.get("gpu", True)]


def _device_inputs(inp, dev, dtype=torch.float16):
    q = torch.from_numpy(inp["q"]).to(dev, dtype)
    k = torch.from_numpy(inp["k_cache"]).to(dev, dtype)
    v = torch.from_numpy(inp["v_cache"]).to(dev, dtype)
    tables = torch.from_numpy(inp["tables"]).to(dev)
    lens = torch.from_numpy(inp["lens"]).to(dev)
    return q, k, v, tables, lens


@pytest.mark.parametrize("name", GPU_CASES)
def test_batched_matches_reference_golden(cuda_ready, golden, name):
    arrays, manifest = golden
    inp = cases.make_attention_inputs(cases.ATTENTION_CASES[name])
    assert cases.sha256_arrays(inp["q"], inp["k_cache"], inp["v_cache"], inp["tables"]) == (
        manifest["attention"][name]["input_sha256"]
    )
    q, k, v, tables, lens = _device_inputs(inp, cuda_ready)
    _native.lib()
    out = pagedkv.paged_attention_decode_batched(q, k, v, tables, lens, inp["scale"])
    launches, family = pagedkv.last_decode_launch_info()
    assert launches >= 1 and family in ("tc", "simt")
    assert out.dtype == torch.float16 and out.shape == q.shape
    expected = torch.from_numpy(arrays[f"{name}__out"])
    torch.testing.assert_close(out.float().cpu(), expected, atol=ATOL, rtol=RTOL)
    assert pagedkv.read_error_flags(cuda_ready) == 0


@pytest.mark.parametrize("name", ["gqa7_qwen", "mqa4_bs8", "long_2048", "large_magnitude_x10", "gqa2_d32"])
def test_v1_v2_single_sequence_match_golden(cuda_ready, golden, name):
    arrays, _ = golden
    inp = cases.make_attention_inputs(cases.ATTENTION_CASES[name])
    q, k, v, tables, lens = _device_inputs(inp, cuda_ready)
    expected = arrays[f"{name}__out"]
    for i, n in enumerate(inp["lens"]):
        bt = torch.tensor(inp["table_lists"][i], dtype=torch.int32, device=cuda_ready)
        o1 = pagedkv.paged_attention_decode_v1(q[i], k, v, bt, int(n), inp["scale"])
        o2 = pagedkv.paged_attention_decode_v2(q[i], k, v, bt, int(n), inp["scale"])
        torch.testing.assert_close(o1.float().cpu(), torch.from_numpy(expected[i]), atol=ATOL, rtol=RTOL)
        torch.testing.assert_close(o2.float().cpu(), torch.from_numpy(expected[i]), atol=ATOL, rtol=RTOL)
        torch.testing.assert_close(o1, o2, atol=0, rtol=0)


def _random_case(seed, n, hq, hkv, d, bs, lens, num_blocks=None, q_scale=1.0, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    need = [max(1, (x + bs - 1) // bs) for x in lens]
    nb = num_blocks or (sum(need) + 16)
    perm = list(range(nb))
    random.Random(seed).shuffle(perm)
    width = max(need)
    tables = torch.zeros((n, width), dtype=torch.int32)
    lists, at = [], 0
    for i, c in enumerate(need):
        row = perm[at : at + c]
        at += c
        tables[i, :c] = torch.tensor(row, dtype=torch.int32)
        lists.append(row)
    q = (torch.randn(n, hq, d, generator=g) * q_scale).to(dtype)
    k = torch.randn(nb, bs, hkv, d, generator=g).to(dtype)
    v = torch.randn(nb, bs, hkv, d, generator=g).to(dtype)
    return q, k, v, tables, lists, torch.tensor(lens, dtype=torch.int32)


def _check_vs_oracle(dev, q, k, v, tables, lists, lens, scale, atol=ATOL, rtol=RTOL):
    out = pagedkv.paged_attention_decode_batched(
        q.to(dev), k.to(dev), v.to(dev), tables.to(dev), lens.to(dev), scale
    )
    ref = paged_ref.paged_attention_ref(q.float(), k.float(), v.float(), lists, lens.tolist(), scale)
    torch.testing.assert_close(out.float().cpu(), ref, atol=atol, rtol=rtol)
    return out


def test_config2_shape_full_size_vs_oracle(cuda_ready):
    """BASELINE config 2 at full size: 256 x 2048 tokens, 14q/2kv, D=64, BS=16,
    pool 40960 blocks, shuffled tables."""
    n, hq, hkv, d, bs, ctx = 256, 14, 2, 64, 16, 2048
    q, k, v, tables, lists, lens = _random_case(2, n, hq, hkv, d, bs, [ctx] * n, num_blocks=40960)
    _check_vs_oracle(cuda_ready, q, k, v, tables, lists, lens, 1 / math.sqrt(d))
    assert pagedkv.read_error_flags(cuda_ready) == 0


@pytest.mark.parametrize("hq", [8, 16, 32, 56])
def test_config3_gqa_sweep_vs_oracle(cuda_ready, hq):
    """BASELINE config 3 (reduced batch): D=128, 8 kv heads, G in {1,2,4,7},
    log-uniform lengths in [16, 8192], q x30."""
    rng = np.random.default_rng(hq)
    lens = [int(round(math.exp(x))) for x in rng.uniform(math.log(16), math.log(8192), size=24)]
    q, k, v, tables, lists, lens_t = _random_case(hq, 24, hq, 8, 128, 16, lens, q_scale=30.0)
    _check_vs_oracle(cuda_ready, q, k, v, tables, lists, lens_t, 1 / math.sqrt(128))


@pytest.mark.parametrize("d", [32, 64, 128, 256])
@pytest.mark.parametrize("g", [1, 2, 3, 4, 7, 8, 12])
def test_head_dim_group_grid_vs_oracle(cuda_ready, d, g):
    hkv = 2
    lens = [1, 15, 16, 17, 130, 777]
    q, k, v, tables, lists, lens_t = _random_case(1000 * d + g, len(lens), g * hkv, hkv, d, 16, lens)
    _check_vs_oracle(cuda_ready, q, k, v, tables, lists, lens_t, 1 / math.sqrt(d))


@pytest.mark.parametrize("bs", [1, 8, 16, 32, 64])
def test_block_sizes_vs_oracle(cuda_ready, bs):
    lens = [1, bs, bs + 1, 3 * bs - 1, 1000]
    q, k, v, tables, lists, lens_t = _random_case(bs, len(lens), 14, 2, 64, bs, lens)
    _check_vs_oracle(cuda_ready, q, k, v, tables, lists, lens_t, 0.125)


@pytest.mark.parametrize("d", [32, 64, 128, 256])
@pytest.mark.parametrize("g,bs", [(1, 4), (2, 5), (4, 4), (7, 4), (12, 3)])
def test_cuda_core_kernel_shapes_vs_oracle(cuda_ready, d, g, bs):
    """Block sizes the tensor-core kernel does not take (below 8, not powers of
    two) run on the CUDA-core kernel: every (head_dim, group width) variant of
    it, contexts from one token to several splits, against the oracle."""
    hkv = 2
    lens = [1, bs, 3 * bs + 1, 130, 777, 2500]
    q, k, v, tables, lists, lens_t = _random_case(7000 + 10 * d + g, len(lens), g * hkv, hkv, d, bs, lens)
    _check_vs_oracle(cuda_ready, q, k, v, tables, lists, lens_t, 1 / math.sqrt(d))
    assert pagedkv.last_decode_launch_info()[1] == "simt"
    assert pagedkv.read_error_flags(cuda_ready) == 0


def test_bf16_pool_vs_oracle(cuda_ready):
    lens = [5, 64, 300, 2048]
    q, k, v, tables, lists, lens_t = _random_case(77, 4, 14, 2, 64, 16, lens, dtype=torch.bfloat16)
    # bf16 output rounding alone is 2^-9 relative.
    _check_vs_oracle(cuda_ready, q, k, v, tables, lists, lens_t, 0.125, atol=8e-3, rtol=8e-3)


def test_zero_length_sequences_give_zeros(cuda_ready):
    lens = [0, 33, 0, 1]
    q, k, v, tables, lists, lens_t = _random_case(9, 4, 14, 2, 64, 16, lens)
    out = _check_vs_oracle(cuda_ready, q, k, v, tables, lists, lens_t, 0.125)
    assert torch.count_nonzero(out[0]) == 0 and torch.count_nonzero(out[2]) == 0


def test_strided_query_view(cuda_ready):
    """q as a strided view (as produced by a fused qkv projection)."""
    lens = [40, 90]
    q, k, v, tables, lists, lens_t = _random_case(11, 2, 14, 2, 64, 16, lens)
    big = torch.randn(2, 20, 64, dtype=torch.float16)
    big[:, 3:17] = q
    qv = big.to(cuda_ready)[:, 3:17]
    assert not qv.is_contiguous()
    out = pagedkv.paged_attention_decode_batched(qv, k.to(cuda_ready), v.to(cuda_ready), tables.to(cuda_ready),
                                                 lens_t.to(cuda_ready), 0.125)
    ref = paged_ref.paged_attention_ref(q.float(), k.float(), v.float(), lists, lens, 0.125)
    torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)


def test_out_of_range_block_id_is_flagged_not_faulted(cuda_ready):
    lens = [20, 20]
    q, k, v, tables, lists, lens_t = _random_case(12, 2, 14, 2, 64, 16, lens)
    nb = k.shape[0]
    tables[1, 1] = nb + 5  # invalid entry the kernel must skip and report
    pagedkv.read_error_flags(cuda_ready, clear=True)
    out = pagedkv.paged_attention_decode_batched(q.to(cuda_ready), k.to(cuda_ready), v.to(cuda_ready),
                                                 tables.to(cuda_ready), lens_t.to(cuda_ready), 0.125)
    flags = pagedkv.read_error_flags(cuda_ready, clear=True)
    assert flags & _native.EFLAG_BLOCK_ID_RANGE
    ref0 = paged_ref.paged_attention_ref(q[:1].float(), k.float(), v.float(), lists[:1], lens[:1], 0.125)
    torch.testing.assert_close(out[:1].float().cpu(), ref0, atol=ATOL, rtol=RTOL)


def test_seq_len_beyond_table_is_flagged(cuda_ready):
    lens = [20, 50]
    q, k, v, tables, lists, lens_t = _random_case(13, 2, 14, 2, 64, 16, lens)
    lens_t[0] = tables.shape[1] * 16 + 7
    pagedkv.read_error_flags(cuda_ready, clear=True)
    pagedkv.paged_attention_decode_batched(q.to(cuda_ready), k.to(cuda_ready), v.to(cuda_ready),
                                           tables.to(cuda_ready), lens_t.to(cuda_ready), 0.125)
    assert pagedkv.read_error_flags(cuda_ready, clear=True) & _native.EFLAG_SEQ_LEN_RANGE


def test_reference_preconditions_raise_assertion(cuda_ready):
    inp = cases.make_attention_inputs(cases.ATTENTION_CASES["gqa7_qwen"])
    q, k, v, tables, lens = _device_inputs(inp, cuda_ready)
    with pytest.raises(AssertionError):
        pagedkv.paged_attention_decode_batched(q.float(), k, v, tables, lens, 0.125)
    with pytest.raises(AssertionError):
        pagedkv.paged_attention_decode_batched(q, k, v, tables.long(), lens, 0.125)
    with pytest.raises(AssertionError):
        pagedkv.paged_attention_decode_batched(q[:, :13], k, v, tables, lens, 0.125)
    with pytest.raises(AssertionError):
        pagedkv.paged_attention_decode_v2(q[0], k, v, tables[0, :1], 67, 0.125)


def test_pad_block_tables_matches_reference_semantics(cuda_ready):
    class BT:
        def __init__(self, ids):
            self.physical_block_ids = ids

    t = pagedkv.pad_block_tables([[3, 1], BT([7]), []], device=cuda_ready)
    assert t.dtype == torch.int32 and t.device.type == "cuda"
    assert t.cpu().tolist() == [[3, 1], [7, 0], [0, 0]]
    assert pagedkv.pad_block_tables([[], []], device=cuda_ready).shape == (2, 1)
    assert pagedkv.pad_block_tables([], device=cuda_ready).shape == (0, 0)


def test_list_entry_point_runs_kernel(cuda_ready, golden):
    arrays, _ = golden
    inp = cases.make_attention_inputs(cases.ATTENTION_CASES["batched_1_17_500_2000"])
    q, k, v, _, _ = _device_inputs(inp, cuda_ready)
    out = pagedkv.paged_attention_decode(q, k, v, inp["table_lists"], [int(x) for x in inp["lens"]], inp["scale"])
    torch.testing.assert_close(out.float().cpu(), torch.from_numpy(arrays["batched_1_17_500_2000__out"]),
                               atol=ATOL, rtol=RTOL)
