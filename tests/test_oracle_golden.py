"""CPU: the oracle restatement against the reference's own golden outputs.

The golden vectors were produced by running the reference implementation
(tests/golden/make_golden.py); these tests pin ``oracle/paged_ref.py`` to it
before the oracle is trusted as the checker of the CUDA path.
"""
import numpy as np
import pytest
import torch

import cases
from oracle import paged_ref


@pytest.mark.parametrize("name", list(cases.ATTENTION_CASES))
def test_attention_oracle_matches_reference_golden(golden, name):
    arrays, manifest = golden
    case = cases.ATTENTION_CASES[name]
    inp = cases.make_attention_inputs(case)
    meta = manifest["attention"][name]
    assert cases.sha256_arrays(inp["q"], inp["k_cache"], inp["v_cache"], inp["tables"]) == meta["input_sha256"], (
        "regenerated inputs differ from the ones the golden was made with"
    )
    assert [int(x) for x in inp["lens"]] == meta["lens"]
    expected = arrays[f"{name}__out"]
    got = paged_ref.paged_attention_ref(
        torch.from_numpy(inp["q"].astype(np.float32)),
        torch.from_numpy(inp["k_cache"].astype(np.float32)),
        torch.from_numpy(inp["v_cache"].astype(np.float32)),
        inp["table_lists"],
        [int(x) for x in inp["lens"]],
        inp["scale"],
    ).numpy()
    # Same fp32 math, different summation order: a few ulp of the scores,
    # amplified by the score magnitude (q and k pre-scaled up to x30).
    tol = 2e-5 * case.get("q_scale", 1.0) * case.get("k_scale", 1.0)
    np.testing.assert_allclose(got, expected, atol=tol, rtol=tol)


@pytest.mark.parametrize("name", ["gqa7_qwen", "large_magnitude_x10", "cfg1_cpu_reference", "cfg3_g7_d128"])
def test_attention_f64_oracle_agrees(golden, name):
    arrays, _ = golden
    inp = cases.make_attention_inputs(cases.ATTENTION_CASES[name])
    got = paged_ref.paged_attention_ref_f64(
        inp["q"], inp["k_cache"], inp["v_cache"], inp["table_lists"], inp["lens"], inp["scale"]
    )
    np.testing.assert_allclose(got, arrays[f"{name}__out"], atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("name", list(cases.APPEND_CASES))
def test_append_oracle_matches_reference_pool(golden, name):
    arrays, manifest = golden
    case = cases.APPEND_CASES[name]
    inp = cases.make_append_inputs(case)
    meta = manifest["append"][name]
    assert cases.sha256_arrays(inp["k_cache"], inp["v_cache"], inp["h"]) == meta["input_sha256"]
    k_cache = inp["k_cache"].copy()
    v_cache = inp["v_cache"].copy()
    slots = paged_ref.decode_slots(inp["tables"], inp["lens"], case["bs"])
    paged_ref.kv_append_ref(k_cache, v_cache, arrays[f"{name}__k_new"], arrays[f"{name}__v_new"], slots)
    assert cases.sha256_arrays(k_cache, v_cache) == meta["pool_after_sha256"], "append restatement is not bit-exact"


def test_copy_blocks_oracle_semantics():
    rng = np.random.default_rng(5)
    layers = 3
    ks = [rng.standard_normal((10, 4, 2, 8)).astype(np.float16) for _ in range(layers)]
    vs = [rng.standard_normal((10, 4, 2, 8)).astype(np.float16) for _ in range(layers)]
    k0 = [k.copy() for k in ks]
    v0 = [v.copy() for v in vs]
    mapping = np.array([[1, 7], [3, 2], [9, 0]], dtype=np.int64)
    paged_ref.copy_blocks_ref(ks, vs, mapping)
    for layer in range(layers):
        for src, dst in mapping:
            assert np.array_equal(ks[layer][dst], k0[layer][src])
            assert np.array_equal(vs[layer][dst], v0[layer][src])
        untouched = [b for b in range(10) if b not in mapping[:, 1]]
        assert np.array_equal(ks[layer][untouched], k0[layer][untouched])


def test_oracle_zero_length_sequence_is_zero():
    inp = cases.make_attention_inputs(cases.ATTENTION_CASES["gqa7_qwen"])
    lens = [0, 13, 0]
    out = paged_ref.paged_attention_ref(
        torch.from_numpy(inp["q"].astype(np.float32)),
        torch.from_numpy(inp["k_cache"].astype(np.float32)),
        torch.from_numpy(inp["v_cache"].astype(np.float32)),
        inp["table_lists"], lens, inp["scale"],
    )
    assert torch.count_nonzero(out[0]) == 0 and torch.count_nonzero(out[2]) == 0
    assert torch.count_nonzero(out[1]) > 0
