"""Deterministic input cases shared by the golden-vector script and the tests.

Inputs are regenerated from a seed with numpy's PCG64 ``Generator`` (values
rounded to fp16, so the kernels and the fp32 oracle see identical numbers);
the committed fixture stores the reference's OUTPUT for each case plus a
SHA-256 of the regenerated inputs, which the tests check before comparing.

Attention cases mirror the reference's own tests
(tests/test_paged_attention_reference.py: GQA 1/2/7 at :216-264, MQA with
block_size 8 at :291, the 2048-token shuffled case at :439-485, the x10
large-magnitude case at :488-537, the batched [1,17,500,2000] case at
:540-643) and, at reduced size, the BASELINE configurations 1 and 3.
"""
from __future__ import annotations

import hashlib
import math

import numpy as np

# name -> parameters. q_scale / k_scale multiply N(0,1) draws (before fp16
# rounding). "gpu": False marks head dims the CUDA library does not build;
# those pin the oracle only.
ATTENTION_CASES: dict[str, dict] = {
    "ref_contig_mha_d16": dict(hq=4, hkv=4, d=16, bs=8, lens=[24], seed=0, gpu=False),
    "ref_shuffled_d8": dict(hq=2, hkv=2, d=8, bs=4, lens=[20], seed=1, gpu=False),
    "ref_multi_var_d8": dict(hq=2, hkv=2, d=8, bs=4, lens=[12, 20, 8], seed=2, gpu=False),
    "gqa1_d32": dict(hq=8, hkv=8, d=32, bs=16, lens=[16, 37, 8], seed=101),
    "gqa2_d32": dict(hq=8, hkv=4, d=32, bs=16, lens=[16, 45, 9], seed=102),
    "gqa7_qwen": dict(hq=14, hkv=2, d=64, bs=16, lens=[13, 32, 67], seed=103),
    "gqa7_exact_block": dict(hq=14, hkv=2, d=64, bs=16, lens=[32], seed=204),
    "mqa4_bs8": dict(hq=4, hkv=1, d=64, bs=8, lens=[19], seed=205),
    "long_2048": dict(hq=14, hkv=2, d=64, bs=16, lens=[2048], seed=401, extra_blocks=20),
    "large_magnitude_x10": dict(hq=8, hkv=2, d=64, bs=16, lens=[250], seed=501, q_scale=10.0, k_scale=10.0),
    "batched_1_17_500_2000": dict(hq=14, hkv=2, d=64, bs=16, lens=[1, 17, 500, 2000], seed=601, extra_blocks=40),
    "cfg1_cpu_reference": dict(hq=14, hkv=2, d=64, bs=16, n=8, lens="uniform_1_512", seed=1, num_blocks=512),
    "cfg3_g1_d128": dict(hq=8, hkv=8, d=128, bs=16, n=6, lens="loguniform_16_8192", seed=31, q_scale=30.0),
    "cfg3_g2_d128": dict(hq=16, hkv=8, d=128, bs=16, n=6, lens="loguniform_16_8192", seed=32, q_scale=30.0),
    "cfg3_g4_d128": dict(hq=32, hkv=8, d=128, bs=16, n=6, lens="loguniform_16_8192", seed=33, q_scale=30.0),
    "cfg3_g7_d128": dict(hq=56, hkv=8, d=128, bs=16, n=6, lens="loguniform_16_8192", seed=34, q_scale=30.0),
    "bs32_gqa7": dict(hq=14, hkv=2, d=64, bs=32, lens=[31, 64, 97, 300], seed=71),
    "d256_gqa4": dict(hq=8, hkv=2, d=256, bs=16, lens=[5, 130, 700], seed=72),
    "gqa8_d64": dict(hq=16, hkv=2, d=64, bs=16, lens=[100, 1000, 3], seed=73),
    "gqa16_d128": dict(hq=16, hkv=1, d=128, bs=16, lens=[77, 513], seed=74),
}

# Decode-append cases: the reference's batched decode forward
# (paged_attention_integration.py:65-176) run on CPU in fp16; the golden is the
# pool after its append (:150-160), hashed.
APPEND_CASES: dict[str, dict] = {
    "append_qwen_shape": dict(hq=14, hkv=2, d=64, bs=16, lens=[5, 16, 17, 33, 1], num_blocks=48, seed=901),
    "append_bs8_mqa": dict(hq=4, hkv=1, d=64, bs=8, lens=[8, 9, 24, 2], num_blocks=24, seed=902),
}


def _draw_lens(spec, n: int, rng: np.random.Generator) -> list[int]:
    if spec == "uniform_1_512":
        return [int(x) for x in rng.integers(1, 513, size=n)]
    if spec == "loguniform_16_8192":
        return [int(round(math.exp(x))) for x in rng.uniform(math.log(16), math.log(8192), size=n)]
    return [int(x) for x in spec]


def make_attention_inputs(case: dict) -> dict:
    """Regenerate one attention case: fp16 q, pools, int32 tables, lens."""
    rng = np.random.default_rng(case["seed"])
    hq, hkv, d, bs = case["hq"], case["hkv"], case["d"], case["bs"]
    lens_spec = case["lens"]
    n = case.get("n", len(lens_spec) if isinstance(lens_spec, list) else 0)
    lens = _draw_lens(lens_spec, n, rng)
    need = [max(1, (x + bs - 1) // bs) for x in lens]
    num_blocks = case.get("num_blocks") or (sum(need) + case.get("extra_blocks", 5 + sum(need)))
    assert num_blocks >= sum(need)
    perm = rng.permutation(num_blocks).astype(np.int32)
    width = max(need)
    tables = np.zeros((len(lens), width), dtype=np.int32)
    table_lists: list[list[int]] = []
    at = 0
    for i, k in enumerate(need):
        row = perm[at : at + k]
        at += k
        tables[i, :k] = row
        table_lists.append([int(x) for x in row])
    q_scale = case.get("q_scale", 1.0)
    k_scale = case.get("k_scale", 1.0)
    q = (rng.standard_normal((len(lens), hq, d), dtype=np.float32) * q_scale).astype(np.float16)
    k_cache = (rng.standard_normal((num_blocks, bs, hkv, d), dtype=np.float32) * k_scale).astype(np.float16)
    v_cache = rng.standard_normal((num_blocks, bs, hkv, d), dtype=np.float32).astype(np.float16)
    return dict(
        q=q, k_cache=k_cache, v_cache=v_cache, tables=tables, table_lists=table_lists,
        lens=np.asarray(lens, dtype=np.int32), scale=1.0 / math.sqrt(d),
    )


def make_append_inputs(case: dict) -> dict:
    """Regenerate one append case: fp16 module weights, hidden states,
    positions, the initial pool and the block tables."""
    rng = np.random.default_rng(case["seed"])
    hq, hkv, d, bs = case["hq"], case["hkv"], case["d"], case["bs"]
    lens = [int(x) for x in case["lens"]]
    num_blocks = case["num_blocks"]
    hidden = 64
    need = [(x + bs - 1) // bs for x in lens]
    perm = rng.permutation(num_blocks)
    tables, at = [], 0
    for k in need:
        tables.append([int(x) for x in perm[at : at + k]])
        at += k
    w = lambda o, i: (rng.standard_normal((o, i), dtype=np.float32) / math.sqrt(i)).astype(np.float16)
    return dict(
        hidden=hidden,
        w_q=w(hq * d, hidden), b_q=(rng.standard_normal(hq * d, dtype=np.float32) * 0.1).astype(np.float16),
        w_k=w(hkv * d, hidden), b_k=(rng.standard_normal(hkv * d, dtype=np.float32) * 0.1).astype(np.float16),
        w_v=w(hkv * d, hidden), b_v=(rng.standard_normal(hkv * d, dtype=np.float32) * 0.1).astype(np.float16),
        w_o=w(hidden, hq * d),
        h=rng.standard_normal((len(lens), 1, hidden), dtype=np.float32).astype(np.float16),
        k_cache=rng.standard_normal((num_blocks, bs, hkv, d), dtype=np.float32).astype(np.float16),
        v_cache=rng.standard_normal((num_blocks, bs, hkv, d), dtype=np.float32).astype(np.float16),
        tables=tables, lens=lens,
    )


def rope_cos_sin(positions: np.ndarray, d: int, theta: float = 1000000.0) -> tuple[np.ndarray, np.ndarray]:
    """Standard rotary cos/sin tables [B, 1, d] (half-split layout)."""
    inv = 1.0 / (theta ** (np.arange(0, d, 2, dtype=np.float64) / d))
    ang = positions.astype(np.float64)[:, None] * inv[None, :]
    emb = np.concatenate([ang, ang], axis=-1)
    return np.cos(emb)[:, None, :].astype(np.float32), np.sin(emb)[:, None, :].astype(np.float32)


def sha256_arrays(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()
