"""Generate the golden vectors by running the REFERENCE implementation.

Run in a checkout that has the reference (XVX-016/vLLM-inference-engine) on
disk; it is not needed afterwards:

    python tests/golden/make_golden.py --reference /path/to/vLLM-inference-engine

For every case of ``cases.py`` it regenerates the seeded inputs and calls

* ``engine.kernels.paged_attention.naive_reference_paged_attention``
  (reference engine/kernels/paged_attention.py:30-83) in fp32 on CPU, storing
  its output;
* ``engine.kernels.paged_attention_integration.paged_decode_attention_forward``
  (reference :65-176, batched branch) in fp16 on CPU, with its GPU-only kernel
  call replaced by the naive reference, storing a SHA-256 of the K/V pool after
  the append it performs at :150-160, the new K/V rows it wrote and the
  attention-layer output.

Outputs: ``golden.npz`` (arrays) and ``manifest.json`` (case parameters,
input hashes, pool hashes), both next to this script.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import cases  # noqa: E402


def _attention_goldens(ref_fn) -> tuple[dict, dict]:
    arrays, meta = {}, {}
    for name, case in cases.ATTENTION_CASES.items():
        inp = cases.make_attention_inputs(case)
        out = ref_fn(
            torch.from_numpy(inp["q"].astype(np.float32)),
            torch.from_numpy(inp["k_cache"].astype(np.float32)),
            torch.from_numpy(inp["v_cache"].astype(np.float32)),
            inp["table_lists"],
            [int(x) for x in inp["lens"]],
            inp["scale"],
        ).numpy()
        arrays[f"{name}__out"] = out.astype(np.float32)
        meta[name] = dict(
            params={k: v for k, v in case.items()},
            lens=[int(x) for x in inp["lens"]],
            input_sha256=cases.sha256_arrays(inp["q"], inp["k_cache"], inp["v_cache"], inp["tables"]),
        )
        print(f"attention {name}: N={len(inp['lens'])} lens={meta[name]['lens'][:6]} |out|max={np.abs(out).max():.3f}")
    return arrays, meta


class _FakeAttention(torch.nn.Module):
    """Just the attributes paged_decode_attention_forward reads."""

    def __init__(self, inp: dict, case: dict):
        super().__init__()
        hq, hkv, d = case["hq"], case["hkv"], case["d"]
        hidden = inp["hidden"]
        self.layer_idx = 0
        self.head_dim = d
        self.scaling = d ** -0.5
        self.q_proj = torch.nn.Linear(hidden, hq * d, bias=True, dtype=torch.float16)
        self.k_proj = torch.nn.Linear(hidden, hkv * d, bias=True, dtype=torch.float16)
        self.v_proj = torch.nn.Linear(hidden, hkv * d, bias=True, dtype=torch.float16)
        self.o_proj = torch.nn.Linear(hq * d, hidden, bias=False, dtype=torch.float16)
        with torch.no_grad():
            self.q_proj.weight.copy_(torch.from_numpy(inp["w_q"]))
            self.q_proj.bias.copy_(torch.from_numpy(inp["b_q"]))
            self.k_proj.weight.copy_(torch.from_numpy(inp["w_k"]))
            self.k_proj.bias.copy_(torch.from_numpy(inp["b_k"]))
            self.v_proj.weight.copy_(torch.from_numpy(inp["w_v"]))
            self.v_proj.bias.copy_(torch.from_numpy(inp["b_v"]))
            self.o_proj.weight.copy_(torch.from_numpy(inp["w_o"]))


def _append_goldens(ref_root: Path) -> tuple[dict, dict]:
    from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb

    import engine.kernels.paged_attention_integration as integ
    from engine.kernels.paged_attention import naive_reference_paged_attention
    from engine.memory.block_allocator import BlockTable, PhysicalBlockPool

    def cpu_batched(q, k_cache, v_cache, block_tables, seq_lens, scale):
        tables = [row.tolist() for row in block_tables]
        lens = [int(x) for x in seq_lens]
        return naive_reference_paged_attention(
            q.float(), k_cache.float(), v_cache.float(), tables, lens, scale
        ).to(q.dtype)

    integ.paged_attention_decode_batched = cpu_batched  # GPU-only Triton launch -> oracle

    arrays, meta = {}, {}
    for name, case in cases.APPEND_CASES.items():
        inp = cases.make_append_inputs(case)
        bs, hkv, d = case["bs"], case["hkv"], case["d"]
        pool = PhysicalBlockPool(
            num_blocks=case["num_blocks"], block_size=bs, num_layers=1, num_kv_heads=hkv,
            head_dim=d, dtype=torch.float16, device="cpu",
        )
        pool.k_cache[0].copy_(torch.from_numpy(inp["k_cache"]))
        pool.v_cache[0].copy_(torch.from_numpy(inp["v_cache"]))
        tables = [
            BlockTable(seq_id=i, block_size=bs, physical_block_ids=list(t), num_tokens=n)
            for i, (t, n) in enumerate(zip(inp["tables"], inp["lens"]))
        ]
        ctx = integ.PagedAttentionContext(pool=pool, block_tables=tables, seq_lens=list(inp["lens"]), block_size=bs)
        mod = _FakeAttention(inp, case)
        mod._paged_attention_context = ctx
        positions = np.asarray(inp["lens"], dtype=np.int64) - 1
        cos, sin = cases.rope_cos_sin(positions, d)
        cos_t = torch.from_numpy(cos).to(torch.float16)
        sin_t = torch.from_numpy(sin).to(torch.float16)
        h = torch.from_numpy(inp["h"])
        with torch.inference_mode():
            attn_out, _ = integ.paged_decode_attention_forward(mod, h, (cos_t, sin_t))
            # The rows the reference wrote, recomputed with the same calls (:103-109).
            bsz = h.shape[0]
            k = mod.k_proj(h).view(bsz, 1, -1, d).transpose(1, 2)
            qq = mod.q_proj(h).view(bsz, 1, -1, d).transpose(1, 2)
            v = mod.v_proj(h).view(bsz, 1, -1, d).transpose(1, 2)
            qq, k = apply_rotary_pos_emb(qq, k, cos_t, sin_t)
        k_new = k.squeeze(2).contiguous().numpy()
        v_new = v.squeeze(2).contiguous().numpy()
        arrays[f"{name}__k_new"] = k_new
        arrays[f"{name}__v_new"] = v_new
        arrays[f"{name}__q_rot"] = qq.squeeze(2).contiguous().numpy()
        arrays[f"{name}__attn_out"] = attn_out.float().numpy()
        meta[name] = dict(
            params=case,
            input_sha256=cases.sha256_arrays(inp["k_cache"], inp["v_cache"], inp["h"]),
            pool_after_sha256=cases.sha256_arrays(pool.k_cache[0].numpy(), pool.v_cache[0].numpy()),
        )
        print(f"append {name}: lens={inp['lens']} pool sha={meta[name]['pool_after_sha256'][:16]}")
    return arrays, meta


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    args = ap.parse_args()
    ref_root = Path(args.reference).resolve()
    sys.path.insert(0, str(ref_root))
    from engine.kernels.paged_attention import naive_reference_paged_attention

    torch.set_num_threads(8)
    a_arrays, a_meta = _attention_goldens(naive_reference_paged_attention)
    p_arrays, p_meta = _append_goldens(ref_root)
    np.savez_compressed(HERE / "golden.npz", **a_arrays, **p_arrays)
    manifest = {
        "generator": "tests/golden/make_golden.py",
        "reference_functions": {
            "attention": "engine/kernels/paged_attention.py:30-83 naive_reference_paged_attention (fp32, CPU)",
            "append": "engine/kernels/paged_attention_integration.py:65-176 paged_decode_attention_forward (fp16, CPU)",
        },
        "torch": torch.__version__,
        "numpy": np.__version__,
        "attention": a_meta,
        "append": p_meta,
    }
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True))
    print("wrote", HERE / "golden.npz", (HERE / "golden.npz").stat().st_size, "bytes")


if __name__ == "__main__":
    main()
