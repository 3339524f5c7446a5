#!/usr/bin/env python
"""Benchmark of the B200 paged KV-cache decode path (one JSON line on rank 0).

Workload (one GPU's shard): 256 sequences x 2048-token
contexts, Qwen2.5-0.5B attention shape (14 query / 2 kv heads, head_dim 64),
block_size 16, fp16 pool of 40960 blocks with shuffled block tables. One
"step" = one decode layer-step of the hot path over that batch: the KV append
of 256 new tokens through a slot mapping, then batched decode attention over
all 256 contexts (which include the appended token).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun, one process per GPU; sequences are sharded
data-parallel (each rank owns its own pool, weak scaling) and nothing crosses
GPUs on the data path: torch.distributed (NCCL) is used only for the barrier
around the timed region and the max-over-ranks of the elapsed time.

``--impl reference`` times the reference algorithm's CPU path (the pinned
oracle restatement of engine/kernels/paged_attention.py:30-83 plus the append
of paged_attention_integration.py:150-160, torch fp32 on all host threads) on
bounded samples of the same workload; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import random
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "vllm-inference-engine_b200"))
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

# ---- workload ---------------------------------------------------------------
NUM_SEQS = 256
NUM_Q_HEADS = 14
NUM_KV_HEADS = 2
HEAD_DIM = 64
BLOCK_SIZE = 16
CTX = 2048
NUM_BLOCKS = 40960
ELEM = 2  # fp16 bytes
L2_BYTES = 126 * 1024 * 1024

WORKLOAD = (
    "cfg2: KV append (256 tokens) + paged GQA decode attention, 256 seqs x 2048 ctx, "
    "14q/2kv heads, head_dim 64, block_size 16, fp16 pool 40960 blocks, shuffled tables"
)


def attention_bytes(num_seqs: int, ctx: int, max_blocks: int) -> int:
    """Algorithmic bytes of one decode-attention call: every K and V row of every
    context once, plus q, out, the block tables and seq_lens."""
    kv = num_seqs * ctx * NUM_KV_HEADS * HEAD_DIM * ELEM * 2
    qo = num_seqs * NUM_Q_HEADS * HEAD_DIM * ELEM * 2
    tables = num_seqs * max_blocks * 4 + num_seqs * 4
    return kv + qo + tables


def append_bytes(num_tokens: int) -> int:
    """Algorithmic bytes of one KV append: read new K/V, write them, read slots."""
    row = NUM_KV_HEADS * HEAD_DIM * ELEM
    return num_tokens * row * 2 * 2 + num_tokens * 8


def attention_flops(num_seqs: int, ctx: int) -> int:
    return num_seqs * ctx * 4 * HEAD_DIM * NUM_Q_HEADS


def build_shard(rank: int, device, num_seqs: int = NUM_SEQS, ctx: int = CTX, num_blocks: int = NUM_BLOCKS):
    """Seeded per-rank shard: pool, shuffled tables, new-token K/V, slots, q."""
    g = torch.Generator(device="cpu").manual_seed(1000 + rank)
    blocks_per_seq = (ctx + BLOCK_SIZE - 1) // BLOCK_SIZE
    assert num_seqs * blocks_per_seq <= num_blocks
    perm = list(range(num_blocks))
    random.Random(42 + rank).shuffle(perm)
    tables = torch.tensor(perm[: num_seqs * blocks_per_seq], dtype=torch.int32).view(num_seqs, blocks_per_seq)
    lens = torch.full((num_seqs,), ctx, dtype=torch.int32)
    pos = lens.to(torch.int64) - 1
    slots = tables.to(torch.int64).gather(1, (pos // BLOCK_SIZE).view(-1, 1)).view(-1) * BLOCK_SIZE + pos % BLOCK_SIZE
    shard = dict(
        tables=tables, lens=lens, slots=slots,
        q=torch.randn(num_seqs, NUM_Q_HEADS, HEAD_DIM, generator=g).half(),
        k_new=torch.randn(num_seqs, NUM_KV_HEADS, HEAD_DIM, generator=g).half(),
        v_new=torch.randn(num_seqs, NUM_KV_HEADS, HEAD_DIM, generator=g).half(),
    )
    if device is not None:
        gd = torch.Generator(device=device).manual_seed(2000 + rank)
        shape = (num_blocks, BLOCK_SIZE, NUM_KV_HEADS, HEAD_DIM)
        shard["k_cache"] = torch.randn(shape, generator=gd, device=device, dtype=torch.float16)
        shard["v_cache"] = torch.randn(shape, generator=gd, device=device, dtype=torch.float16)
    return shard


# ---- clocks -------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling while the timed region runs."""

    QUERY = (
        "timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, gpu_indices: list[int], interval_ms: int = 50):
        self.gpus = gpu_indices
        self.interval = interval_ms
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", str(self.interval)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
        except (OSError, ValueError):
            self.proc = None
        time.sleep(0.3)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.2)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        n = 0
        for line in out.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                idx = int(parts[1])
            except ValueError:
                continue
            if idx not in self.gpus:
                continue
            n += 1
            try:
                sm.append(float(parts[2]))
                smax.append(float(parts[3]))
            except ValueError:
                pass
            for name, flag in zip(names, parts[6:10]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(smax) if smax else None,
            "reasons": sorted(reasons),
            "samples": n,
        }


# ---- reference arm / CPU baseline ---------------------------------------------
def _cpu_sample(num_seqs: int):
    """A bounded sample of the workload for the CPU reference: ``num_seqs``
    sequences of the rank-0 shard with their pool blocks gathered into a
    compact pool (same values the GPU reads; fp32 as the reference's CPU path)."""
    shard = build_shard(0, None, num_seqs=num_seqs, ctx=CTX, num_blocks=num_seqs * (CTX // BLOCK_SIZE))
    g = torch.Generator().manual_seed(7)
    nb = num_seqs * (CTX // BLOCK_SIZE)
    k = torch.randn(nb, BLOCK_SIZE, NUM_KV_HEADS, HEAD_DIM, generator=g).half().float()
    v = torch.randn(nb, BLOCK_SIZE, NUM_KV_HEADS, HEAD_DIM, generator=g).half().float()
    return shard, k, v


def cpu_reference_step(shard, k, v) -> None:
    from oracle import paged_ref

    tables = shard["tables"].tolist()
    lens = shard["lens"].tolist()
    kc, vc = k.numpy(), v.numpy()
    paged_ref.kv_append_ref(kc, vc, shard["k_new"].float().numpy(), shard["v_new"].float().numpy(), shard["slots"].numpy())
    paged_ref.paged_attention_ref(shard["q"].float(), k, v, tables, lens, 1.0 / math.sqrt(HEAD_DIM))


def time_cpu_reference(num_seqs: int, min_seconds: float) -> dict:
    shard, k, v = _cpu_sample(num_seqs)
    threads = torch.get_num_threads()
    cpu_reference_step(shard, k, v)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        cpu_reference_step(shard, k, v)
        n += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    per = el / n
    nbytes = attention_bytes(num_seqs, CTX, CTX // BLOCK_SIZE) + append_bytes(num_seqs)
    return {
        "value": round(nbytes / per / 1e9, 3),
        "unit": "GB/s",
        "cores": threads,
        "kind": "port",
        "sample": (
            f"{num_seqs} of the 256 sequences (2048 tokens each), fp32 torch restatement of the reference's "
            f"naive_reference_paged_attention + append, {n} calls over {el:.1f} s, {threads} threads "
            f"(os.cpu_count()={os.cpu_count()})"
        ),
        "seconds_per_sample": per,
    }


def run_reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    sample = 8
    shard, k, v = _cpu_sample(sample)
    for _ in range(args.warmup):
        cpu_reference_step(shard, k, v)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        cpu_reference_step(shard, k, v)
        times.append(time.perf_counter() - t0)
    per = sum(times) / len(times)
    nbytes = attention_bytes(sample, CTX, CTX // BLOCK_SIZE) + append_bytes(sample)
    value = nbytes / per / 1e9
    threads = torch.get_num_threads()
    line = {
        "impl": "reference",
        "metric": "paged-decode KV HBM GB/s",
        "value": round(value, 3),
        "unit": "GB/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(per * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample_seqs_per_step": sample, "parallelism": "host cores of rank 0"},
        "cpu_baseline": {
            "value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{sample} sequences x 2048 tokens per step (fp32 oracle restatement, torch CPU)",
        },
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---- our arm ------------------------------------------------------------------
def _dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and world > 1:
        raise SystemExit(f"--gpus {args.gpus} disagrees with WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=torch.device("cuda", local))
    return dist, rank, world, local


def _max_over_ranks(dist, value: float, device) -> float:
    if dist is None:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _sum_over_ranks(dist, value: float, device) -> float:
    if dist is None:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def _read_traffic(kernel: str) -> int | None:
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        data = json.loads(p.read_text())
        entry = data.get(kernel)
        return int(entry["bytes_per_launch"]) if entry else None
    except (ValueError, KeyError, TypeError):
        return None


def run_ours(args) -> None:
    import pagedkv
    from pagedkv import _native

    dist, rank, world, local = _dist_setup(args)
    dev = torch.device("cuda", local)
    _native.lib()
    shard = build_shard(rank, dev)
    q = shard["q"].to(dev)
    tables = shard["tables"].to(dev)
    lens = shard["lens"].to(dev)
    slots = shard["slots"].to(dev)
    k_new = shard["k_new"].to(dev)
    v_new = shard["v_new"].to(dev)
    kc, vc = shard["k_cache"], shard["v_cache"]
    scale = 1.0 / math.sqrt(HEAD_DIM)
    stream = torch.cuda.current_stream(dev)

    def step():
        pagedkv.kv_append(k_new, v_new, kc, vc, slots)
        return pagedkv.paged_attention_decode_batched(q, kc, vc, tables, lens, scale)

    # correctness spot-check of this shard against the oracle (2 sequences)
    out = step()
    torch.cuda.synchronize(dev)
    from oracle import paged_ref  # checker only, outside the timed region

    sel = [0, NUM_SEQS - 1]
    used = sorted({int(b) for s in sel for b in shard["tables"][s].tolist()})
    remap = {b: i for i, b in enumerate(used)}
    idx = torch.tensor(used, device=dev)
    ref = paged_ref.paged_attention_ref(
        q[sel].float().cpu(), kc[idx].float().cpu(), vc[idx].float().cpu(),
        [[remap[int(b)] for b in shard["tables"][s].tolist()] for s in sel], [CTX, CTX], scale,
    )
    max_err = (out[sel].float().cpu() - ref).abs().max().item()
    if not max_err < 2e-3 + 2e-3 * ref.abs().max().item():
        raise SystemExit(f"bench spot-check failed: max |err| {max_err}")
    launches_attn, family = pagedkv.last_decode_launch_info()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)

    # The decode step (append + attention) and the attention alone, each
    # captured once as a CUDA graph and replayed: a serving engine replays the
    # decode step the same way, so the device time is not bounded by Python.
    g_step = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_step):
        step()
    g_attn = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_attn):
        pagedkv.paged_attention_decode_batched(q, kc, vc, tables, lens, scale)
    for _ in range(args.warmup):
        g_step.replay()
        g_attn.replay()
    torch.cuda.synchronize(dev)

    def timed(fn, n):
        if dist:
            dist.barrier()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(n):
            fn()
        b.record(stream)
        torch.cuda.synchronize(dev)
        if dist:
            dist.barrier()
        return a.elapsed_time(b)

    sampler = ClockSampler([local] if world == 1 else list(range(world))) if rank == 0 else None
    if sampler:
        sampler.start()
    total_ms = timed(g_step.replay, args.steps)
    clocks = sampler.stop() if sampler else None
    attn_ms = timed(g_attn.replay, args.steps) / args.steps
    eager_ms = timed(step, max(10, args.steps // 10)) / max(10, args.steps // 10)
    append_ms = _max_over_ranks(dist, max(0.0, total_ms / args.steps - attn_ms), dev)
    total_ms = _max_over_ranks(dist, total_ms, dev)
    attn_ms_max = _max_over_ranks(dist, attn_ms, dev)
    eager_ms = _max_over_ranks(dist, eager_ms, dev)
    ms_per_step = total_ms / args.steps

    max_blocks = CTX // BLOCK_SIZE
    a_bytes = attention_bytes(NUM_SEQS, CTX, max_blocks)
    p_bytes = append_bytes(NUM_SEQS)
    step_bytes = a_bytes + p_bytes
    value = world * step_bytes / (ms_per_step * 1e-3) / 1e9

    # ---- end to end through the public API from pinned host buffers -------------
    h_q = shard["q"].pin_memory()
    h_k = shard["k_new"].pin_memory()
    h_v = shard["v_new"].pin_memory()
    h_slots = shard["slots"].pin_memory()
    h_tables = shard["tables"].pin_memory()
    h_lens = shard["lens"].pin_memory()
    h_out = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in (h_q, h_k, h_v, h_slots, h_tables, h_lens))
    d2h = h_out.numel() * h_out.element_size()

    def e2e_step():
        dq = h_q.to(dev, non_blocking=True)
        dk = h_k.to(dev, non_blocking=True)
        dv = h_v.to(dev, non_blocking=True)
        ds = h_slots.to(dev, non_blocking=True)
        dt = h_tables.to(dev, non_blocking=True)
        dl = h_lens.to(dev, non_blocking=True)
        pagedkv.kv_append(dk, dv, kc, vc, ds)
        o = pagedkv.paged_attention_decode_batched(dq, kc, vc, dt, dl, scale)
        h_out.copy_(o, non_blocking=True)

    for _ in range(max(3, args.warmup)):
        e2e_step()
    torch.cuda.synchronize(dev)
    if dist:
        dist.barrier()
    e_s, e_e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_s.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e_e.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = _max_over_ranks(dist, e_s.elapsed_time(e_e), dev) / args.steps
    e2e_value = world * step_bytes / (e2e_ms * 1e-3) / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        torch.set_num_threads(os.cpu_count() or 1)
        cpu = time_cpu_reference(num_seqs=16, min_seconds=args.cpu_seconds)
        cpu.pop("seconds_per_sample", None)

    peaks = {}
    pp = ROOT / "MEASURED_PEAKS.json"
    if pp.exists():
        peaks = json.loads(pp.read_text())
    peak = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    achieved = a_bytes / (attn_ms * 1e-3) / 1e9
    kernel_name = f"decode_{family}"
    traffic = _read_traffic(kernel_name)
    launches_per_step = 1 + launches_attn  # append + (counter reset and) attention kernel
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": "paged-decode KV HBM GB/s",
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic",
        "config": {
            "workload": WORKLOAD,
            "num_seqs_per_gpu": NUM_SEQS,
            "ctx": CTX,
            "heads": f"{NUM_Q_HEADS}q/{NUM_KV_HEADS}kv",
            "head_dim": HEAD_DIM,
            "block_size": BLOCK_SIZE,
            "num_blocks": NUM_BLOCKS,
            "decode_kernel": family,
            "l2": f"inputs exceed L2: {a_bytes / 1e6:.1f} MB read per step vs {L2_BYTES / 2**20:.0f} MiB L2, no flush",
            "parallelism": f"dp{world}: sequences sharded, one pool per GPU, no collective on the data path",
            "bytes_per_step": step_bytes,
        },
        "decode_tokens_per_s": round(world * NUM_SEQS / (ms_per_step * 1e-3), 1),
        "attention_ms": round(attn_ms_max, 5),
        "append_ms": round(append_ms, 5),
        "timing": "CUDA-graph replay of the step (append + attention), CUDA events on the launch stream",
        "eager_ms_per_step": round(eager_ms, 5),
        "roofline": {
            "bound": "hbm",
            "kernel": kernel_name,
            "achieved": round(achieved, 1),
            "peak": peak,
            "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured" else "fallback 6650 GB/s",
            "unit": "GB/s",
            "frac": round(achieved / peak, 4),
            "traffic": traffic,
            "algorithmic_bytes_per_launch": a_bytes,
            "flops_per_launch": attention_flops(NUM_SEQS, CTX),
        },
        "cpu_baseline": cpu,
        "e2e": {
            "value": round(e2e_value, 2),
            "unit": "GB/s",
            "ms_per_step": round(e2e_ms, 5),
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "api": "pagedkv.kv_append + pagedkv.paged_attention_decode_batched from pinned host buffers",
        },
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
        "spot_check_max_abs_err": max_err,
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference_arm(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
