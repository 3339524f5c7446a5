#!/usr/bin/env python
"""Benchmark of the B200 paged KV-cache decode path (one JSON line on rank 0).

Default workload (one GPU's shard): 256 sequences x
2048-token contexts, Qwen2.5-0.5B attention shape (14 query / 2 kv heads,
head_dim 64), block_size 16, fp16 pools of 40960 blocks with shuffled block
tables. One "step" = one decode step of the hot path over that batch in
every layer of the model (``--layers``, 24 for Qwen2.5-0.5B, each layer its
own pool): per layer, the KV append of 256 new tokens through a slot mapping,
then batched decode attention over all 256 contexts (which include the
appended token). The line also carries ``model_decode``: decode tokens/s of
the whole random-init model (BASELINE config 5's architecture) over a short
saturated trace per GPU.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload cfg1|cfg2|cfg3|cfg4|cfg4-cow|cfg5|ops|d256|cuda-core] [--gqa G]
                  [--layers L] [--model-requests R]

Extra workloads (not the headline): ``cfg1`` = BASELINE config 1 (the
reference's CPU case: 8 sequences of U[1,512] tokens, 512-block pool; the CPU
reference is timed on all host threads and on one); ``cfg3`` = config 3 (head_dim
128, 8 kv heads, GQA G, 128 sequences with log-uniform lengths 16..8192,
q x30); ``cfg4`` = config 4 (512 sequences in 8 groups sharing a 1024-token
prefix + 256 own tokens; roofline over the unique bytes); ``cfg4-cow`` = the
same with each sequence's last block shared by its group when the step
starts and copied to the sequence's private block (all layers) before its
append; ``cfg5`` = config 5 alone (``--requests`` at ``--rate`` per GPU);
``ops`` = the pool-write kernels alone; ``d256`` = the head_dim-256 mode
(64 x 2048 tokens, 8 query / 4 kv heads; not a BASELINE config);
``cuda-core`` = the CUDA-core decode kernel alone, which serves the block
sizes the tensor-core kernel does not take (here block_size 4).

N > 1 runs under torchrun, one process per GPU; sequences are sharded
data-parallel (each rank owns its own pools, weak scaling) and nothing
crosses GPUs on the data path: a gloo (host) process group carries only the
barrier around each timed region and the max / sum of the per-rank timings.

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
from dataclasses import dataclass
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "vllm-inference-engine_b200"))
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

L2_BYTES = 126 * 1024 * 1024
ELEM = 2  # fp16 bytes
METRIC = "paged-decode KV HBM GB/s"


# ---- workloads ------------------------------------------------------------------
@dataclass
class Workload:
    """One GPU's shard: host tensors of the step's inputs and the pool shape."""

    name: str
    description: str
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    block_size: int
    num_blocks: int
    tables: torch.Tensor        # int32 [N, W]
    lens: torch.Tensor          # int32 [N] (include the appended token)
    slots: torch.Tensor         # int64 [N] slot of the appended token
    q: torch.Tensor             # fp16 [N, Hq, D]
    k_new: torch.Tensor         # fp16 [N, Hkv, D]
    v_new: torch.Tensor
    pairs: torch.Tensor | None  # int64 [M, 2] copy-on-write (src, dst), or None

    @property
    def num_seqs(self) -> int:
        return int(self.lens.numel())

    @property
    def row_bytes(self) -> int:
        return self.num_kv_heads * self.head_dim * ELEM

    def attention_bytes(self) -> int:
        """Algorithmic bytes of one decode-attention call: every K and V row of
        every context once (shared prefixes counted per sequence, as the
        reference's formula does), plus q, out, the block tables and lengths."""
        kv = int(self.lens.to(torch.int64).sum()) * self.row_bytes * 2
        qo = self.num_seqs * self.num_q_heads * self.head_dim * ELEM * 2
        return kv + qo + self.tables.numel() * 4 + self.num_seqs * 4

    def append_bytes(self) -> int:
        """Read new K/V, write them into the pool, read the slots."""
        return self.num_seqs * self.row_bytes * 2 * 2 + self.num_seqs * 8

    def copy_bytes(self, layers: int = 1) -> int:
        """Copy-on-write: read + write of each pair's K and V block in every
        layer, plus the pair list."""
        if self.pairs is None:
            return 0
        block = self.block_size * self.row_bytes
        return int(self.pairs.shape[0]) * (layers * block * 2 * 2 + 16)

    def step_bytes(self, layers: int = 1) -> int:
        """A decode step over ``layers`` layers: the copy-on-write copy (one
        launch for all layers), then per layer the append and the attention."""
        return layers * (self.attention_bytes() + self.append_bytes()) + self.copy_bytes(layers)

    def attention_unique_bytes(self) -> int:
        """Attention bytes counting each distinct K/V block once (shared
        prefixes read once from HBM) plus q, out, tables and lengths."""
        qo = self.num_seqs * self.num_q_heads * self.head_dim * ELEM * 2
        return self.unique_kv_bytes() + qo + self.tables.numel() * 4 + self.num_seqs * 4

    def flops(self) -> int:
        return int(self.lens.to(torch.int64).sum()) * 4 * self.head_dim * self.num_q_heads

    def unique_kv_bytes(self) -> int:
        """K/V bytes of the distinct blocks the step reads (shared prefixes once)."""
        blocks = set()
        for s in range(self.num_seqs):
            nb = (int(self.lens[s]) + self.block_size - 1) // self.block_size
            blocks.update(self.tables[s, :nb].tolist())
        return len(blocks) * self.block_size * self.row_bytes * 2


def _slots_for(tables: torch.Tensor, lens: torch.Tensor, bs: int) -> torch.Tensor:
    pos = lens.to(torch.int64) - 1
    blk = tables.to(torch.int64).gather(1, (pos // bs).view(-1, 1)).view(-1)
    return blk * bs + pos % bs


def _tables_from_lists(rows: list[list[int]]) -> torch.Tensor:
    width = max(1, max(len(r) for r in rows))
    t = torch.zeros(len(rows), width, dtype=torch.int32)
    for i, r in enumerate(rows):
        t[i, : len(r)] = torch.tensor(r, dtype=torch.int32)
    return t


def _qkv(g: torch.Generator, n: int, hq: int, hkv: int, d: int, q_scale: float = 1.0):
    q = (torch.randn(n, hq, d, generator=g) * q_scale).half()
    return q, torch.randn(n, hkv, d, generator=g).half(), torch.randn(n, hkv, d, generator=g).half()


def build_shard(rank: int, device=None, num_seqs: int = 256, ctx: int = 2048, num_blocks: int = 40960):
    """Config 2 shard as a dict (seeded per rank): shuffled tables, lengths,
    slots of the appended tokens, q and the new K/V; with a device, also the
    N(0,1) fp16 K/V pools."""
    bs, hq, hkv, d = 16, 14, 2, 64
    g = torch.Generator(device="cpu").manual_seed(1000 + rank)
    blocks_per_seq = (ctx + bs - 1) // bs
    assert num_seqs * blocks_per_seq <= num_blocks
    perm = list(range(num_blocks))
    random.Random(42 + rank).shuffle(perm)
    tables = torch.tensor(perm[: num_seqs * blocks_per_seq], dtype=torch.int32).view(num_seqs, blocks_per_seq)
    lens = torch.full((num_seqs,), ctx, dtype=torch.int32)
    q, k_new, v_new = _qkv(g, num_seqs, hq, hkv, d)
    shard = dict(tables=tables, lens=lens, slots=_slots_for(tables, lens, bs), q=q, k_new=k_new, v_new=v_new)
    if device is not None:
        shard.update(make_pools(rank, device, num_blocks, bs, hkv, d))
    return shard


def make_pools(rank: int, device, num_blocks: int, bs: int, hkv: int, d: int) -> dict:
    gd = torch.Generator(device=device).manual_seed(2000 + rank)
    shape = (num_blocks, bs, hkv, d)
    return dict(
        k_cache=torch.randn(shape, generator=gd, device=device, dtype=torch.float16),
        v_cache=torch.randn(shape, generator=gd, device=device, dtype=torch.float16),
    )


def make_workload(name: str, rank: int, gqa: int = 7) -> Workload:
    if name == "cfg2":
        s = build_shard(rank)
        return Workload(
            "cfg2",
            "cfg2: KV append (256 tokens) + paged GQA decode attention, 256 seqs x 2048 ctx, 14q/2kv heads, "
            "head_dim 64, block_size 16, fp16 pool 40960 blocks, shuffled tables",
            14, 2, 64, 16, 40960, s["tables"], s["lens"], s["slots"], s["q"], s["k_new"], s["v_new"], None,
        )
    if name == "cfg1":
        n, hq, hkv, d, bs, nb = 8, 14, 2, 64, 16, 512
        rng = np.random.default_rng(3100 + rank)
        lens_l = [int(x) for x in rng.integers(1, 513, n)]
        perm = list(range(nb))
        random.Random(45 + rank).shuffle(perm)
        rows, at = [], 0
        for x in lens_l:
            c = (x + bs - 1) // bs
            rows.append(perm[at : at + c])
            at += c
        tables = _tables_from_lists(rows)
        lens = torch.tensor(lens_l, dtype=torch.int32)
        g = torch.Generator().manual_seed(1050 + rank)
        q, k_new, v_new = _qkv(g, n, hq, hkv, d)
        return Workload(
            "cfg1",
            "cfg1: KV append + paged decode attention, 8 seqs, lengths U[1,512], 14q/2kv heads, head_dim 64, "
            "block_size 16, pool 512 blocks, shuffled tables (the reference's CPU case; fp16 on the GPU, "
            "the CPU reference in fp32)",
            hq, hkv, d, bs, nb, tables, lens, _slots_for(tables, lens, bs), q, k_new, v_new, None,
        )
    if name == "cfg3":
        n, hkv, d, bs = 128, 8, 128, 16
        hq = hkv * gqa
        rng = np.random.default_rng(3000 + rank)
        lens_l = [int(round(math.exp(x))) for x in rng.uniform(math.log(16), math.log(8192), n)]
        need = [(x + bs - 1) // bs for x in lens_l]
        nb = sum(need) + 1024
        perm = list(range(nb))
        random.Random(43 + rank).shuffle(perm)
        rows, at = [], 0
        for c in need:
            rows.append(perm[at : at + c])
            at += c
        tables = _tables_from_lists(rows)
        lens = torch.tensor(lens_l, dtype=torch.int32)
        g = torch.Generator().manual_seed(1100 + rank)
        q, k_new, v_new = _qkv(g, n, hq, hkv, d, q_scale=30.0)
        return Workload(
            "cfg3",
            f"cfg3: KV append + paged decode attention, 128 seqs, lengths log-uniform 16..8192, head_dim 128, "
            f"{hq}q/{hkv}kv heads (GQA {gqa}), block_size 16, q x30, shuffled tables",
            hq, hkv, d, bs, nb, tables, lens, _slots_for(tables, lens, bs), q, k_new, v_new, None,
        )
    if name == "cfg5l":
        # one layer of a config-5 decode step at its saturated batch: 256
        # sequences of the Qwen2.5-0.5B shape, prompts U[64, 1024] plus up to
        # 128 generated tokens
        n, hq, hkv, d, bs = 256, 14, 2, 64, 16
        rng = np.random.default_rng(3500 + rank)
        lens_l = [int(x) for x in rng.integers(64, 1025, n) + rng.integers(1, 129, n)]
        need = [(x + bs - 1) // bs for x in lens_l]
        nb = sum(need) + 64
        perm = list(range(nb))
        random.Random(47 + rank).shuffle(perm)
        rows, at = [], 0
        for c in need:
            rows.append(perm[at : at + c])
            at += c
        tables = _tables_from_lists(rows)
        lens = torch.tensor(lens_l, dtype=torch.int32)
        g = torch.Generator().manual_seed(1400 + rank)
        q, k_new, v_new = _qkv(g, n, hq, hkv, d)
        return Workload(
            "cfg5l",
            "cfg5l: one layer of a config-5 decode step at batch 256 (14q/2kv, head_dim 64, block_size 16, "
            "lengths = prompt U[64,1024] + U[1,128] generated), KV append + decode attention",
            hq, hkv, d, bs, nb, tables, lens, _slots_for(tables, lens, bs), q, k_new, v_new, None,
        )
    if name == "d256":
        # beyond the BASELINE configs: the head_dim-256 mode (Gemma-2-9B-like
        # 8 query / 4 kv heads per shard), 64 sequences x 2048 tokens
        n, hq, hkv, d, bs, ctx = 64, 8, 4, 256, 16, 2048
        nb = n * ctx // bs + 64
        perm = list(range(nb))
        random.Random(46 + rank).shuffle(perm)
        tables = torch.tensor(perm[: n * ctx // bs], dtype=torch.int32).view(n, ctx // bs)
        lens = torch.full((n,), ctx, dtype=torch.int32)
        g = torch.Generator().manual_seed(1300 + rank)
        q, k_new, v_new = _qkv(g, n, hq, hkv, d)
        return Workload(
            "d256",
            "d256: KV append + paged decode attention, 64 seqs x 2048 ctx, 8q/4kv heads, head_dim 256, "
            "block_size 16, fp16, shuffled tables",
            hq, hkv, d, bs, nb, tables, lens, _slots_for(tables, lens, bs), q, k_new, v_new, None,
        )
    if name in ("cfg4", "cfg4-cow"):
        # 8 groups x 64 sequences; a group's tables share one 1024-token prefix
        # (64 identical block ids), then 256 tokens of the sequence's own (16
        # private blocks); the step appends the 1280th token. cfg4-cow: the
        # last of those blocks (15 of 16 rows filled) starts the step shared by
        # the group's 64 sequences, and each sequence copies it to its private
        # block (over all layers) before its append.
        groups, per_group, hq, hkv, d, bs = 8, 64, 14, 2, 64, 16
        n = groups * per_group
        prefix_blocks, own = 1024 // bs, 256 // bs
        cow = name == "cfg4-cow"
        nb = groups * (prefix_blocks + (1 if cow else 0)) + n * own + 64
        perm = list(range(nb))
        random.Random(44 + rank).shuffle(perm)
        at = 0
        prefixes, forks = [], []
        for _ in range(groups):
            prefixes.append(perm[at : at + prefix_blocks])
            at += prefix_blocks
            if cow:
                forks.append(perm[at])
                at += 1
        rows, pairs = [], []
        for s in range(n):
            gi = s // per_group
            mine = perm[at : at + own]
            at += own
            rows.append(prefixes[gi] + mine)
            if cow:
                pairs.append((forks[gi], mine[-1]))
        tables = _tables_from_lists(rows)
        lens = torch.full((n,), 1024 + 256, dtype=torch.int32)
        g = torch.Generator().manual_seed(1200 + rank)
        q, k_new, v_new = _qkv(g, n, hq, hkv, d)
        desc = (
            "cfg4-cow: 8 groups x 64 seqs sharing a 1024-token prefix (identical block ids) + 256 own tokens, "
            "ctx 1280; each sequence's last block (15 rows) starts the step shared by its group (ref count 64) "
            "and is copied to a private block over all layers (512 pairs) before the KV append + decode attention"
            if cow
            else "cfg4: KV append + decode attention; 8 groups x 64 seqs sharing a 1024-token prefix "
            "(identical block ids) + 256 own tokens, ctx 1280"
        ) + ", 14q/2kv heads, head_dim 64, block_size 16, fp16"
        return Workload(
            name, desc, hq, hkv, d, bs, nb, tables, lens, _slots_for(tables, lens, bs), q, k_new, v_new,
            torch.tensor(pairs, dtype=torch.int64) if cow else None,
        )
    raise SystemExit(f"unknown workload {name}")


# ---- clocks -------------------------------------------------------------------
_REASON_BITS = {
    "hw_slowdown": 0x8,
    "hw_thermal_slowdown": 0x40,
    "sw_thermal_slowdown": 0x20,
    "sw_power_cap": 0x4,
}


class ClockSampler:
    """SM clock, power and throttle-reason samples taken WHILE the timed
    region runs: a thread of this process polls NVML every ``interval_s``
    (the GPUs found by UUID, so the indices agree whatever
    CUDA_VISIBLE_DEVICES maps); without NVML, ``nvidia-smi -lms`` instead."""

    QUERY = (
        "timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, devices: list[int], interval_s: float = 0.002):
        self.devices = devices
        self.interval = interval_s
        self.samples: list[tuple[float, float, int]] = []  # (sm MHz, power W, reason bits)
        self.smax: list[float] = []
        self.thread = None
        self.proc = None
        self.source = "none"

    def start(self):
        import threading

        try:
            import pynvml

            pynvml.nvmlInit()
            handles = []
            for d in self.devices:
                uuid = str(torch.cuda.get_device_properties(d).uuid)
                uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
                handles.append(pynvml.nvmlDeviceGetHandleByUUID(uuid))
            self.smax = [float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)) for h in handles]
            self._stop = threading.Event()

            def loop():
                while not self._stop.is_set():
                    for h in handles:
                        try:
                            sm = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                            pw = pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
                            rs = int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(h))
                        except pynvml.NVMLError:
                            continue
                        self.samples.append((sm, pw, rs))
                    self._stop.wait(self.interval)

            self.thread = threading.Thread(target=loop, daemon=True)
            self.thread.start()
            self.source = f"NVML in-process, every {self.interval * 1e3:g} ms"
        except Exception:  # noqa: BLE001 - any NVML failure falls back to nvidia-smi
            self.thread = None
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "50"],
                    stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
                )
                self.source = "nvidia-smi -lms 50"
            except (OSError, ValueError):
                self.proc = None
            time.sleep(0.3)

    def stop(self) -> dict:
        if self.thread is not None:
            self._stop.set()
            self.thread.join(timeout=5)
            sm = [x[0] for x in self.samples]
            reasons = sorted({name for _, _, bits in self.samples for name, b in _REASON_BITS.items() if bits & b})
            return {
                "sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(self.smax) if self.smax else None,
                "reasons": reasons,
                "samples": len(self.samples),
                "power_w_max": round(max(x[1] for x in self.samples), 1) if self.samples else None,
                "source": self.source,
            }
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no NVML and no nvidia-smi"], "samples": 0}
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
            "source": self.source,
        }


# ---- reference arm / CPU baseline ---------------------------------------------
def _cpu_sample(wl: Workload, num_seqs: int):
    """A bounded sample of the workload for the CPU reference: its first
    ``num_seqs`` sequences with their pool blocks gathered into a compact fp32
    pool (shared blocks stay shared)."""
    n = min(num_seqs, wl.num_seqs)
    blocks = []
    rows = []
    index = {}
    for s in range(n):
        nb = (int(wl.lens[s]) + wl.block_size - 1) // wl.block_size
        row = []
        for b in wl.tables[s, :nb].tolist():
            if b not in index:
                index[b] = len(blocks)
                blocks.append(b)
            row.append(index[b])
        rows.append(row)
    pairs = None
    if wl.pairs is not None:
        pl = []
        for src, dst in wl.pairs[:n].tolist():
            for b in (src, dst):
                if b not in index:
                    index[b] = len(blocks)
                    blocks.append(b)
            pl.append((index[src], index[dst]))
        pairs = np.asarray(pl, dtype=np.int64)
    g = torch.Generator().manual_seed(7)
    shape = (len(blocks), wl.block_size, wl.num_kv_heads, wl.head_dim)
    k = torch.randn(shape, generator=g).half().float()
    v = torch.randn(shape, generator=g).half().float()
    lens = [int(x) for x in wl.lens[:n]]
    slots = np.asarray(
        [rows[s][(lens[s] - 1) // wl.block_size] * wl.block_size + (lens[s] - 1) % wl.block_size for s in range(n)],
        dtype=np.int64,
    )
    sample_bytes = (
        sum(lens) * wl.row_bytes * 2 + n * wl.num_q_heads * wl.head_dim * ELEM * 2 + n * wl.tables.shape[1] * 4 + n * 4
        + n * wl.row_bytes * 2 * 2 + n * 8
        + (0 if pairs is None else len(pairs) * (wl.block_size * wl.row_bytes * 2 * 2 + 16))
    )
    return dict(rows=rows, lens=lens, slots=slots, pairs=pairs, k=k, v=v, q=wl.q[:n].float(),
                k_new=wl.k_new[:n].float().numpy(), v_new=wl.v_new[:n].float().numpy(), n=n,
                bytes=sample_bytes, scale=1.0 / math.sqrt(wl.head_dim))


def cpu_reference_step(sm: dict) -> None:
    from oracle import paged_ref

    kc, vc = sm["k"].numpy(), sm["v"].numpy()
    if sm["pairs"] is not None:
        paged_ref.copy_blocks_ref([kc], [vc], sm["pairs"])
    paged_ref.kv_append_ref(kc, vc, sm["k_new"], sm["v_new"], sm["slots"])
    paged_ref.paged_attention_ref(sm["q"], sm["k"], sm["v"], sm["rows"], sm["lens"], sm["scale"])


def _time_cpu_calls(sm: dict, min_seconds: float) -> tuple[float, int, float]:
    cpu_reference_step(sm)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        cpu_reference_step(sm)
        n += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    return el / n, n, el


def time_cpu_reference(wl: Workload, num_seqs: int, min_seconds: float) -> dict:
    """The oracle on all host threads (the reported value) and on one thread
    (``value_1thread``), each for about ``min_seconds`` (half of it for the
    single thread)."""
    sm = _cpu_sample(wl, num_seqs)
    all_threads = os.cpu_count() or 1
    torch.set_num_threads(all_threads)
    per, n, el = _time_cpu_calls(sm, min_seconds)
    torch.set_num_threads(1)
    per1, n1, el1 = _time_cpu_calls(sm, min_seconds / 2)
    torch.set_num_threads(all_threads)
    return {
        "value": round(sm["bytes"] / per / 1e9, 3),
        "unit": "GB/s",
        "cores": all_threads,
        "kind": "port",
        "value_1thread": round(sm["bytes"] / per1 / 1e9, 3),
        "ms_per_call": round(per * 1e3, 3),
        "ms_per_call_1thread": round(per1 * 1e3, 3),
        "sample": (
            f"first {sm['n']} of the {wl.num_seqs} sequences of {wl.name}, fp32 torch restatement of the "
            f"reference's naive_reference_paged_attention + append"
            f"{' + copy-on-write' if sm['pairs'] is not None else ''}: {n} calls over {el:.1f} s on "
            f"{all_threads} threads, {n1} calls over {el1:.1f} s on 1 thread (os.cpu_count()={os.cpu_count()}, "
            f"torch.get_num_threads()={torch.get_num_threads()})"
        ),
    }


def time_cpu_model_step(min_seconds: float, source: torch.nn.Module | None = None, batch: int = 8,
                        ctx: int = 512) -> dict:
    """Config 5 on the host cores, bounded: one decode step of a batch of
    ``batch`` sequences at context ``ctx`` through the same random-init
    Qwen2.5-0.5B-architecture model in fp32 on CPU (the weights of ``source``
    when given), with the oracle's RoPE, append and paged attention in place of
    the kernels (the reference runner's CPU path). The whole trace is not
    feasible on CPU."""
    from oracle import paged_ref
    from pagedkv.decode_runner import random_qwen2

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    if source is None:
        model = random_qwen2(dtype=torch.float32, device="cpu", seed=0)
    else:
        # same weights without a second random init: an empty fp32 copy on the
        # host filled from the source's state dict; the rotary table is not in
        # the state dict and is rebuilt
        model = random_qwen2(dtype=torch.float32, device="meta", seed=0).to_empty(device="cpu")
        model.load_state_dict({k: v.detach().float().cpu() for k, v in source.state_dict().items()})
        model.model.rotary_emb = type(model.model.rotary_emb)(config=model.config)
        model.eval()
    m = model.model
    hq, hkv, d, bs = 14, 2, 64, 16
    per_seq = (ctx + 1 + bs - 1) // bs
    g = torch.Generator().manual_seed(5)
    layers = len(m.layers)
    kc = [torch.randn(batch * per_seq, bs, hkv, d, generator=g) for _ in range(layers)]
    vc = [torch.randn(batch * per_seq, bs, hkv, d, generator=g) for _ in range(layers)]
    tables = [list(range(s * per_seq, (s + 1) * per_seq)) for s in range(batch)]
    lens = [ctx + 1] * batch
    slots = paged_ref.decode_slots(tables, lens, bs)
    ids = torch.randint(0, model.config.vocab_size, (batch,), generator=g)
    pos = torch.full((batch,), ctx, dtype=torch.int64)

    @torch.inference_mode()
    def step():
        x = m.embed_tokens(ids[:, None])
        cos, sin = m.rotary_emb(x, pos[:, None])
        c2, s2 = cos[:, 0], sin[:, 0]
        for li, layer in enumerate(m.layers):
            attn = layer.self_attn
            h = layer.input_layernorm(x)
            q = paged_ref.rope_ref(attn.q_proj(h).view(batch, hq, d), c2, s2)
            k = paged_ref.rope_ref(attn.k_proj(h).view(batch, hkv, d), c2, s2)
            v = attn.v_proj(h).view(batch, hkv, d)
            paged_ref.kv_append_ref(kc[li].numpy(), vc[li].numpy(), k.numpy(), v.numpy(), slots)
            o = paged_ref.paged_attention_ref(q, kc[li], vc[li], tables, lens, attn.scaling)
            x = x + attn.o_proj(o.reshape(batch, 1, -1))
            x = x + layer.mlp(layer.post_attention_layernorm(x))
        return model.lm_head(m.norm(x)[:, 0]).argmax(-1)

    step()  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        step()
        n += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    per = el / n
    return {
        "value": round(batch / per, 2),
        "unit": "decode tok/s",
        "cores": threads,
        "kind": "port",
        "ms_per_step": round(per * 1e3, 2),
        "sample": (
            f"{n} decode steps over {el:.1f} s of a batch of {batch} at context {ctx} through the random-init "
            f"model in fp32 on CPU with the oracle's RoPE, append and paged attention ({threads} threads); "
            "the full trace is not feasible on CPU"
        ),
    }


def run_reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    wl = make_workload(args.workload, 0, args.gqa)
    sm = _cpu_sample(wl, 8)
    # a step runs the sample once per layer, as our arm's step runs every layer
    layers = args.layers if args.workload != "cfg5" else 1
    for _ in range(args.warmup):
        cpu_reference_step(sm)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        for _ in range(layers):
            cpu_reference_step(sm)
        times.append(time.perf_counter() - t0)
    per = sum(times) / len(times)
    value = layers * sm["bytes"] / per / 1e9
    threads = torch.get_num_threads()
    line = {
        "impl": "reference",
        "metric": METRIC,
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
        "config": {"workload": wl.description, "layers_per_step": layers, "sample_seqs_per_step": sm["n"],
                   "parallelism": "host cores of rank 0"},
        "cpu_baseline": {
            "value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"first {sm['n']} sequences of {wl.name}, {layers} layer passes per step (fp32 oracle "
                      "restatement, torch CPU)",
        },
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---- our arm ------------------------------------------------------------------
def _dist_setup(args):
    """One process per GPU. The ranks share nothing on the data path; a gloo
    (host) group carries only the barrier around each timed region and the
    max / sum of the per-rank timings, so NCCL is not used at all."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and world > 1:
        raise SystemExit(f"--gpus {args.gpus} disagrees with WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("gloo", timeout=timedelta(seconds=180))
    return dist, rank, world, local


def _max_over_ranks(dist, value: float, device=None) -> float:
    if dist is None:
        return value
    t = torch.tensor([value], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _sum_over_ranks(dist, value: float, device=None) -> float:
    if dist is None:
        return value
    t = torch.tensor([value], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def _read_traffic(kernel: str, workload: str, rope: bool = False) -> int | None:
    """ncu DRAM bytes per launch of ``kernel`` on ``workload`` from
    profiles/traffic.json (keys "kernel" for config 2, "kernel:workload" for
    the others; the RoPE instantiation under "kernel:rope" for config 2 and
    "kernel:workload_rope" for the others), or None where no capture exists."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        data = json.loads(p.read_text())
        if rope:
            key = f"{kernel}:rope" if workload == "cfg2" else f"{kernel}:{workload}_rope"
        else:
            key = kernel if workload == "cfg2" else f"{kernel}:{workload}"
        entry = data.get(key)
        return int(entry["bytes_per_launch"]) if entry else None
    except (ValueError, KeyError, TypeError):
        return None


def run_ours(args) -> None:
    import pagedkv
    from pagedkv import _native
    from oracle import paged_ref  # checker only, outside the timed region

    dist, rank, world, local = _dist_setup(args)
    dev = torch.device("cuda", local)
    _native.lib()
    wl = make_workload(args.workload, rank, args.gqa)
    L = args.layers
    # One pool per layer, as the model's PhysicalBlockPool holds them: a step
    # runs the paged path of every layer, and no layer's K/V is in L2 when
    # the next layer's kernels read theirs.
    kcs, vcs = [], []
    for layer in range(L):
        pl = make_pools(rank * 1000 + layer, dev, wl.num_blocks, wl.block_size, wl.num_kv_heads, wl.head_dim)
        kcs.append(pl["k_cache"])
        vcs.append(pl["v_cache"])
    # per-layer step inputs: distinct buffers holding the same seeded values
    qs = [wl.q.to(dev) for _ in range(L)]
    # --rope: the step rotates q and k as the model's decode forward does
    # (cos / sin rows of each sequence's position, fused into the launch)
    if args.rope:
        inv = 1.0 / (1000000.0 ** (torch.arange(0, wl.head_dim, 2, dtype=torch.float32) / wl.head_dim))
        ang = (wl.lens.to(torch.float32) - 1)[:, None] * inv[None]
        emb = torch.cat([ang, ang], dim=-1)
        cos_t, sin_t = emb.cos().half().to(dev), emb.sin().half().to(dev)
    else:
        cos_t = sin_t = None
    kns = [wl.k_new.to(dev) for _ in range(L)]
    vns = [wl.v_new.to(dev) for _ in range(L)]
    tables = wl.tables.to(dev)
    lens = wl.lens.to(dev)
    slots = wl.slots.to(dev)
    pairs = wl.pairs.to(dev) if wl.pairs is not None else None
    scale = 1.0 / math.sqrt(wl.head_dim)
    stream = torch.cuda.current_stream(dev)
    outs: list = [None] * L

    def fused_layers():
        # per layer ONE launch: the KV append of the step's token fused into
        # the decode attention (pagedkv.paged_attention_decode_append)
        for layer in range(L):
            outs[layer] = pagedkv.paged_attention_decode_append(qs[layer], kcs[layer], vcs[layer], tables, lens,
                                                                scale, kns[layer], vns[layer], cos_t, sin_t,
                                                                slot_mapping=slots)

    def step():
        if pairs is not None:
            pagedkv.copy_blocks(kcs, vcs, pairs)  # copy-on-write: one launch for every layer
        fused_layers()

    def attention_only():
        for layer in range(L):
            pagedkv.paged_attention_decode_batched(qs[layer], kcs[layer], vcs[layer], tables, lens, scale)

    # correctness spot-check of this shard against the oracle (first and last
    # sequence of the first and last layer; with --rope on the rotated q)
    step()
    if args.rope:
        qs_chk = [paged_ref.rope_ref(qs[layer].cpu(), cos_t.cpu(), sin_t.cpu()) for layer in range(L)]
    else:
        qs_chk = qs
    torch.cuda.synchronize(dev)
    sel = [0, wl.num_seqs - 1]
    nbk = [(int(wl.lens[s_]) + wl.block_size - 1) // wl.block_size for s_ in sel]
    used = sorted({int(b) for s_, n in zip(sel, nbk) for b in wl.tables[s_, :n].tolist()})
    remap = {b: i for i, b in enumerate(used)}
    idx = torch.tensor(used, device=dev)
    max_err = 0.0
    for layer in sorted({0, L - 1}):
        ref = paged_ref.paged_attention_ref(
            qs_chk[layer][sel].float().cpu(), kcs[layer][idx].float().cpu(), vcs[layer][idx].float().cpu(),
            [[remap[int(b)] for b in wl.tables[s_, :n].tolist()] for s_, n in zip(sel, nbk)],
            [int(wl.lens[s_]) for s_ in sel], scale,
        )
        err = (outs[layer][sel].float().cpu() - ref).abs().max().item()
        if not err < 2e-3 + 2e-3 * ref.abs().max().item():
            raise SystemExit(f"bench spot-check failed on layer {layer}: max |err| {err}")
        max_err = max(max_err, err)
    launches_attn, family = pagedkv.last_decode_launch_info()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)

    # The decode step and its attention launches alone, each captured once as
    # a CUDA graph and replayed: a serving engine replays the decode step the
    # same way, so the device time is not bounded by Python.
    g_step = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_step):
        step()
    g_attn = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_attn):
        attention_only()
    g_fused = None
    if pairs is not None:  # the fused launches without the copy-on-write copy
        g_fused = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_fused):
            fused_layers()
    for _ in range(args.warmup):
        g_step.replay()
        g_attn.replay()
        if g_fused is not None:
            g_fused.replay()
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

    sampler = ClockSampler(list(range(world)) if world > 1 else [local]) if rank == 0 else None
    if sampler:
        sampler.start()
    total_ms = timed(g_step.replay, args.steps)
    clocks = sampler.stop() if sampler else None
    attn_ms = timed(g_attn.replay, args.steps) / args.steps  # L launches per replay
    fused_ms = timed(g_fused.replay, args.steps) / args.steps if g_fused is not None else None
    eager_n = max(3, args.steps // 4)
    eager_ms = timed(step, eager_n) / eager_n
    total_ms = _max_over_ranks(dist, total_ms)
    attn_ms_max = _max_over_ranks(dist, attn_ms)
    eager_ms = _max_over_ranks(dist, eager_ms)
    ms_per_step = total_ms / args.steps
    fused_ms = ms_per_step if fused_ms is None else fused_ms  # without a copy the step IS the fused launches
    other_ms = max(0.0, ms_per_step - attn_ms_max)

    a_bytes = wl.attention_bytes()
    step_bytes = wl.step_bytes(L)
    value = world * step_bytes / (ms_per_step * 1e-3) / 1e9

    # ---- end to end through the public API from pinned host buffers -------------
    # Every step copies its inputs host->device (the block tables, lengths and
    # slots once; each layer's q and new K/V rows) and reads every layer's
    # attention output back device->host.
    parts = [wl.slots, wl.tables, wl.lens] + [t for _ in range(L) for t in (wl.q, wl.k_new, wl.v_new)]
    sizes = [t.numel() * t.element_size() for t in parts]
    offs = [0]
    for sz in sizes:
        offs.append(offs[-1] + (sz + 255) // 256 * 256)
    h_in = torch.empty(offs[-1], dtype=torch.uint8).pin_memory()
    for t, o, sz in zip(parts, offs, sizes):
        h_in[o : o + sz].copy_(t.contiguous().view(-1).view(torch.uint8))
    out_elems = wl.q.numel()
    h2d = sum(sizes)
    d2h = L * out_elems * ELEM

    def make_views(buf):
        return [buf[o : o + sz].view(t.dtype).view(t.shape) for t, o, sz in zip(parts, offs, sizes)]

    def run_layers(views, out_buf):
        ds, dt, dl = views[:3]
        if pairs is not None:
            pagedkv.copy_blocks(kcs, vcs, pairs)
        for layer in range(L):
            dq, dk, dv = views[3 + 3 * layer : 6 + 3 * layer]
            pagedkv.paged_attention_decode_append(dq, kcs[layer], vcs[layer], dt, dl, scale, dk, dv, cos_t,
                                                  sin_t, slot_mapping=ds, out=out_buf[layer])

    d_in = torch.empty(offs[-1], dtype=torch.uint8, device=dev)
    views = make_views(d_in)
    d_out = torch.empty((L,) + tuple(wl.q.shape), dtype=torch.float16, device=dev)
    h_out = torch.empty((L,) + tuple(wl.q.shape), dtype=torch.float16).pin_memory()

    def e2e_step():
        d_in.copy_(h_in, non_blocking=True)
        run_layers(views, d_out)
        h_out.copy_(d_out, non_blocking=True)

    for _ in range(max(3, args.warmup)):
        e2e_step()
    torch.cuda.synchronize(dev)
    serial_ms = _max_over_ranks(dist, timed(e2e_step, args.steps)) / args.steps
    serial_out = h_out.clone()

    # Pipelined: the same calls and copies, with step i+1's inputs copied on a
    # side stream into the other of two device buffers before step i's
    # kernels are issued, and step i's outputs read back on a second side
    # stream (the copy engines run beside the SMs). Every step still moves all
    # of its inputs host->device and its outputs device->host inside the
    # timed region.
    d_in2 = [d_in, torch.empty_like(d_in)]
    views2 = [views, make_views(d_in2[1])]
    d_out2 = [d_out, torch.empty_like(d_out)]
    h_out2 = [h_out, torch.empty_like(h_out).pin_memory()]
    s_h2d, s_d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    free = [torch.cuda.Event(), torch.cuda.Event()]
    ready = [torch.cuda.Event(), torch.cuda.Event()]
    done = [torch.cuda.Event(), torch.cuda.Event()]
    out_free = [torch.cuda.Event(), torch.cuda.Event()]

    def stage_inputs(i):
        free[i].wait(s_h2d)  # the step that last read this buffer is done
        torch.cuda.set_stream(s_h2d)
        d_in2[i].copy_(h_in, non_blocking=True)
        torch.cuda.set_stream(stream)
        ready[i].record(s_h2d)

    def e2e_pipelined_step(i, prefetch):
        # A serving loop consumes each result: the host waits for the read-back
        # of step i-2 before issuing step i, so it runs at most two steps ahead.
        b = i % 2
        if i >= 2:
            done[b].synchronize()
        if prefetch:
            stage_inputs((i + 1) % 2)
        ready[b].wait(stream)
        out_free[b].wait(stream)
        run_layers(views2[b], d_out2[b])
        free[b].record(stream)
        free[b].wait(s_d2h)
        torch.cuda.set_stream(s_d2h)
        h_out2[b].copy_(d_out2[b], non_blocking=True)
        torch.cuda.set_stream(stream)
        done[b].record(s_d2h)
        out_free[b].record(s_d2h)

    def e2e_pipelined(n):
        # the side streams start after the region's opening event and the
        # launch stream waits for both before its closing event
        s_h2d.wait_stream(stream)
        s_d2h.wait_stream(stream)
        stage_inputs(0)
        for i in range(n):
            e2e_pipelined_step(i, i + 1 < n)
        stream.wait_stream(s_h2d)
        stream.wait_stream(s_d2h)

    e2e_pipelined(max(3, args.warmup))
    torch.cuda.synchronize(dev)
    e2e_ms = _max_over_ranks(dist, timed(lambda: e2e_pipelined(args.steps), 1)) / args.steps
    pipe_match = bool(torch.equal(h_out2[(args.steps - 1) % 2], serial_out))
    e2e_value = world * step_bytes / (e2e_ms * 1e-3) / 1e9

    # release this workload's pools before the model-level run
    del kcs, vcs, g_step, g_attn, g_fused, d_in, d_in2, views, views2, d_out, d_out2, outs
    torch.cuda.empty_cache()

    model_block = None
    if args.model_requests > 0 and args.workload == "cfg2":
        model_block = model_decode_trace(args, dist, rank, world, dev, args.model_requests, args.model_rate,
                                         args.model_kv_gb, with_cpu=False)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = time_cpu_reference(wl, 16, args.cpu_seconds)

    peaks = {}
    pp = ROOT / "MEASURED_PEAKS.json"
    if pp.exists():
        peaks = json.loads(pp.read_text())
    peak = float(peaks.get("hbm_gbs", 6650.0))
    measured_peak = "hbm_gbs" in peaks
    # The dominant kernel is the fused decode launch as the step runs it: its
    # bytes are the attention's plus the append's (new rows read, pool rows
    # written).
    per_launch_ms = fused_ms / L
    shared_prefix = wl.name.startswith("cfg4")
    append_b = wl.append_bytes() - wl.num_seqs * 8  # no slot list is read
    roof_bytes = (wl.attention_unique_bytes() if shared_prefix else a_bytes) + append_b
    achieved = roof_bytes / (per_launch_ms * 1e-3) / 1e9
    kernel_name = f"decode_{family}"
    traffic = _read_traffic(kernel_name, wl.name, args.rope)
    launches_per_step = L * launches_attn + (1 if pairs is not None else 0)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    roofline = {
        "bound": "hbm",
        "kernel": kernel_name + " with the KV append fused in",
        "achieved": round(achieved, 1),
        "peak": peak,
        "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if measured_peak else "fallback 6650 GB/s",
        "unit": "GB/s",
        "frac": round(achieved / peak, 4),
        "traffic": traffic,
        "algorithmic_bytes_per_launch": roof_bytes,
        "launch_us": round(per_launch_ms * 1e3, 3),
        "launches_timed": L * args.steps,
        "flops_per_launch": wl.flops(),
    }
    if shared_prefix:
        roofline["bytes_basis"] = "unique: each distinct K/V block once (a shared prefix is read once from HBM)"
        roofline["logical_bytes_per_launch"] = a_bytes + append_b
        roofline["achieved_logical"] = round((a_bytes + append_b) / (per_launch_ms * 1e-3) / 1e9, 1)
    line = {
        "metric": METRIC,
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
            "workload": wl.description,
            "layers_per_step": L,
            "step": f"one decode step of the paged path over {L} layers (one pool per layer): "
                    + ("the copy-on-write copy over all layers, then " if pairs is not None else "")
                    + ("per layer the RoPE of q and k, " if args.rope else "per layer ")
                    + "the KV append and the decode attention, fused into one launch",
            "num_seqs_per_gpu": wl.num_seqs,
            "total_context_tokens_per_gpu": int(wl.lens.to(torch.int64).sum()),
            "heads": f"{wl.num_q_heads}q/{wl.num_kv_heads}kv",
            "head_dim": wl.head_dim,
            "block_size": wl.block_size,
            "num_blocks": wl.num_blocks,
            "decode_kernel": family,
            "l2": f"inputs exceed L2: each layer reads {a_bytes / 1e6:.1f} MB of its own pool, a step "
                  f"{L * a_bytes / 1e9:.2f} GB, vs {L2_BYTES / 2**20:.0f} MiB L2; no flush",
            "parallelism": f"dp{world}: sequences sharded, one pool per GPU, no collective on the data path",
            "bytes_per_step": step_bytes,
            "unique_kv_bytes_per_layer": wl.unique_kv_bytes(),
        },
        "paged_path_tokens_per_s": round(world * wl.num_seqs / (ms_per_step * 1e-3), 1),
        "fused_us_per_layer": round(per_launch_ms * 1e3, 3),
        "attention_only_us_per_layer": round(attn_ms_max / L * 1e3, 3),
        "other_us_per_layer": round(other_ms / L * 1e3, 3),
        "timing": f"CUDA-graph replay of the {L}-layer step, CUDA events on the launch stream; the attention "
                  f"without the append from a graph of its {L} launches, for comparison",
        "eager_ms_per_step": round(eager_ms, 5),
        "roofline": roofline,
        "cpu_baseline": cpu,
        "e2e": {
            "value": round(e2e_value, 2),
            "unit": "GB/s",
            "ms_per_step": round(e2e_ms, 5),
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "api": "pagedkv public API; each step's inputs staged in one pinned buffer (one H2D copy) and the "
                   "outputs of all layers read back with one D2H copy",
            "overlap": "step i+1's H2D (issued before step i's kernels) and step i's D2H run on side streams "
                       "(double-buffered) while the SMs compute; the host waits for step i-2's read-back before "
                       "issuing step i",
            "serial_ms_per_step": round(serial_ms, 5),
            "serial_value": round(world * step_bytes / (serial_ms * 1e-3) / 1e9, 2),
            "pipelined_output_matches_serial": pipe_match,
        },
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
        "spot_check_max_abs_err": max_err,
    }
    if model_block is not None:
        line["model_decode"] = model_block
    print(json.dumps(line), flush=True)


# ---- config 5: full-model decode under continuous batching ------------------
def model_decode_trace(args, dist, rank: int, world: int, dev, requests: int, rate: float, kv_gb: float,
                       with_cpu: bool) -> dict:
    """Config 5 on this rank: a random-init Qwen2.5-0.5B-architecture model
    (24 layers, 896 hidden, 14/2 heads, MLP 4864, vocab 151936, fp16) served by
    the continuous-batching decode runner over a seeded Poisson trace
    (``requests`` per GPU at ``rate`` req/s per GPU, prompts U[64, 1024]
    random ids, 128 output tokens, greedy), the requests of the global trace
    routed to the GPUs by least outstanding tokens. Returns the figures of the
    whole job (decode tokens/s over all GPUs, max elapsed over ranks) and, per
    decode step, the split between graph-replay device time and host time."""
    import numpy as np
    from pagedkv.decode_runner import PagedDecodeRunner, random_qwen2

    model = random_qwen2(device=dev, seed=0)
    block_size = 16
    block_bytes = 2 * model.config.num_hidden_layers * block_size * model.config.num_key_value_heads * 64 * 2
    num_blocks = min(int(kv_gb * 1e9) // block_bytes, (2**31 - 1) // block_size)
    runner = PagedDecodeRunner(model, num_blocks=num_blocks, block_size=block_size, max_batch=256,
                               max_seq_len=1024 + 128)
    # One global trace (world x requests at world x rate), routed by
    # least-outstanding-tokens (pagedkv.router.route_trace): every rank computes
    # the same assignment and serves its share; nothing is exchanged.
    from pagedkv.router import route_trace

    rng = np.random.default_rng(5000)
    n_all = requests * world
    arr_all = np.cumsum(rng.exponential(1.0 / (rate * world), n_all))
    lens_all = rng.integers(64, 1025, n_all)
    out_tokens = 128
    mine = [i for i, r_ in enumerate(route_trace([int(L) + out_tokens for L in lens_all], world)) if r_ == rank]
    n_req = len(mine)
    arrivals = arr_all[mine]
    prompt_lens = lens_all[mine]
    vocab = model.config.vocab_size
    prng = np.random.default_rng(6000 + rank)
    prompts = [prng.integers(0, vocab, int(L)).tolist() for L in prompt_lens]

    # warm-up: graphs for every bucket and one prefill, outside the timed trace
    runner.warm_prefill(1024, batches=(2, 4, 8))
    warm = [runner.prefill(prompts[i % n_req][:64], 2) for i in range(2)]
    for b in (1, 2, 4, 8, 16, 32, 64, 128, 256):
        runner._graph_for(b)
    runner.decode_step(warm)
    for s_ in warm:
        runner.release(s_)
    torch.cuda.synchronize(dev)
    if dist:
        dist.barrier()

    runner.timing = []  # (start event, end event) around every decode replay
    waiting = list(range(n_req))
    running = []
    ttft, finish, decode_time, decode_steps, prefill_time = [], [], 0.0, 0, 0.0
    t0 = time.perf_counter()
    while waiting or running:
        now = time.perf_counter() - t0
        # admit the arrived requests that fit, up to 8 per step, prefilled together
        batch, free_blocks = [], len(runner.free)
        while (waiting and arrivals[waiting[0]] <= now and len(running) + len(batch) < runner.max_batch
               and len(batch) < 8):
            i = waiting[0]
            need = (int(prompt_lens[i]) + out_tokens + runner.block_size - 1) // runner.block_size
            if need > free_blocks or need > runner.max_blocks_per_seq:
                break
            free_blocks -= need
            batch.append(waiting.pop(0))
        if batch:
            tp = time.perf_counter()
            new_seqs = runner.prefill_many([prompts[i] for i in batch], out_tokens)
            torch.cuda.synchronize(dev)
            prefill_time += time.perf_counter() - tp
            for i, seq in zip(batch, new_seqs):
                seq.arrival = arrivals[i]
                ttft.append(time.perf_counter() - t0 - arrivals[i])
                running.append(seq)
        if running:
            td = time.perf_counter()
            runner.decode_step(running)
            decode_time += time.perf_counter() - td
            decode_steps += 1
            still = []
            for s_ in running:
                if s_.done:
                    finish.append(time.perf_counter() - t0 - s_.arrival)
                    runner.release(s_)
                else:
                    still.append(s_)
            running = still
        elif waiting:
            time.sleep(max(0.0, min(0.01, arrivals[waiting[0]] - (time.perf_counter() - t0))))
    elapsed = time.perf_counter() - t0
    torch.cuda.synchronize(dev)
    replay_ms = sum(a.elapsed_time(b) for a, b in runner.timing)
    runner.timing = None
    profile = None
    if getattr(args, "profile_decode", 0) > 0 and rank == 0:
        profile = profile_decode_steps(runner, prompts, out_tokens, args.profile_decode, dev)
    gen = n_req * out_tokens
    elapsed_max = _max_over_ranks(dist, elapsed)
    gen_all = _sum_over_ranks(dist, float(gen))
    dec_tok = n_req * (out_tokens - 1)  # the first token of each request comes from its prefill
    cpu = None
    if with_cpu and rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = time_cpu_model_step(args.cpu_seconds, source=model)
    del runner, model
    torch.cuda.empty_cache()
    mean_step = 1e3 * decode_time / max(1, decode_steps)
    mean_dev = replay_ms / max(1, decode_steps)
    return {
        "metric": "decode tokens/s",
        "value": round(gen_all / elapsed_max, 1),
        "unit": "tok/s",
        "n_gpus": world,
        "higher_is_better": True,
        "scaling": "weak",
        "config": {
            "workload": "cfg5: random-init Qwen2.5-0.5B architecture (24 layers, hidden 896, 14q/2kv, head_dim 64, "
                        "MLP 4864, vocab 151936, tied embeddings, fp16), continuous batching over a seeded Poisson "
                        f"trace of {n_all} requests at {rate * world:g} req/s ({rate:g} per GPU), "
                        f"prompts U[64,1024] random ids, {out_tokens} output tokens, greedy",
            "kv_budget_gb": kv_gb,
            "num_blocks": num_blocks,
            "requests_this_rank": n_req,
            "parallelism": f"dp{world}: one runner and pool per GPU; requests routed by least outstanding tokens "
                           "(the same deterministic assignment computed on every rank, no exchange)",
        },
        "elapsed_s": round(elapsed_max, 3),
        "generated_tokens": int(gen_all),
        "decode_only_tokens_per_s": round(dec_tok / decode_time, 1) if decode_time > 0 else None,
        "decode_steps": decode_steps,
        "mean_decode_step_ms": round(mean_step, 3),
        "mean_decode_replay_device_ms": round(mean_dev, 3),
        "mean_decode_host_ms": round(max(0.0, mean_step - mean_dev), 3),
        "prefill_s": round(prefill_time, 3),
        "ttft_ms_p50": round(1e3 * float(np.median(ttft)), 2),
        "request_latency_s_p50": round(float(np.median(finish)), 3),
        "timing": "wall clock of the trace replay (max over ranks); decode steps are CUDA-graph replays whose "
                  "device time comes from CUDA events around each replay",
        "cpu_baseline": cpu,
        **({"decode_step_profile": profile} if profile is not None else {}),
    }


def profile_decode_steps(runner, prompts, out_tokens: int, steps: int, dev, batch: int = 256) -> dict:
    """Per-kernel device time of ``steps`` decode steps at a full batch
    (``batch`` sequences prefilled from the trace's prompts), from the CUDA
    activity records of torch.profiler (kernel durations as they ran, inside
    the graph replays), grouped by kernel name; plus the CUDA-event time of
    the same replays and the host wall time per step."""
    from torch.profiler import ProfilerActivity, profile

    seqs = []
    i = 0
    while len(seqs) < batch:
        chunk = [prompts[(i + j) % len(prompts)] for j in range(8)]
        seqs += runner.prefill_many(chunk, out_tokens)
        i += 8
    seqs = seqs[:batch]
    runner.decode_step(seqs)  # warm
    torch.cuda.synchronize(dev)
    runner.timing = []
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        t0 = time.perf_counter()
        for _ in range(steps):
            runner.decode_step(seqs)
        torch.cuda.synchronize(dev)
        wall = time.perf_counter() - t0
    replay_ms = sum(a.elapsed_time(b) for a, b in runner.timing) / steps
    runner.timing = None
    ctx = float(np.mean([s_.num_tokens for s_ in seqs])) if seqs else 0.0
    for s_ in seqs:
        runner.release(s_)
    rows = {}
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            r = rows.setdefault(ev.name, [0, 0.0])
            r[0] += 1
            r[1] += ev.device_time_total
    total_us = sum(v[1] for v in rows.values())
    top = sorted(rows.items(), key=lambda kv: -kv[1][1])
    return {
        "batch": batch,
        "steps": steps,
        "mean_context_tokens": round(ctx, 1),
        "event_ms_per_step": round(replay_ms, 4),
        "host_wall_ms_per_step": round(1e3 * wall / steps, 4),
        "kernel_us_per_step": round(total_us / steps, 2),
        "kernels_per_step": round(sum(v[0] for v in rows.values()) / steps, 1),
        "by_kernel": [
            {"kernel": k[:120], "launches_per_step": round(v[0] / steps, 2), "us_per_step": round(v[1] / steps, 2),
             "share": round(v[1] / total_us, 4)}
            for k, v in top[:25]
        ],
    }


def run_model(args) -> None:
    """``--workload cfg5``: config 5 on its own, one JSON line."""
    dist, rank, world, local = _dist_setup(args)
    dev = torch.device("cuda", local)
    block = model_decode_trace(args, dist, rank, world, dev, args.requests, args.rate, args.kv_budget_gb,
                               with_cpu=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {k: v for k, v in block.items()}
    line["vs_baseline"] = None
    line["dtype"] = "f16"
    line["data"] = "synthetic"
    print(json.dumps(line), flush=True)


# ---- the pool-write kernels on their own -------------------------------------
def run_ops(args) -> None:
    """The four pool-write kernels (decode append, fused RoPE + append,
    copy-on-write block copy, prefill write), each timed at the size one decode
    layer-step gives it (latency-bound: microseconds) and at a bulk size whose
    traffic exceeds L2 (bandwidth-bound: GB/s against the measured HBM peak).
    CUDA-graph replay of one launch, K replays between CUDA events."""
    import pagedkv

    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        raise SystemExit("--workload ops runs on one GPU")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(7)
    stream = torch.cuda.current_stream(dev)
    pp = ROOT / "MEASURED_PEAKS.json"
    peak = float(json.loads(pp.read_text()).get("hbm_gbs", 6650.0)) if pp.exists() else 6650.0

    def rnd(*shape):
        return torch.randn(shape, generator=g, device=dev, dtype=torch.float16)

    def distinct_slots(n, num_blocks, bs):
        return torch.randperm(num_blocks * bs, generator=g, device=dev)[:n].contiguous()

    def time_graph(fn, steps):
        fn()
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        for _ in range(max(3, args.warmup)):
            graph.replay()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(steps):
            graph.replay()
        b.record(stream)
        torch.cuda.synchronize(dev)
        del graph
        return a.elapsed_time(b) / steps * 1e3  # us

    results = {}

    def record(name, us, nbytes, shape):
        gbs = nbytes / (us * 1e-6) / 1e9
        results[name] = {"us": round(us, 3), "bytes": int(nbytes), "GB/s": round(gbs, 1),
                         "frac_of_measured_hbm": round(gbs / peak, 4), "shape": shape}

    steps = min(args.steps, 500)
    # decode append (paged_attention_integration.py:150-160) at config 2 and in bulk
    for tag, n, hkv, d, nb in (("decode", 256, 2, 64, 40960), ("bulk", 65536, 8, 128, 8192)):
        kc, vc = rnd(nb, 16, hkv, d), rnd(nb, 16, hkv, d)
        kn, vn = rnd(n, hkv, d), rnd(n, hkv, d)
        sl = distinct_slots(n, nb, 16)
        us = time_graph(lambda: pagedkv.kv_append(kn, vn, kc, vc, sl), steps)
        record(f"kv_append_{tag}", us, n * hkv * d * 2 * 2 * 2 + n * 8, f"{n} tokens x {hkv}x{d}")
        del kc, vc, kn, vn
    # fused RoPE + append at the Qwen2.5-0.5B attention shape (14 q / 2 kv heads, head_dim 64)
    for tag, n, nb in (("decode", 256, 40960), ("bulk", 262144, 40960)):
        hq, hkv, d = 14, 2, 64
        kc, vc = rnd(nb, 16, hkv, d), rnd(nb, 16, hkv, d)
        q, kn, vn = rnd(n, hq, d), rnd(n, hkv, d), rnd(n, hkv, d)
        cos, sin = rnd(n, d), rnd(n, d)
        qo = torch.empty_like(q)
        sl = distinct_slots(n, nb, 16)
        us = time_graph(lambda: pagedkv.kv_append_rope(q, kn, vn, cos, sin, kc, vc, sl, q_out=qo), steps)
        nbytes = n * d * 2 * (2 * hq + 4 * hkv + 2) + n * 8
        record(f"kv_append_rope_{tag}", us, nbytes, f"{n} tokens x {hq}q/{hkv}kv x {d}")
        del kc, vc, q, kn, vn, cos, sin, qo
    # copy-on-write over 24 layers (config-4 block: 16 x 2 x 64 fp16 = 4 KiB for K and for V)
    for tag, pairs_n, nb in (("decode", 512, 1024), ("bulk", 8192, 16384)):
        layers = 24
        kcs = [rnd(nb, 16, 2, 64) for _ in range(layers)]
        vcs = [rnd(nb, 16, 2, 64) for _ in range(layers)]
        perm = torch.randperm(nb, generator=g, device=dev)
        mapping = torch.stack([perm[:pairs_n], perm[pairs_n : 2 * pairs_n]], dim=1).contiguous()
        us = time_graph(lambda: pagedkv.copy_blocks(kcs, vcs, mapping), steps)
        block = 16 * 2 * 64 * 2
        record(f"copy_blocks_{tag}", us, layers * pairs_n * block * 2 * 2 + pairs_n * 16,
               f"{pairs_n} pairs x {layers} layers x 2 x {block} B")
        del kcs, vcs
    # prefill write of one prompt into every layer's pool (fp16 sources)
    for tag, ntok in (("prompt", 1000), ("bulk", 65536)):
        layers, hkv, d, bs = 24, 2, 64, 16
        nw = (ntok + bs - 1) // bs
        nb = nw + 64
        kcs = [rnd(nb, bs, hkv, d) for _ in range(layers)]
        vcs = [rnd(nb, bs, hkv, d) for _ in range(layers)]
        ks = [rnd(ntok, hkv, d) for _ in range(layers)]
        vs = [rnd(ntok, hkv, d) for _ in range(layers)]
        ids = torch.randperm(nb, generator=g, device=dev)[:nw].contiguous()
        us = time_graph(lambda: pagedkv.kv_write_prefill(ks, vs, kcs, vcs, ids, ntok), min(steps, 200))
        nbytes = layers * 2 * (ntok * hkv * d * 2 + nw * bs * hkv * d * 2)
        record(f"kv_write_prefill_{tag}", us, nbytes, f"{ntok}-token prompt x {layers} layers, {hkv}x{d}")
        del kcs, vcs, ks, vs
    line = {
        "metric": "pool-write kernels: us per launch and GB/s",
        "workload": "ops",
        "n_gpus": 1,
        "steps": steps,
        "warmup": args.warmup,
        "peak_hbm_gbs": peak,
        "timing": "CUDA-graph replay of one launch, CUDA events on the launch stream; bulk sizes exceed L2",
        "data": "synthetic",
        "ops": results,
    }
    print(json.dumps(line), flush=True)


def run_cuda_core(args) -> None:
    """The CUDA-core decode kernel (block sizes below 8 or not a power of two)
    on five shapes at block_size 4, 2048-token contexts, pools larger than L2.
    Eager calls of the public batched entry point, K calls between CUDA
    events; algorithmic bytes = the K and V rows read."""
    import pagedkv

    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        raise SystemExit("--workload cuda-core runs on one GPU")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    pp = ROOT / "MEASURED_PEAKS.json"
    peak = float(json.loads(pp.read_text()).get("hbm_gbs", 6650.0)) if pp.exists() else 6650.0
    steps = min(args.steps, 50)
    results = {}
    for n, ctx, hkv, g, d, bs in ((128, 2048, 8, 7, 128, 4), (128, 2048, 8, 2, 128, 4), (128, 2048, 8, 1, 128, 4),
                                  (256, 2048, 2, 7, 64, 4), (64, 2048, 4, 4, 256, 4)):
        nbk = n * ctx // bs
        gen = torch.Generator(device=dev).manual_seed(0)
        k = torch.randn(nbk, bs, hkv, d, generator=gen, device=dev, dtype=torch.float16)
        v = torch.randn(nbk, bs, hkv, d, generator=gen, device=dev, dtype=torch.float16)
        q = torch.randn(n, hkv * g, d, generator=gen, device=dev, dtype=torch.float16)
        tables = torch.randperm(nbk, generator=gen, device=dev).to(torch.int32).view(n, ctx // bs)
        lens = torch.full((n,), ctx, dtype=torch.int32, device=dev)

        def call():
            return pagedkv.paged_attention_decode_batched(q, k, v, tables, lens, d ** -0.5)

        for _ in range(max(3, args.warmup)):
            call()
        if pagedkv.last_decode_launch_info()[1] != "simt":
            raise SystemExit("--workload cuda-core: the shape did not run on the CUDA-core kernel")
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            call()
        b.record()
        torch.cuda.synchronize(dev)
        us = a.elapsed_time(b) / steps * 1e3
        nbytes = n * ctx * hkv * d * 2 * 2
        gbs = nbytes / (us * 1e-6) / 1e9
        results[f"d{d}_hkv{hkv}_gqa{g}_bs{bs}"] = {
            "us": round(us, 1), "bytes": nbytes, "GB/s": round(gbs, 1),
            "frac_of_measured_hbm": round(gbs / peak, 4), "shape": f"{n} seqs x {ctx} tokens"}
        del k, v, q, tables
        torch.cuda.empty_cache()
    print(json.dumps({
        "metric": "CUDA-core decode kernel: us per call and GB/s", "workload": "cuda-core", "n_gpus": 1,
        "steps": steps, "warmup": args.warmup, "peak_hbm_gbs": peak,
        "timing": "eager calls of paged_attention_decode_batched (decode + split combine), CUDA events; "
                  "pools exceed L2", "data": "synthetic", "shapes": results}), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["cfg1", "cfg2", "cfg3", "cfg4", "cfg4-cow", "cfg5", "cfg5l", "ops", "d256",
                                           "cuda-core"],
                    default="cfg2")
    ap.add_argument("--requests", type=int, default=2000, help="cfg5: requests per GPU")
    ap.add_argument("--rate", type=float, default=32.0, help="cfg5: Poisson arrival rate per GPU (req/s)")
    ap.add_argument("--kv-budget-gb", type=float, default=60.0, help="cfg5: KV pool budget per GPU")
    ap.add_argument("--gqa", type=int, default=7, help="GQA group for --workload cfg3 (1, 2, 4 or 7)")
    ap.add_argument("--rope", action="store_true",
                    help="the step also rotates q and k (RoPE fused into the launch, as the model's forward)")
    ap.add_argument("--layers", type=int, default=24,
                    help="layers per decode step (one pool each; Qwen2.5-0.5B has 24)")
    ap.add_argument("--model-requests", type=int, default=256,
                    help="cfg2 line: requests per GPU of the saturated config-5 trace in its model_decode block "
                         "(0 = skip)")
    ap.add_argument("--model-rate", type=float, default=1000.0,
                    help="cfg2 line: arrival rate per GPU (req/s) of that trace")
    ap.add_argument("--model-kv-gb", type=float, default=60.0, help="cfg2 line: KV budget per GPU of that trace")
    ap.add_argument("--profile-decode", type=int, default=0,
                    help="cfg5: after the trace, profile this many decode steps at batch 256 per kernel "
                         "(torch.profiler CUDA activity)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference_arm(args)
    elif args.workload == "cfg5":
        run_model(args)
    elif args.workload == "ops":
        run_ops(args)
    elif args.workload == "cuda-core":
        run_cuda_core(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
