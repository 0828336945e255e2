#!/usr/bin/env python
"""KV-cache commitment throughput on B200 (trace bytes committed GB/s + kv_roots/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c2|c3|c5] [--impl ours|reference]

A step is one pass of the commitment hot path over one batch of synthetic
input resident in HBM: every (sequence, layer) K/V tree of the workload is
hashed (leaf encoding "vi-kv-v1" || layer || pos || f64(K) || f64(V),
SHA-256) and reduced to its kv_root with all nodes stored for openings; at
N > 1 the roots are all-gathered (NCCL) and the root-of-roots is built.

Workloads (seeded synthetic data, bf16 K/V ~ N(0, 1)):
  c2  Llama-3.1-8B shape: 32 layers x 8 KV heads x 128, 1 sequence x 4096 tokens (default)
  c3  Qwen2.5-7B shape: 28 layers x 4 x 128, 16 sequences x 8192, paged 16-token blocks, permuted pages
  c5  Llama-3.1-70B shape: 80 layers x 8 x 128, 4 sequences x 32768 per GPU (32 at 8 GPUs)
Every rank commits its own copy of the workload (weak scaling).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

BLK_OPS = 1384          # int32 ops per SHA-256 block (one compression), see DESIGN.md
WORKLOADS = {
    "c2": dict(name="llama3.1-8b-kv", n_layers=32, n_heads=8, head_dim=128, n_seqs=1, seq_len=4096, paged=False),
    "c3": dict(name="qwen2.5-7b-kv-paged", n_layers=28, n_heads=4, head_dim=128, n_seqs=16, seq_len=8192, paged=True),
    "c5": dict(name="llama3.1-70b-kv-shard", n_layers=80, n_heads=8, head_dim=128, n_seqs=4, seq_len=32768, paged=False),
}


def sha_blocks(msg_len: int) -> int:
    return (msg_len + 9 + 63) // 64


def algorithmic(w):
    """SHA-256 blocks and source bytes of one step (one rank)."""
    kv = w["n_heads"] * w["head_dim"]
    leaves = w["n_seqs"] * w["seq_len"] * w["n_layers"]
    pad = 1 << (w["seq_len"] - 1).bit_length()
    nodes = w["n_seqs"] * w["n_layers"] * (pad - 1)
    blocks = leaves * sha_blocks(16 + 16 * kv) + nodes * 2
    src_bytes = leaves * kv * 2 * 2
    msg_bytes = leaves * (16 + 16 * kv)
    return blocks, src_bytes, msg_bytes, leaves


class Clocks:
    """Samples nvidia-smi clocks and throttle reasons; summary() keeps the
    samples taken between mark_start() and mark_end() (host monotonic time)."""

    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self._p = None
        self.t_start = self.t_end = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self._p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                        "--format=csv,noheader,nounits", "-lms", "50"],
                                       stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
            deadline = time.monotonic() + 10
            while not self.rows and time.monotonic() < deadline:
                time.sleep(0.02)
        except OSError:
            self._p = None
        return self

    def _read(self):
        for line in self._p.stdout:
            self.rows.append((time.monotonic(), [x.strip() for x in line.split(",")]))

    def mark_start(self):
        self.t_start = time.monotonic()

    def mark_end(self):
        self.t_end = time.monotonic()

    def __exit__(self, *a):
        if self._p:
            time.sleep(0.06)
            self._p.terminate()
            try:
                self._p.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._p.kill()

    def summary(self):
        rows = [r for t, r in self.rows if len(r) > 8 and (self.t_start is None or self.t_start <= t <= self.t_end)]

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = sorted(v for v in (num(r[1]) for r in rows) if v is not None)
        mx = [v for v in (num(r[2]) for r in rows) if v is not None]
        pw = [v for v in (num(r[3]) for r in rows) if v is not None]
        reasons = set()
        for r in rows:
            for i, n in enumerate(self.NAMES):
                if r[5 + i].lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx[0] if mx else None,
                "reasons": sorted(reasons), "samples": len(sm), "power_w_max": max(pw) if pw else None}


def make_view(w, device, seed):
    import torch
    from commitllm_b200.commit import KvCacheView
    g = torch.Generator(device=f"cuda:{device}")
    g.manual_seed(seed)
    L, H, D, S, N = w["n_layers"], w["n_heads"], w["head_dim"], w["n_seqs"], w["seq_len"]
    if w["paged"]:
        bs = 16
        pages = S * N // bs
        k = [torch.randn(pages, bs, H, D, generator=g, device=f"cuda:{device}", dtype=torch.bfloat16) for _ in range(L)]
        v = [torch.randn(pages, bs, H, D, generator=g, device=f"cuda:{device}", dtype=torch.bfloat16) for _ in range(L)]
        perm = torch.randperm(pages, generator=g, device=f"cuda:{device}").to(torch.int32)
        bt = perm.view(S, N // bs).contiguous()
        return KvCacheView(k, v, [N] * S, block_tables=bt)
    k = [torch.randn(S * N, H, D, generator=g, device=f"cuda:{device}", dtype=torch.bfloat16) for _ in range(L)]
    v = [torch.randn(S * N, H, D, generator=g, device=f"cuda:{device}", dtype=torch.bfloat16) for _ in range(L)]
    return KvCacheView(k, v, [N] * S)


def host_transcript(w, seed, n_layers=None):
    """The workload's K/V as host bf16 bit arrays (numpy), for the CPU legs."""
    import numpy as np
    from tests import synth
    L = w["n_layers"] if n_layers is None else n_layers
    rows = w["n_seqs"] * w["seq_len"]
    rng = np.random.default_rng(seed)
    shape = (L, rows, w["n_heads"], w["head_dim"])
    k = synth.f32_to_bf16_bits(rng.standard_normal(shape, dtype=np.float32))
    v = synth.f32_to_bf16_bits(rng.standard_normal(shape, dtype=np.float32))
    return k, v


def cpu_commit_seconds(w, n_layers, n_threads, seed=7):
    """Time the oracle's C restatement (reference algorithm) on n_layers of the workload."""
    import numpy as np
    from commitllm_b200._lib import VC_DTYPE_BF16
    from tests.kvref import Transcript
    k, v = host_transcript(w, seed, n_layers)
    tr = Transcript(k, v, [w["seq_len"]] * w["n_seqs"], VC_DTYPE_BF16)
    t0 = time.perf_counter()
    tr.oracle(n_threads=n_threads, with_nodes=True)
    return time.perf_counter() - t0


def cpu_baseline_leg(w, reference_threads=False, budget_s=20.0):
    """(value GB/s, cores, sample text) of the CPU restatement on a bounded sample."""
    ncpu = os.cpu_count() or 1
    if reference_threads:
        threads = 1  # the reference hashes KV trees in a sequential per-layer loop
    else:
        threads = max(1, min(ncpu, w["n_seqs"] * w["n_layers"]))
    # size the sample: start with a few layers and grow within the budget
    layers = max(1, min(w["n_layers"], threads))
    dt = cpu_commit_seconds(w, layers, threads)
    per_layer = dt / layers
    more = int(min(w["n_layers"], max(layers, (budget_s * 0.5) / max(per_layer, 1e-6))))
    if more > layers and more * per_layer < budget_s:
        layers = more
        dt = cpu_commit_seconds(w, layers, threads)
    _, src, _, _ = algorithmic(dict(w, n_layers=layers))
    return src / dt / 1e9, threads, layers, dt


def run_reference(args, w, rank, world):
    """The reference's CPU algorithm (oracle port, all host threads) on bounded samples."""
    if rank != 0:
        return
    from commitllm_b200._lib import VC_DTYPE_BF16
    from tests.kvref import Transcript
    ncpu = os.cpu_count() or 1
    threads = max(1, min(ncpu, w["n_seqs"] * w["n_layers"]))
    layers = max(1, min(w["n_layers"], threads))
    k, v = host_transcript(w, 7, layers)
    tr = Transcript(k, v, [w["seq_len"]] * w["n_seqs"], VC_DTYPE_BF16)
    vals = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        tr.oracle(n_threads=threads, with_nodes=True)
        if i >= args.warmup:
            vals.append(time.perf_counter() - t0)
    t = sorted(vals)[len(vals) // 2]
    _, src, _, leaves = algorithmic(dict(w, n_layers=layers))
    value = src / t / 1e9
    sample = (f"{layers} of {w['n_layers']} layers x {w['n_seqs']} seq x {w['seq_len']} tokens per step, "
              f"oracle C restatement (OpenSSL SHA-256), {threads} threads over trees, median of {len(vals)} steps")
    line = {
        "impl": "reference", "metric": "trace bytes committed GB/s", "value": round(value, 4), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": {"workload": w["name"], "layers": w["n_layers"], "kv_heads": w["n_heads"], "head_dim": w["head_dim"],
                   "seqs": w["n_seqs"], "seq_len": w["seq_len"], "paged": w["paged"]},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "kv_roots_per_s": round(w["n_seqs"] * layers / t, 3),
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="c2", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    w = WORKLOADS[args.workload]
    if args.steps is None:
        # about a second of timed work, so the clock sampler sees the region
        args.steps = {"c2": 400, "c3": 40, "c5": 8}[args.workload] if args.impl == "ours" else 10

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, w, rank, world)
        return

    import torch
    import torch.distributed as dist
    from commitllm_b200 import commit as C
    from commitllm_b200 import dist as D

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device(f"cuda:{local}"))
    stream = torch.cuda.Stream(local)
    ctx = C.Context(local, stream)
    view = make_view(w, local, seed=1000 + rank)
    torch.cuda.synchronize()
    blocks, src_bytes, msg_bytes, leaves = algorithmic(w)
    n_trees = w["n_seqs"] * w["n_layers"]
    # weak scaling: rank r holds all trees of its own copy of the workload
    plan = [D.Shard(r, r + 1, 0, n_trees) for r in range(world)] if world > 1 else None

    roots_buf = ctx.empty(w["n_seqs"], w["n_layers"], 32)
    ror_buf = ctx.empty(1, 32)
    kern_ms = []

    def step(timed):
        e0 = e1 = None
        if timed:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        roots, trees = C.kv_commit(ctx, view, keep_trees=True, roots_out=roots_buf)
        if timed:
            e1.record(stream)
            kern_ms.append((e0, e1))
        if world > 1:
            with torch.cuda.stream(stream):
                full = D.gather_roots(roots.view(-1, 32), plan, world, n_trees, group=None)
                C.build_trees(ctx, full.view(-1, 32), [0, world * n_trees], keep_trees=False, roots_out=ror_buf)
        trees.free()

    for _ in range(args.warmup):
        step(False)
    ctx.sync(timeout_ms=600000)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()

    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        torch.cuda.synchronize()
        clk.mark_start()
        t0.record(stream)
        for _ in range(args.steps):
            step(True)
        t1.record(stream)
        torch.cuda.synchronize()
        clk.mark_end()
    ctx.sync(timeout_ms=600000)
    total_ms = t0.elapsed_time(t1)
    if world > 1:
        tt = torch.tensor([total_ms], device=f"cuda:{local}")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        total_ms = float(tt.item())
        dist.barrier()
    ms_step = total_ms / args.steps
    kms = sorted(a.elapsed_time(b) for a, b in kern_ms)
    k_avg = sum(kms) / len(kms)

    # integer-ALU peak probe on the same GPU, same run
    peak_ops = C.int_peak(ctx, 0, 4000)
    ctx.sync(timeout_ms=600000)

    # end to end through the public API from pinned host memory
    e2e = None
    if not args.no_e2e:
        host_k = [t.cpu().pin_memory() for t in view.k_layers]
        host_v = [t.cpu().pin_memory() for t in view.v_layers]
        dev_k = [torch.empty_like(t) for t in view.k_layers]
        dev_v = [torch.empty_like(t) for t in view.v_layers]
        view2 = C.KvCacheView(dev_k, dev_v, view.seq_lens, block_tables=view.block_tables)
        roots_host = torch.empty(w["n_seqs"], w["n_layers"], 32, dtype=torch.uint8).pin_memory()
        h2d = sum(t.numel() * t.element_size() for t in host_k + host_v)

        def e2e_step():
            with torch.cuda.stream(stream):
                for d, h in zip(dev_k + dev_v, host_k + host_v):
                    d.copy_(h, non_blocking=True)
                roots, trees = C.kv_commit(ctx, view2, keep_trees=True, roots_out=roots_buf)
                roots_host.copy_(roots, non_blocking=True)
                trees.free()

        for _ in range(3):
            e2e_step()
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        n_e2e = max(3, min(args.steps, 10))
        a.record(stream)
        for _ in range(n_e2e):
            e2e_step()
        b.record(stream)
        torch.cuda.synchronize()
        e_ms = a.elapsed_time(b) / n_e2e
        if world > 1:
            tt = torch.tensor([e_ms], device=f"cuda:{local}")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            e_ms = float(tt.item())
        e2e = {"value": round(src_bytes * world / (e_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": w["n_seqs"] * w["n_layers"] * 32,
               "ms_per_step": round(e_ms, 3)}
        del host_k, host_v, dev_k, dev_v

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        val, cores, layers, dt = cpu_baseline_leg(w, reference_threads=True)
        cpu = {"value": round(val, 4), "unit": "GB/s", "cores": cores, "kind": "port",
               "sample": f"{layers} of {w['n_layers']} layers x {w['n_seqs']} seq x {w['seq_len']} tokens "
                         f"({dt:.2f} s), oracle C restatement with OpenSSL SHA-256, the reference's sequential "
                         f"per-layer KV-tree loop (1 thread)"}

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except OSError:
        pass
    hbm = peaks.get("hbm_gbs", 6650.0)
    alu_achieved = blocks * BLK_OPS / (k_avg * 1e-3) / 1e12
    alu_peak = peak_ops / 1e12
    hbm_achieved = src_bytes / (k_avg * 1e-3) / 1e9
    clocks = clk.summary()
    value = src_bytes * world / (ms_step * 1e-3) / 1e9
    line = {
        "metric": "trace bytes committed GB/s", "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": {"workload": w["name"], "layers": w["n_layers"], "kv_heads": w["n_heads"],
                   "head_dim": w["head_dim"], "seqs_per_gpu": w["n_seqs"], "seq_len": w["seq_len"],
                   "paged": w["paged"], "parallelism": f"shard-by-sequence x{world}",
                   "l2": "inputs larger than L2 (%.0f MB per GPU)" % (src_bytes / 1e6)},
        "kv_roots_per_s": round(n_trees * world / (ms_step * 1e-3), 2),
        "hashed_msg_GBps": round(msg_bytes * world / (ms_step * 1e-3) / 1e9, 3),
        "roofline": {"bound": "int_alu", "achieved": round(alu_achieved, 3), "peak": round(alu_peak, 3),
                     "unit": "Tops/s", "frac": round(alu_achieved / alu_peak, 4), "traffic": None,
                     "kernel_ms": round(k_avg, 4), "sha_blocks": blocks, "ops_per_block": BLK_OPS,
                     "peak_source": "vc_int_peak SHA-mix probe, this GPU, this run",
                     "hbm": {"achieved": round(hbm_achieved, 1), "peak": hbm, "unit": "GB/s",
                             "frac": round(hbm_achieved / hbm, 4), "peak_source": "MEASURED_PEAKS.json hbm_gbs"}},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": args.steps * (1 + (1 if world > 1 else 0)),
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
