#!/usr/bin/env python
"""Trace-commitment throughput on B200 (trace bytes committed GB/s, + kv_roots/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c5|c2|c2t|c3|c4|online|request|capture] [--impl ours|reference]

A step is one pass of the commitment hot path over one batch of synthetic
input already resident in HBM.

KV workloads (bf16 K/V ~ N(0, 1), seeded): every (sequence, layer) tree is
hashed -- leaf "vi-kv-v1" || u32 layer || u32 pos || f64(K) || f64(V),
SHA-256 -- and reduced to its kv_root, nodes kept for openings.
  c5  Llama-3.1-70B shape: 80 layers x 8 x 128, 32 sequences x 32768 tokens, ONE job split over the
      N GPUs by sequence (strong scaling; default).  A GPU's share (32/N sequences x 80 layers, up to
      344 GB) does not fit HBM below N=4, so each GPU holds at most 8 distinct sequences x 80 layers
      (86 GB) resident and commits its share in calls of up to 8 sequences; sequence s of a share
      reads resident sequence s mod 8 (every leaf hashed, the same bytes re-read from HBM).  After
      the last call the 2 560 kv_roots are all-gathered (NCCL) and the root-of-roots is built.
  c2  Llama-3.1-8B shape: 32 layers x 8 KV heads x 128, 1 sequence x 4096 tokens
  c3  Qwen2.5-7B shape: 28 layers x 4 x 128, 16 sequences x 8192, paged 16-token blocks, permuted pages
Retained-state workload:
  c4  Llama-3.1-8B sampled decode: 256 sequences x 512 steps; per token 32 layers of a_i8[4096] +
      scale_a + x_attn_i8[4096] + scale_x_attn, and f32 captured logits[128256] ~ N(0, 3^2).
      A step = retained leaves of all 131 072 tokens, the 256 IO chains, the 512 trace/IO trees,
      prompt hashes and seed commitments.
Whole-request workload:
  request  one c2-shaped request through verilm_rs.commit_minimal_from_captures: retained leaves with
      the captured-logits wrap, the IO chain, the trace/IO trees and the 32 KV trees of its cache,
      on overlapped streams.
Capture workload:
  capture  a batch-1 decode step of a Llama-3.1-8B-shaped stand-in model (bf16 weights; four
      cutlass_scaled_mm-shaped calls per layer, lm_head, argmax sampler) with no capture, with the
      device capture (commitllm_b200.capture), and with the reference's host-copy capture restated;
      then each path's commit of the captured request.
Except c5, every rank commits its own copy of the workload (weak scaling); at
N > 1 the roots are all-gathered (NCCL) and the root-of-roots is built inside
the step.
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

# int32 ops per SHA-256 block (one compression): 64 rounds x (6 rotates + 4 logic + 4 adds)
# + 48 schedule words x (6 shifts + 2 logic + 2 adds) + 8 final adds
BLK_OPS = 1384
METRIC = "trace bytes committed GB/s"
WORKLOADS = {
    "c2": dict(kind="kv", name="llama3.1-8b-kv", n_layers=32, n_heads=8, head_dim=128, n_seqs=1, seq_len=4096,
               paged=False, steps=400),
    "c3": dict(kind="kv", name="qwen2.5-7b-kv-paged", n_layers=28, n_heads=4, head_dim=128, n_seqs=16,
               seq_len=8192, paged=True, steps=40),
    "c4": dict(kind="trace", name="llama3.1-8b-retained-logits", n_layers=32, hidden=4096, n_seqs=256,
               seq_len=512, vocab=128256, x_attn=True, steps=8),
    "c5": dict(kind="kv", name="llama3.1-70b-kv-32x32768", n_layers=80, n_heads=8, head_dim=128, n_seqs=32,
               seq_len=32768, paged=False, job=True, resident_seqs=8, steps=8),
    # the reference's weight-provider path: KV recomputed from x_attn (compute_kv_transcript), then committed
    # online per-step commit of a decode batch: 256 sequences, one token each per step (c4 shapes)
    "online": dict(kind="online", name="llama3.1-8b-online-decode", n_layers=32, hidden=4096, n_seqs=256,
                   vocab=128256, x_attn=True, steps=6),
    "c2t": dict(kind="kvt", name="llama3.1-8b-kv-transcript", n_layers=32, n_heads=8, head_dim=128, hidden=4096,
                n_seqs=1, seq_len=4096, rope="llama3", steps=250),
    # one whole request through verilm_rs.commit_request: Llama-3.1-8B shapes, 1024 prompt tokens + 3 072
    # decode steps (4 096 committed tokens), captured logits for the 3 073 generated tokens, its KV cache
    "request": dict(kind="request", name="llama3.1-8b-request-4096", n_layers=32, hidden=4096, n_heads=8,
                    head_dim=128, n_seqs=1, seq_len=4096, n_prompt=1024, vocab=128256, x_attn=False, steps=20),
    # capture cost per batch-1 decode step (Llama-3.1-8B shapes): no capture, the device capture, and the
    # reference's host-copy capture; then each path's commit of the captured request
    "capture": dict(kind="capture", name="llama3.1-8b-decode-capture", n_layers=32, hidden=4096, q_dim=4096,
                    kv_dim=1024, intermediate=14336, vocab=128256, steps=64),
}


def sha_blocks(msg_len: int) -> int:
    return (msg_len + 9 + 63) // 64


def tree_blocks(n_leaves: int) -> int:
    """SHA blocks of build_tree's internal nodes (2 per node, padded size)."""
    pad = 1 << (n_leaves - 1).bit_length() if n_leaves > 1 else 1
    return 2 * (pad - 1)


def algorithmic(w):
    """(SHA blocks of the dominant kernel, other blocks, source bytes, hashed bytes, n_roots) per rank-step.

    kvt: the source bytes are the f64 KvEntry rows the reference commits on
    this path (16 bytes per K/V element pair)."""
    if w["kind"] == "kvt":
        kv = w["n_heads"] * w["head_dim"]
        leaves = w["n_seqs"] * w["seq_len"] * w["n_layers"]
        blocks = leaves * sha_blocks(16 + 16 * kv) + w["n_seqs"] * w["n_layers"] * tree_blocks(w["seq_len"])
        return blocks, 0, leaves * kv * 16, leaves * (16 + 16 * kv), w["n_seqs"] * w["n_layers"]
    if w["kind"] == "kv":
        kv = w["n_heads"] * w["head_dim"]
        if w.get("split"):
            # split trees: this rank's range of the one sequence (aligned power of two)
            from commitllm_b200.dist import split_ranges
            rng = split_ranges(w["seq_len"], w["split"])[w.get("rank", 0)]
            leaves = rng.count * w["n_layers"]
            blocks = leaves * sha_blocks(16 + 16 * kv) + w["n_layers"] * tree_blocks(1 << rng.sub_log2)
            return blocks, 0, leaves * kv * 4, leaves * (16 + 16 * kv), w["n_layers"]
        leaves = w["n_seqs"] * w["seq_len"] * w["n_layers"]
        blocks = leaves * sha_blocks(16 + 16 * kv) + w["n_seqs"] * w["n_layers"] * tree_blocks(w["seq_len"])
        return blocks, 0, leaves * kv * 4, leaves * (16 + 16 * kv), w["n_seqs"] * w["n_layers"]
    if w["kind"] == "request":
        L, H, V, n = w["n_layers"], w["hidden"], w["vocab"], w["seq_len"]
        kv = w["n_heads"] * w["head_dim"]
        n_gen = n - (w["n_prompt"] - 1)
        base = 14 + L * (H + 4 + 1)
        trace = n * sha_blocks(base) + n_gen * sha_blocks(21 + 32 + 4 * V)
        kv_blocks = n * L * sha_blocks(16 + 16 * kv) + L * tree_blocks(n)
        other = 2 * n + 2 * tree_blocks(n) + kv_blocks
        src = n * L * (H + 4) + n_gen * 4 * V + n * L * kv * 4
        return trace, other, src, n * base + n_gen * (21 + 32 + 4 * V) + n * L * (16 + 16 * kv), 2 + L
    L, H, V = w["n_layers"], w["hidden"], w["vocab"]
    per_layer = H + 4 + 1 + ((H + 4) if w["x_attn"] else 0)
    base = 14 + L * per_layer
    logits = 21 + 32 + 4 * V
    n = w["n_seqs"] * w["seq_len"]
    leaf_blocks = n * (sha_blocks(base) + sha_blocks(logits))
    other = n * 2 + 2 * w["n_seqs"] * tree_blocks(w["seq_len"])          # IO chain + trace/IO trees
    src = n * (L * (H + 4 + ((H + 4) if w["x_attn"] else 0)) + 4 * V)
    return leaf_blocks, other, src, n * (base + logits), 2 * w["n_seqs"]


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


# ---------------------------------------------------------------------------
# KV workloads
# ---------------------------------------------------------------------------

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
        return KvCacheView(k, v, [N] * S, block_tables=perm.view(S, N // bs).contiguous())
    k = [torch.randn(S * N, H, D, generator=g, device=f"cuda:{device}", dtype=torch.bfloat16) for _ in range(L)]
    v = [torch.randn(S * N, H, D, generator=g, device=f"cuda:{device}", dtype=torch.bfloat16) for _ in range(L)]
    return KvCacheView(k, v, [N] * S)


class KvStep:
    """One KV commit of the whole workload (+ the exchange at N > 1)."""

    def __init__(self, w, ctx, stream, device, rank, world):
        import torch
        from commitllm_b200 import commit as C
        from commitllm_b200 import dist as D
        self.C, self.D, self.torch = C, D, torch
        self.w, self.ctx, self.stream, self.world = w, ctx, stream, world
        self.view = make_view(w, device, seed=1000 + rank)
        self.n_trees = w["n_seqs"] * w["n_layers"]
        self.plan = [D.Shard(r, r + 1, 0, self.n_trees) for r in range(world)] if world > 1 else None
        self.roots = ctx.empty(w["n_seqs"], w["n_layers"], 32)
        self.ror = ctx.empty(1, 32)
        self.kernel_events = []
        self.launches = 1 + (1 if world > 1 else 0)

    def __call__(self, timed: bool):
        torch, C = self.torch, self.C
        if timed:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(self.stream)
        roots, trees = C.kv_commit(self.ctx, self.view, keep_trees=True, roots_out=self.roots)
        if timed:
            e1.record(self.stream)
            self.kernel_events.append((e0, e1))
        if self.world > 1:
            with torch.cuda.stream(self.stream):
                full = self.D.gather_roots(roots.view(-1, 32), self.plan, self.world, self.n_trees)
                C.build_trees(self.ctx, full.view(-1, 32), [0, self.world * self.n_trees], keep_trees=False,
                              roots_out=self.ror)
        trees.free()

    def host_inputs(self):
        return list(self.view.k_layers) + list(self.view.v_layers)

    def e2e_step(self, host, dev_tensors, roots_host):
        """Public host-buffer API: layer groups copied while earlier groups hash."""
        C = self.C
        L = self.w["n_layers"]
        if not hasattr(self, "_copy_stream"):
            self._copy_stream = self.torch.cuda.Stream(self.ctx.device)
        roots, trees = C.kv_commit_host(self.ctx, host[:L], host[L:], self.view.seq_lens,
                                        block_tables=self.view.block_tables, dev_k=dev_tensors[:L],
                                        dev_v=dev_tensors[L:], roots_out=self.roots, copy_stream=self._copy_stream)
        with self.torch.cuda.stream(self.stream):
            roots_host.copy_(roots.view(-1), non_blocking=True)
        trees.free()
        return roots.numel()


class KvJobStep:
    """One KV job split over the ranks by sequence (``dist.shard_plan``): rank
    r commits its share of sequences x layers in calls of up to
    ``resident_seqs`` sequences over the resident K/V (sequence s of the share
    reads resident sequence s mod resident_seqs), keeping every tree for
    openings; then the job's kv_roots are all-gathered and the root-of-roots
    is built.  Every hash kernel of the job runs inside the step."""

    def __init__(self, w, ctx, stream, device, rank, world):
        import torch
        from commitllm_b200 import commit as C
        from commitllm_b200 import dist as D
        self.C, self.D, self.torch = C, D, torch
        self.w, self.ctx, self.stream, self.world = w, ctx, stream, world
        self.plan = D.shard_plan(w["n_seqs"], w["n_layers"], world)
        sh = self.plan[rank]
        self.shard = sh
        self.n_local = sh.seq_end - sh.seq_begin
        self.n_layers_local = sh.layer_end - sh.layer_begin
        self.resident = max(1, min(self.n_local, int(w.get("resident_seqs") or self.n_local)))
        res = dict(w, n_seqs=self.resident, n_layers=self.n_layers_local)
        self.view = make_view(res, device, seed=1000 + rank)
        self.view.layer_base = sh.layer_begin
        self.calls = [(b, min(self.resident, self.n_local - b)) for b in range(0, self.n_local, self.resident)]
        self.roots = ctx.empty(self.n_local, self.n_layers_local, 32)
        self.ror = ctx.empty(1, 32)
        self.trees = []                  # [(first local sequence, count, TreeSet)] of the last step
        self.kernel_events = []          # per call: (start, end) on the step stream
        self.exchange_events = []        # per step at N > 1: the all-gather of the roots + the root-of-roots
        self.launches = len(self.calls) + (1 if world > 1 else 0)

    def local_view(self, n):
        from dataclasses import replace
        return replace(self.view, seq_lens=list(self.view.seq_lens[:n]))

    def __call__(self, timed: bool):
        torch, C = self.torch, self.C
        for _, _, ts in self.trees:      # last step's node blocks go back to the context's pool
            ts.free()
        self.trees = []
        for b, n in self.calls:
            if timed:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(self.stream)
            _, ts = C.kv_commit(self.ctx, self.local_view(n), keep_trees=True, roots_out=self.roots[b:b + n])
            if timed:
                e1.record(self.stream)
                self.kernel_events.append((e0, e1))
            self.trees.append((b, n, ts))
        if self.world > 1:
            if timed:
                x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                x0.record(self.stream)
            with torch.cuda.stream(self.stream):
                full = self.D.gather_roots(self.roots.view(-1, 32), self.plan, self.w["n_seqs"], self.w["n_layers"])
                C.build_trees(self.ctx, full.view(-1, 32), [0, self.w["n_seqs"] * self.w["n_layers"]],
                              keep_trees=False, roots_out=self.ror)
            if timed:
                x1.record(self.stream)
                self.exchange_events.append((x0, x1))

    def locate(self, seq_local: int, layer_local: int):
        for b, n, ts in self.trees:
            if b <= seq_local < b + n:
                return ts, (seq_local - b) * self.n_layers_local + layer_local
        raise IndexError(seq_local)

    def host_inputs(self):
        return list(self.view.k_layers) + list(self.view.v_layers)


class SplitKvStep:
    """One request's KV trees split over the ranks by position (strong
    scaling): each rank holds and commits its aligned range of positions,
    the subtree roots are all-gathered, and every rank builds the top levels."""

    def __init__(self, w, ctx, stream, device, rank, world):
        import torch
        from commitllm_b200 import commit as C
        from commitllm_b200 import dist as D
        self.C, self.D, self.torch = C, D, torch
        self.w, self.ctx, self.stream, self.world = w, ctx, stream, world
        if w["n_seqs"] != 1:
            raise ValueError("split trees commit one sequence")
        self.rng = D.split_ranges(w["seq_len"], world)[rank]
        local = dict(w, seq_len=max(self.rng.count, 1))
        self.view = make_view(local, device, seed=5000 + rank)     # this rank's rows only
        self.launches = 3
        self.kernel_events = []

    def __call__(self, timed: bool):
        torch = self.torch
        if timed:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(self.stream)
        roots, trees, top = self.D.split_kv_commit(self.ctx, self.view, self.rng, self.w["n_layers"])
        if timed:
            e1.record(self.stream)
            self.kernel_events.append((e0, e1))

    def host_inputs(self):
        return list(self.view.k_layers) + list(self.view.v_layers)


# ---------------------------------------------------------------------------
# KV transcript workload (c2t): compute_kv_transcript + KV commit of its rows
# ---------------------------------------------------------------------------

class KvtStep:
    """K/V recomputed from captured x_attn and the resident Wk/Wv weights on the
    tensor cores (f64 dequant + RoPE) and the per-layer KV trees of those f64
    rows, in one pass (vc_kv_transcript_commit: the rows are hashed as they are
    computed, never stored); the exchange of roots at N > 1 as for the KV
    workloads.  two_call() times the same commitment as two kernels with the
    f64 rows through HBM, for comparison."""

    def __init__(self, w, ctx, stream, device, rank, world):
        import torch
        from commitllm_b200 import commit as C
        from commitllm_b200 import dist as D
        self.C, self.D, self.torch = C, D, torch
        self.w, self.ctx, self.stream, self.world = w, ctx, stream, world
        dev = f"cuda:{device}"
        g = torch.Generator(device=dev)
        g.manual_seed(3000 + rank)
        L, H, T = w["n_layers"], w["hidden"], w["n_seqs"] * w["seq_len"]
        self.kv = kv = w["n_heads"] * w["head_dim"]
        # captures in token order [T, L, hidden] (one int8 row per token and layer)
        self.x = torch.randint(-128, 128, (T, L, H), generator=g, device=dev, dtype=torch.int8)
        self.sx = torch.rand(T, L, generator=g, device=dev) * 0.05 + 1e-3
        self.wk = [torch.randint(-128, 128, (kv, H), generator=g, device=dev, dtype=torch.int8) for _ in range(L)]
        self.wv = [torch.randint(-128, 128, (kv, H), generator=g, device=dev, dtype=torch.int8) for _ in range(L)]
        self.sw = [(0.0021 + 1e-5 * l, 0.0017 + 1e-5 * l) for l in range(L)]
        self.inp = self.inputs(self.x, self.sx)
        self.k = ctx.empty(L, T, kv, dtype=torch.float64)
        self.v = ctx.empty(L, T, kv, dtype=torch.float64)
        self.view = C.kv_transcript_view(self.k, self.v)
        self.view.seq_lens = [w["seq_len"]] * w["n_seqs"]
        self.n_trees = w["n_seqs"] * L
        self.plan = [D.Shard(r, r + 1, 0, self.n_trees) for r in range(world)] if world > 1 else None
        self.roots = ctx.empty(w["n_seqs"], L, 32)
        self.ror = ctx.empty(1, 32)
        self.kernel_events = []     # the one-pass transcript + KV commit
        self.launches = 1 + (1 if world > 1 else 0)

    def inputs(self, x, sx):
        C, w = self.C, self.w
        return C.KvTranscriptInputs(x_attn=[x[:, l] for l in range(w["n_layers"])], wk=self.wk, wv=self.wv,
                                    scale_x=sx, n_kv_heads=w["n_heads"], head_dim=w["head_dim"], per_tensor=self.sw,
                                    rope=C.RopeConfig(theta=500000.0, scaling=w["rope"]))

    def __call__(self, timed: bool, inp=None):
        torch, C = self.torch, self.C
        if timed:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(self.stream)
        roots, _ = C.kv_transcript_commit(self.ctx, self.inp if inp is None else inp, keep_trees=False,
                                          roots_out=self.roots)
        if timed:
            e1.record(self.stream)
            self.kernel_events.append((e0, e1))
        if self.world > 1:
            with torch.cuda.stream(self.stream):
                full = self.D.gather_roots(roots.view(-1, 32), self.plan, self.world, self.n_trees)
                C.build_trees(self.ctx, full.view(-1, 32), [0, self.world * self.n_trees], keep_trees=False,
                              roots_out=self.ror)

    def two_call(self, reps: int = 10):
        """(transcript ms, KV commit ms) of the two-kernel path, and whether its
        roots equal the one-pass roots (device check)."""
        torch, C = self.torch, self.C
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(reps)]
        roots2 = self.ctx.empty(self.w["n_layers"], 32)
        for e in ev:
            e[0].record(self.stream)
            C.kv_transcript(self.ctx, self.inp, self.k, self.v)
            e[1].record(self.stream)
            C.kv_commit(self.ctx, self.view, keep_trees=False, roots_out=roots2)
            e[2].record(self.stream)
        torch.cuda.synchronize()
        t = sum(e[0].elapsed_time(e[1]) for e in ev) / reps
        k = sum(e[1].elapsed_time(e[2]) for e in ev) / reps
        self(False)
        torch.cuda.synchronize()
        return t, k, bool(torch.equal(roots2, self.roots.view(-1, 32)[: self.w["n_layers"]]))

    def host_inputs(self):
        return [self.x, self.sx]

    def e2e_step(self, host, dev_tensors, roots_host):
        """Public API from host captures: x_attn and scale_x copied in, weights resident."""
        with self.torch.cuda.stream(self.stream):
            for d, h in zip(dev_tensors, host):
                d.copy_(h, non_blocking=True)
        key = tuple(t.data_ptr() for t in dev_tensors)
        if getattr(self, "_e2e_key", None) != key:
            self._e2e_inp = self.inputs(*dev_tensors)
            self._e2e_key = key
        self(False, inp=self._e2e_inp)
        with self.torch.cuda.stream(self.stream):
            roots_host.copy_(self.roots.view(-1), non_blocking=True)
        return self.roots.numel()


# ---------------------------------------------------------------------------
# Retained-state workload (c4)
# ---------------------------------------------------------------------------

class TraceStep:
    """Retained leaves + IO chains + trace/IO trees + prompt/seed hashes of n_seqs requests."""

    def __init__(self, w, ctx, stream, device, rank, world):
        import torch
        from commitllm_b200 import commit as C
        from commitllm_b200 import dist as D
        self.C, self.D, self.torch = C, D, torch
        self.w, self.ctx, self.stream, self.world = w, ctx, stream, world
        dev = f"cuda:{device}"
        g = torch.Generator(device=dev)
        g.manual_seed(2000 + rank)
        L, H, B, T, V = w["n_layers"], w["hidden"], w["n_seqs"], w["seq_len"], w["vocab"]
        # captures as a decode engine lays them out: step k, layer l, batch row = sequence
        self.a = torch.randint(-128, 128, (T, L, B, H), generator=g, device=dev, dtype=torch.int8)
        self.x = torch.randint(-128, 128, (T, L, B, H), generator=g, device=dev, dtype=torch.int8) if w["x_attn"] else None
        self.sa = torch.rand(T, L, B, generator=g, device=dev) * 0.05 + 1e-3
        self.sx = torch.rand(T, L, B, generator=g, device=dev) * 0.05 + 1e-3
        self.logits = torch.randn(B * T, V, generator=g, device=dev) * 3.0       # row = token s*T + k
        self.tok = torch.randint(0, V, (B * T,), generator=g, device=dev, dtype=torch.int32)
        self.seeds = torch.randint(0, 256, (B, 32), generator=g, device=dev, dtype=torch.uint8)
        self.prompts = [f"synthetic prompt {rank}:{s}".encode() for s in range(B)]
        self.n = B * T
        self.plan = self.make_plan()
        self.both = ctx.empty(2 * self.n, 32)
        self.tree_off = [s * T for s in range(B)] + [self.n + s * T for s in range(B + 1)]
        self.roots = ctx.empty(2 * B, 32)
        self.n_roots = 2 * B
        self.rplan = [D.Shard(r, r + 1, 0, self.n_roots) for r in range(world)] if world > 1 else None
        self.ror = ctx.empty(1, 32)
        self.kernel_events = []
        self.launches = 5 + (1 if world > 1 else 0)

    def make_plan(self, a=None, x=None, sa=None, sx=None, logits=None):
        import numpy as np
        C, w = self.C, self.w
        a = self.a if a is None else a
        x = self.x if x is None else x
        sa = self.sa if sa is None else sa
        sx = self.sx if sx is None else sx
        logits = self.logits if logits is None else logits
        L, H, B, T = w["n_layers"], w["hidden"], w["n_seqs"], w["seq_len"]
        t = np.arange(B * T)
        lay = C.TraceLayout(
            n_layers=L, hidden=H, fwd_rows=[B] * T, tok_fwd=t % T, tok_row=t // T,
            a_rows=[[a.data_ptr() + ((k * L + l) * B) * H for l in range(L)] for k in range(T)],
            scale_a=[[sa.data_ptr() + 4 * ((k * L + l) * B) for l in range(L)] for k in range(T)], scale_stride=1,
            x_attn_rows=None if x is None else [[x.data_ptr() + ((k * L + l) * B) * H for l in range(L)] for k in range(T)],
            scale_x_attn=None if x is None else [[sx.data_ptr() + 4 * ((k * L + l) * B) for l in range(L)] for k in range(T)],
            scale_x_stride=1, logits=logits, tok_logits_row=t)
        return C.TracePlan(lay)

    def __call__(self, timed: bool, plan=None, tok=None, seeds=None):
        torch, C = self.torch, self.C
        plan = self.plan if plan is None else plan
        n = self.n
        if timed:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(self.stream)
        plan.run(self.ctx, self.both[:n])
        if timed:
            e1.record(self.stream)
            self.kernel_events.append((e0, e1))
        ph = C.prompt_hashes(self.ctx, self.prompts)
        C.io_chain(self.ctx, self.both[:n], self.tok if tok is None else tok, ph,
                   [s * self.w["seq_len"] for s in range(self.w["n_seqs"] + 1)], out=self.both[n:])
        C.build_trees(self.ctx, self.both, self.tree_off, keep_trees=False, roots_out=self.roots)
        C.seed_commitments(self.ctx, self.seeds if seeds is None else seeds)
        if self.world > 1:
            with torch.cuda.stream(self.stream):
                full = self.D.gather_roots(self.roots, self.rplan, self.world, self.n_roots)
                C.build_trees(self.ctx, full.view(-1, 32), [0, self.world * self.n_roots], keep_trees=False,
                              roots_out=self.ror)

    def host_inputs(self):
        out = [self.a, self.sa, self.sx, self.logits, self.tok, self.seeds]
        if self.x is not None:
            out.insert(1, self.x)
        return out

    def e2e_step(self, host, dev_tensors, roots_host):
        with self.torch.cuda.stream(self.stream):
            for d, h in zip(dev_tensors, host):
                d.copy_(h, non_blocking=True)
        if self.x is not None:
            a, x, sa, sx, logits, tok, seeds = dev_tensors
        else:
            a, sa, sx, logits, tok, seeds = dev_tensors
            x = None
        key = tuple(t.data_ptr() for t in dev_tensors)
        if getattr(self, "_e2e_key", None) != key:
            self._e2e_plan = self.make_plan(a, x, sa, sx, logits)
            self._e2e_key = key
        self(False, plan=self._e2e_plan, tok=tok, seeds=seeds)
        roots_host.copy_(self.roots.view(-1), non_blocking=True)
        return self.roots.numel()


# ---------------------------------------------------------------------------
# Whole-request workload
# ---------------------------------------------------------------------------

REQUEST_MANIFEST = {"tokenizer_hash": "11" * 32, "temperature": 0.7, "top_k": 50, "top_p": 0.9, "eos_policy": "stop",
                    "weight_hash": "22" * 32, "quant_hash": "33" * 32, "system_prompt_hash": "44" * 32,
                    "max_tokens": 3072, "sampler_version": "chacha20-vi-sample-v1", "decode_mode": "sampled",
                    "n_layers": 32, "hidden_dim": 4096, "vocab_size": 128256, "kv_dim": 1024, "d_head": 128,
                    "n_q_heads": 32, "n_kv_heads": 8, "rope_theta": 500000.0, "rmsnorm_eps": 1e-5}


class RequestStep:
    """One request's whole commitment through ``verilm_rs.commit_request`` (captures
    and KV cache resident), ending with the commitment read back to the host, as a
    server returns it.  The timed interval is the request's latency on the GPU
    timeline, host orchestration included."""

    def __init__(self, w, ctx, stream, device, rank, world):
        import torch
        from commitllm_b200 import commit as C
        from commitllm_b200 import verilm_rs as V
        self.C, self.V, self.torch = C, V, torch
        self.w, self.ctx, self.stream, self.world = w, ctx, stream, world
        dev = f"cuda:{device}"
        g = torch.Generator(device=dev)
        g.manual_seed(6000 + rank)
        L, H, n, Vb = w["n_layers"], w["hidden"], w["seq_len"], w["vocab"]
        self.n_gen = n - (w["n_prompt"] - 1)
        self.a = torch.randint(-128, 128, (n, L, H), generator=g, device=dev, dtype=torch.int8)
        self.sa = torch.rand(n, L, generator=g, device=dev) * 0.05 + 1e-3
        self.logits = torch.randn(self.n_gen, Vb, generator=g, device=dev) * 3.0
        self.tok = torch.randint(0, Vb, (n,), generator=g, device=dev, dtype=torch.int32)
        self.view = make_view(dict(w, paged=False), device, seed=7000 + rank)
        self.kernel_events = []
        self.launches = 6     # trace leaves, prompt hash, IO chain, trace/IO trees, seed commitment, KV trees

    def commit(self, ctx=None):
        return self.V.commit_request(self.a, self.sa, self.tok, b"synthetic prompt", b"\x07" * 32,
                                     n_prompt_tokens=self.w["n_prompt"], captured_logits_f32=self.logits,
                                     kv_cache=self.view, manifest=REQUEST_MANIFEST, ctx=ctx or self.ctx)

    def __call__(self, timed: bool):
        torch = self.torch
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        h = self.commit()
        self.last = h.commitment_json()        # synchronises: the roots are on the host
        e1.record(self.stream)
        if timed:
            self.kernel_events.append((e0, e1))

    def phases(self):
        """Device time of each part on its own (ms): trace leaves, IO chain, KV trees."""
        torch, C = self.torch, self.C
        n = self.w["seq_len"]
        h = self.commit()
        lay = h._layout
        leaves = self.ctx.empty(n, 32)
        ph = C.prompt_hashes(self.ctx, [b"synthetic prompt"])
        io = self.ctx.empty(n, 32)
        out = {}
        for name, fn in (("trace_leaves", lambda: C.trace_leaves(self.ctx, lay, out=leaves)),
                         ("io_chain", lambda: C.io_chain(self.ctx, leaves, self.tok, ph, [0, n], out=io)),
                         ("kv_trees", lambda: C.kv_commit(self.ctx, self.view, keep_trees=True)[1].free())):
            fn()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(self.stream)
            fn()
            b.record(self.stream)
            torch.cuda.synchronize()
            out[name] = round(a.elapsed_time(b), 3)
        return out


# ---------------------------------------------------------------------------
# CPU legs: the oracle's C restatement of the reference algorithm
# ---------------------------------------------------------------------------

def host_kv(w, seed, n_layers):
    """bf16 K/V [n_layers, rows, heads, dim] on the host: one layer of N(0, 1)
    values repeated over the layers (SHA-256 costs the same for any bytes; the
    layer index in each leaf keeps the trees distinct)."""
    import numpy as np
    from tests import synth
    rows = w["n_seqs"] * w["seq_len"]
    rng = np.random.default_rng(seed)
    shape = (rows, w["n_heads"], w["head_dim"])
    k1 = synth.f32_to_bf16_bits(rng.standard_normal(shape, dtype=np.float32))
    v1 = synth.f32_to_bf16_bits(rng.standard_normal(shape, dtype=np.float32))
    return np.repeat(k1[None], n_layers, axis=0), np.repeat(v1[None], n_layers, axis=0)


def cpu_kv(w, n_layers, n_threads, reps=1, seed=7):
    """Seconds per commit of n_layers of the KV workload (median of reps), reference algorithm."""
    from commitllm_b200._lib import VC_DTYPE_BF16
    from tests.kvref import Transcript
    k, v = host_kv(w, seed, n_layers)
    tr = Transcript(k, v, [w["seq_len"]] * w["n_seqs"], VC_DTYPE_BF16)
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        tr.oracle(n_threads=n_threads, with_nodes=True)
        ts.append(time.perf_counter() - t0)
    return sorted(ts)[len(ts) // 2]


def cpu_trace(w, n_tokens, n_threads, reps=1, seed=9, logits_wrap=True):
    """Seconds to hash n_tokens retained leaves (+ their IO chain) of the c4 / request workload on the host."""
    import ctypes
    import numpy as np
    from commitllm_b200._lib import TraceDesc
    from oracle import vco
    L, H, V = w["n_layers"], w["hidden"], w["vocab"]
    rng = np.random.default_rng(seed)
    a = rng.integers(-128, 128, size=(L, n_tokens, H), dtype=np.int8)
    x = rng.integers(-128, 128, size=(L, n_tokens, H), dtype=np.int8)
    sc = rng.random((L, n_tokens), dtype=np.float32)
    logits = rng.standard_normal((n_tokens, V), dtype=np.float32)
    keep = [a, x, sc, logits]

    def per_layer(arr, stride):
        p = (ctypes.c_void_p * L)(*[arr.ctypes.data + l * stride for l in range(L)])
        keep.append(p)
        return ctypes.cast(p, ctypes.POINTER(ctypes.c_void_p))

    def i32(vals):
        arr = (ctypes.c_int32 * len(vals))(*vals)
        keep.append(arr)
        return ctypes.cast(arr, ctypes.POINTER(ctypes.c_int32))

    d = TraceDesc()
    d.n_tokens, d.n_layers, d.hidden, d.n_fwd = n_tokens, L, H, 1
    d.fwd_rows, d.tok_fwd, d.tok_row = i32([n_tokens]), i32([0] * n_tokens), i32(list(range(n_tokens)))
    d.a_rows = per_layer(a, n_tokens * H)        # layer l, row r at a + l*n*H + r*H
    d.scale_a = per_layer(sc, n_tokens * 4)
    d.scale_stride = 1
    if w["x_attn"]:
        d.x_attn_rows = per_layer(x, n_tokens * H)
        d.scale_x_attn = per_layer(sc, n_tokens * 4)
        d.scale_x_stride = 1
    if logits_wrap:
        d.logits, d.vocab, d.logits_rows, d.logits_stride = logits.ctypes.data, V, n_tokens, V
        d.tok_logits_row = i32(list(range(n_tokens)))
    leaves = np.zeros((n_tokens, 32), np.uint8)
    toks = rng.integers(0, V, size=n_tokens, dtype=np.uint32)
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        vco.lib().vco_trace_leaves(ctypes.byref(d), leaves.ctypes.data, n_threads)
        vco.io_chain(leaves, toks, b"synthetic prompt")
        ts.append(time.perf_counter() - t0)
    return sorted(ts)[len(ts) // 2]


def cpu_kvt(w, n_pos, n_threads, seed=11):
    """Seconds to recompute n_pos positions x all layers of the c2t transcript on the host
    (compute_kv_transcript restated in C, one position range per thread)."""
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor
    from oracle import commit_oracle as O
    from oracle import vco
    L, H, nh, hd = w["n_layers"], w["hidden"], w["n_heads"], w["head_dim"]
    kv = nh * hd
    rng = np.random.default_rng(seed)
    x = rng.integers(-128, 128, (n_pos, L, H), dtype=np.int8)
    wk = [rng.integers(-128, 128, (kv, H), dtype=np.int8) for _ in range(L)]
    wv = [rng.integers(-128, 128, (kv, H), dtype=np.int8) for _ in range(L)]
    sx = rng.random((n_pos, L), dtype=np.float32)
    sw = np.full((L, 2), 0.002, np.float32)
    inv = np.array(O.scaled_inv_freq(hd, 500000.0, O.RopeScaling()))
    parts = np.array_split(np.arange(n_pos), max(1, min(n_threads, n_pos)))
    t0 = time.perf_counter()
    with ThreadPoolExecutor(len(parts)) as ex:
        list(ex.map(lambda p: vco.kv_transcript(x[p], wk, wv, sx[p], nh, hd, sw=sw, inv_freq=inv), parts))
    return time.perf_counter() - t0


def cpu_host():
    """The host CPU the CPU legs ran on: model name and hardware threads."""
    model = "unknown"
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"cpu_model": model, "host_threads": os.cpu_count() or 1}


def cpu_leg(w, reference_threads: bool, budget_s: float = 20.0, reps: int = 1):
    """(GB/s, threads, sample text, seconds) of the CPU restatement on a bounded sample of w."""
    ncpu = os.cpu_count() or 1
    _, _, src_full, _, _ = algorithmic(w)
    if w["kind"] == "kvt":
        # transcript: the reference runs compute_kv_transcript on one thread (prover/src/lib.rs:207-329);
        # the KV trees of its f64 rows cost what the c2 trees cost (same SHA blocks per leaf)
        threads = 1 if reference_threads else ncpu
        n_pos = max(1, threads)
        per_pos = cpu_kvt(w, n_pos, threads) / n_pos
        n_pos = int(max(n_pos, min(w["seq_len"], budget_s * 0.5 / max(per_pos, 1e-6))))
        dt_t = cpu_kvt(w, n_pos, threads)
        wkv = dict(w, kind="kv", paged=False)
        kv_threads = 1 if reference_threads else max(1, min(ncpu, w["n_layers"]))
        layers = max(1, min(w["n_layers"], kv_threads))
        dt_h = cpu_kv(wkv, layers, kv_threads)
        positions = w["n_seqs"] * w["seq_len"]
        total = dt_t * positions / n_pos + dt_h * w["n_layers"] / layers
        sample = (f"transcript of {n_pos} of {positions} positions x {w['n_layers']} layers ({dt_t:.2f} s, "
                  f"{threads} thread(s)) + KV trees of {layers} of {w['n_layers']} layers ({dt_h:.2f} s, "
                  f"{kv_threads} thread(s)), oracle C restatement, extrapolated linearly to the workload")
        return src_full / total / 1e9, threads, sample, total
    if w["kind"] == "request":
        # commit_minimal as the reference runs it (prover/src/lib.rs:336-544): trace leaves on all host
        # threads (rayon, 371-393), the IO chain serial (403-410), the KV trees in a sequential
        # per-layer loop (454-478); each part timed on a sample and scaled to the request
        n = w["seq_len"]
        n_gen = n - (w["n_prompt"] - 1)
        threads = ncpu
        n_tok = max(64, 8 * threads)
        dt_l = cpu_trace(w, n_tok, threads, logits_wrap=True) / n_tok
        dt_b = cpu_trace(w, n_tok, threads, logits_wrap=False) / n_tok
        kv_threads = 1 if reference_threads else max(1, min(ncpu, w["n_layers"]))
        wkv = dict(w, kind="kv", paged=False)
        layers = max(1, min(w["n_layers"], kv_threads, 8))
        dt_kv = cpu_kv(wkv, layers, kv_threads) / layers * w["n_layers"]
        total = dt_l * n_gen + dt_b * (n - n_gen) + dt_kv
        sample = (f"{n_tok} tokens with and {n_tok} without the logits wrap ({threads} threads, IO chain serial) + "
                  f"{layers} of {w['n_layers']} KV trees ({kv_threads} thread(s)), oracle C restatement, scaled to "
                  f"{n_gen} + {n - n_gen} tokens and {w['n_layers']} trees; KV part {dt_kv:.2f} s")
        return src_full / total / 1e9, threads, sample, total
    if w["kind"] == "kv":
        # the reference hashes KV trees in a sequential per-layer loop (prover/src/lib.rs:454-478);
        # every (sequence, layer) tree costs the same, so the sample is whole trees of one
        # sequence (up to all its layers), extrapolated by tree count
        n_trees = w["n_seqs"] * w["n_layers"]
        w1 = dict(w, n_seqs=1, paged=False)
        threads = 1 if reference_threads else max(1, min(ncpu, n_trees))
        # at most ~2 GB of host K/V per sample
        cap = max(1, min(w["n_layers"], int(2e9 // (4 * w["seq_len"] * w["n_heads"] * w["head_dim"]))))
        layers = max(1, min(cap, threads))
        per = cpu_kv(w1, layers, threads) / layers
        layers = int(min(cap, max(layers, budget_s * 0.5 / max(per, 1e-6))))
        if layers > threads:
            layers -= layers % threads          # whole rounds of trees over the threads
        dt = cpu_kv(w1, layers, threads, reps=reps)
        src = src_full * layers / n_trees
        sample = (f"{layers} of {n_trees} trees ({w['n_seqs']} seq x {w['n_layers']} layers) of {w['seq_len']} "
                  f"tokens, oracle C restatement (OpenSSL SHA-256), {threads} thread(s) over trees, bytes per "
                  f"second of the sample (every tree costs the same)")
        return src / dt / 1e9, threads, sample, dt
    # retained leaves: the reference uses rayon over tokens (prover/src/lib.rs:371-393), IO chain serial
    threads = ncpu
    n_tok = 32 * threads
    dt = cpu_trace(w, n_tok, threads)
    n_tok = int(min(4096, max(n_tok, n_tok * budget_s * 0.5 / max(dt, 1e-6))))   # <= ~3.2 GB of host data
    dt = cpu_trace(w, n_tok, threads, reps=reps)
    per_tok = src_full / (w["n_seqs"] * w["seq_len"])
    sample = (f"{n_tok} of {w['n_seqs'] * w['seq_len']} tokens (retained leaves with x_attn + logits wrap, "
              f"IO chain), oracle C restatement (OpenSSL SHA-256), {threads} threads over tokens")
    return per_tok * n_tok / dt / 1e9, threads, sample, dt


def run_online(args, w, local):
    """Online commit (OnlineCommitter.step) of a decode batch, alone and beside
    a stream of bf16 GEMMs standing in for the model's forward pass."""
    import torch
    from commitllm_b200 import commit as C
    from commitllm_b200.online import OnlineCommitter
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    L, H, V, B = w["n_layers"], w["hidden"], w["vocab"], w["n_seqs"]
    stream = torch.cuda.Stream(local)
    ctx = C.Context(local, stream)
    n_steps = args.steps + args.warmup
    oc = OnlineCommitter(ctx, max_slots=B, max_tokens=2 * n_steps + 4, defer_tokens=0)
    for s_ in range(B):
        oc.open(s_, b"synthetic prompt %d" % s_, bytes([s_ % 256]) * 32, n_prompt_tokens=1)
    g = torch.Generator(device=dev)
    g.manual_seed(4000)
    a = torch.randint(-128, 128, (L, B, H), dtype=torch.int8, device=dev, generator=g)
    x = torch.randint(-128, 128, (L, B, H), dtype=torch.int8, device=dev, generator=g)
    sa = torch.rand(L, B, device=dev, generator=g) * 0.05 + 1e-3
    logits = torch.randn(B, V, device=dev, generator=g) * 3.0
    tok = torch.randint(0, V, (B,), dtype=torch.int32, device=dev, generator=g)
    lay = C.TraceLayout(n_layers=L, hidden=H, fwd_rows=[B], tok_fwd=[0] * B, tok_row=list(range(B)),
                        a_rows=[[a[l].data_ptr() for l in range(L)]], scale_a=[[sa[l].data_ptr() for l in range(L)]],
                        scale_stride=1, x_attn_rows=[[x[l].data_ptr() for l in range(L)]],
                        scale_x_attn=[[sa[l].data_ptr() for l in range(L)]], scale_x_stride=1,
                        logits=logits, tok_logits_row=list(range(B)))
    slots = list(range(B))
    for _ in range(args.warmup):
        oc.step(slots, lay, tok)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        clk.mark_start()
        e0.record(stream)
        for _ in range(args.steps):
            oc.step(slots, lay, tok)
        e1.record(stream)
        torch.cuda.synchronize()
        clk.mark_end()
    ms = e0.elapsed_time(e1) / args.steps
    # beside a model: bf16 GEMMs on another stream while one more step commits
    A = torch.randn(8192, 8192, dtype=torch.bfloat16, device=dev)
    Bm = torch.randn(8192, 8192, dtype=torch.bfloat16, device=dev)
    gs = torch.cuda.Stream(local)
    with torch.cuda.stream(gs):
        for _ in range(3):
            torch.matmul(A, Bm)
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_g = 40
    with torch.cuda.stream(gs):
        s0.record(gs)
        for _ in range(n_g):
            torch.matmul(A, Bm)
        s1.record(gs)
    torch.cuda.synchronize()
    g_alone = s0.elapsed_time(s1) / n_g
    with torch.cuda.stream(gs):
        s0.record(gs)
    oc.step(slots, lay, tok)
    with torch.cuda.stream(gs):
        for _ in range(n_g):
            torch.matmul(A, Bm)
        s1.record(gs)
    torch.cuda.synchronize()
    g_with = s0.elapsed_time(s1) / n_g
    for s_ in range(B):
        oc.close(s_)
    ctx.sync(600000)
    # deferred: 32 decode steps queued, then hashed in one launch (8 192 chains instead of 256)
    n_def = 32
    od = OnlineCommitter(ctx, max_slots=B, max_tokens=2 * n_def + 4, defer_tokens=B * n_def)
    for s_ in range(B):
        od.open(s_, b"synthetic prompt %d" % s_, bytes([s_ % 256]) * 32, n_prompt_tokens=1)
    for _ in range(n_def):                       # warm-up round
        od.step(slots, lay, tok)
    torch.cuda.synchronize()
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0.record(stream)
    for _ in range(n_def):
        od.step(slots, lay, tok)
    d1.record(stream)
    torch.cuda.synchronize()
    ms_def = d0.elapsed_time(d1) / n_def
    for s_ in range(B):
        od.close(s_)
    ctx.sync(600000)
    per_tok = 14 + L * (H + 4 + 1 + (H + 4 if w["x_attn"] else 0)) + 21 + 32 + 4 * V
    blocks = B * (sha_blocks(14 + L * (H + 4 + 1 + (H + 4 if w["x_attn"] else 0))) + sha_blocks(21 + 32 + 4 * V))
    peak_ops = C.int_peak(ctx, 0, 4000)
    achieved = blocks * BLK_OPS / (ms * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": round(B * per_tok / (ms * 1e-3) / 1e9, 3), "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": {"workload": w["name"], "n_layers": L, "hidden": H, "vocab": V, "sequences": B,
                   "tokens_per_step": B, "x_attn": w["x_attn"], "l2": "inputs reused per step (%.0f MB)" %
                   (B * per_tok / 1e6)},
        "roofline": {"bound": "latency", "achieved": round(achieved, 3), "peak": round(peak_ops / 1e12, 3),
                     "unit": "Tops/s", "frac": round(achieved / (peak_ops / 1e12), 4), "traffic": None,
                     "kernel": "trace_leaf_kernel + io_chain_kernel",
                     "note": "one thread per token: %d CTAs of %d SMs, each thread hashes %d serial blocks" %
                             ((B + 127) // 128, ctx_sm(), blocks // B)},
        "beside_gemm": {"gemm_ms_alone": round(g_alone, 3), "gemm_ms_with_online_step": round(g_with, 3),
                        "gemm": "bf16 8192^3 on another stream"},
        "deferred": {"steps_per_flush": n_def, "ms_per_step": round(ms_def, 3),
                     "GBps": round(B * per_tok / (ms_def * 1e-3) / 1e9, 3),
                     "note": "OnlineCommitter(defer_tokens=%d): the 32 steps' tokens hashed in one launch" % (B * n_def)},
        "gpu_launches": args.steps * 2, "clocks": clk.summary(), "e2e": None, "cpu_baseline": None,
    }
    print(json.dumps(line), flush=True)


class _HostCopyCapture:
    """The reference's capture path restated for timing: each o_proj input
    copied to a pinned host slab with a non-blocking device-to-host copy
    (sidecar/verilm/capture.py:733-763), each qkv_proj input copied to the host
    (x_attn capture, on by default at the server; capture.py:352-373, 930-933),
    each call's scale kept as a GPU reference (capture.py:918-920), and each
    sampled logits row pulled to the host with ``.float().cpu()``
    (sampler.py:153-154).  The drain waits for the transfers and concatenates
    the scales on the host."""

    def __init__(self, n_layers, hidden, capacity_rows=32768):
        import torch
        self.L, self.H = n_layers, hidden
        self.calls_per_fwd = 4 * n_layers
        self.slab = torch.empty(capacity_rows, hidden, dtype=torch.int8, pin_memory=True)
        self.reset()

    def reset(self):
        self.counter, self.idx = 0, 0
        self.offsets, self.x_attn, self.scales, self.logits = [], [], [], []

    def wrap(self, real):
        def wrapped(a, b, scale_a, scale_b, out_dtype, bias=None):
            out = real(a, b, scale_a, scale_b, out_dtype, bias)
            proj = (self.counter % self.calls_per_fwd) % 4
            self.counter += 1
            self.scales.append(scale_a)
            if proj == 1:
                rows = a.shape[0]
                self.slab[self.idx:self.idx + rows].copy_(a, non_blocking=True)
                self.offsets.append((self.idx, self.idx + rows))
                self.idx += rows
            elif proj == 0:
                self.x_attn.append(a.to("cpu", non_blocking=True))
            return out
        return wrapped

    def capture_logits(self, logits):
        self.logits.append(logits[-1].float().cpu().numpy())

    def drain(self):
        import torch
        torch.cuda.synchronize()
        o = [self.slab[s:e].numpy() for s, e in self.offsets]
        sc = torch.cat([t.flatten() for t in self.scales]).cpu().numpy()
        out = (o, sc, [t.numpy() for t in self.x_attn], self.logits)
        self.reset()
        return out


def run_capture(args, w, local):
    """Capture cost per batch-1 decode step, three ways, then each path's commit.

    The stand-in model runs per layer the four cutlass_scaled_mm-shaped calls
    (qkv_proj, o_proj, gate_up_proj, down_proj; bf16 weights of Llama-3.1-8B
    shapes, int8 activation rows) through the op the capture wraps, then the
    lm_head and an argmax sampler whose ``.item()`` ends the step (so a step's
    wall time is its latency).  Arms: the bare op; the device capture
    (DeviceCaptureBuffer + DeviceLogitsCapture); the reference's host-copy
    capture restated (_HostCopyCapture).  Each captured request (warm-up and
    timed steps) is then committed: the device captures in place
    (commit_captures), the host copies through commit_minimal_from_captures."""
    import numpy as np
    import torch
    from commitllm_b200 import capture as K
    from commitllm_b200 import commit as C
    from commitllm_b200 import verilm_rs as VR
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    L, H, I, V = w["n_layers"], w["hidden"], w["intermediate"], w["vocab"]
    q = w["q_dim"] + 2 * w["kv_dim"]
    g = torch.Generator(device=dev)
    g.manual_seed(21)
    bf = torch.bfloat16
    W = [[torch.randn(q, H, generator=g, device=dev, dtype=bf) * 0.02,
          torch.randn(H, w["q_dim"], generator=g, device=dev, dtype=bf) * 0.02,
          torch.randn(2 * I, H, generator=g, device=dev, dtype=bf) * 0.02,
          torch.randn(H, I, generator=g, device=dev, dtype=bf) * 0.02] for _ in range(L)]
    W_lm = torch.randn(V, H, generator=g, device=dev, dtype=bf) * 0.02
    a_h = torch.randint(-128, 128, (1, H), generator=g, device=dev, dtype=torch.int8)
    a_q = torch.randint(-128, 128, (1, w["q_dim"]), generator=g, device=dev, dtype=torch.int8)
    a_i = torch.randint(-128, 128, (1, I), generator=g, device=dev, dtype=torch.int8)
    s_row = torch.rand(1, 1, generator=g, device=dev) * 0.05 + 1e-3
    h_last = torch.randn(1, H, generator=g, device=dev, dtype=bf)

    def real(a, b, sa, sb, dt, bias=None):
        return torch.matmul(a.to(bf), b.t())

    def step(op, on_logits):
        for l in range(L):
            op(a_h, W[l][0], s_row, None, bf, None)
            op(a_q, W[l][1], s_row, None, bf, None)
            op(a_h, W[l][2], s_row, None, bf, None)
            op(a_i, W[l][3], s_row, None, bf, None)
        logits = torch.matmul(h_last, W_lm.t())
        on_logits(logits)
        return int(logits[-1].argmax().item())

    dbuf = K.DeviceCaptureBuffer(L, H, o_dim=w["q_dim"], device=dev)
    dlog = K.DeviceLogitsCapture(V, device=dev)
    hcap = _HostCopyCapture(L, w["q_dim"])
    arms = {"none": (real, lambda lg: None), "device": (dbuf.wrap(real), dlog.capture),
            "host_copy": (hcap.wrap(real), hcap.capture_logits)}
    n_req = args.warmup + args.steps
    res = {}
    with Clocks(local) as clk:
        clk.mark_start()
        for name, (op, on_logits) in arms.items():
            for _ in range(args.warmup):
                step(op, on_logits)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            walls = []
            e0.record()
            for _ in range(args.steps):
                t0 = time.perf_counter()
                step(op, on_logits)
                walls.append(time.perf_counter() - t0)
            e1.record()
            torch.cuda.synchronize()
            res[name] = {"ms_per_step": round(float(np.mean(walls)) * 1e3, 4),
                         "median_ms": round(float(np.median(walls)) * 1e3, 4),
                         "max_ms": round(float(np.max(walls)) * 1e3, 4),
                         "device_ms_per_step": round(e0.elapsed_time(e1) / args.steps, 4)}
        clk.mark_end()
    ids = [int(t) for t in np.random.default_rng(3).integers(0, V, n_req + 1)]
    ctx = C.Context(local)
    prompt, seed = b"capture workload prompt", bytes(32)
    commit_ms = {}
    for rep in range(2):                      # the first commit of each path warms its plans
        t0 = time.perf_counter()
        caps, logits = (dbuf.drain(), dlog.drain()) if rep == 0 else (caps, logits)
        hd = K.commit_captures(caps, ids[1:], prompt, seed, n_prompt_tokens=1, logits=logits, ctx=ctx)
        root_d = hd.merkle_root_hex()
        commit_ms["device"] = round((time.perf_counter() - t0) * 1e3, 3)
        t0 = time.perf_counter()
        if rep == 0:
            o, sc, xs, lg = hcap.drain()
        hh = VR.commit_minimal_from_captures(o, sc, L, [1] * n_req, ids[1:], prompt, seed, n_prompt_tokens=1,
                                             captured_logits_f32=lg, ctx=ctx)
        root_h = hh.merkle_root_hex()
        commit_ms["host_copy"] = round((time.perf_counter() - t0) * 1e3, 3)
    if root_d != root_h:
        raise SystemExit("device and host-copy captures committed different roots")
    d2h = L * (H + w["q_dim"]) + 4 * V + 4 * L * 4
    ov = {k: round(res[k]["ms_per_step"] - res["none"]["ms_per_step"], 4) for k in ("device", "host_copy")}
    line = {
        "metric": "decode step with capture (ms)", "value": res["device"]["ms_per_step"], "unit": "ms",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["device"]["ms_per_step"],
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "i8", "data": "synthetic",
        "config": {"workload": w["name"], "n_layers": L, "hidden": H, "intermediate": I, "vocab": V, "batch": 1,
                   "model": "stand-in: bf16 weights of Llama-3.1-8B shapes, random init"},
        "arms": res, "capture_overhead_ms": ov,
        "d2h_bytes_per_step": {"device": 0, "host_copy": d2h},
        "commit_ms": dict(commit_ms, tokens=n_req, note="warm commit of the captured request (second of two)"),
        "roots_equal": True, "clocks": clk.summary(), "e2e": None, "cpu_baseline": None, "roofline": None,
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


def ctx_sm():
    import torch
    return torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count


def config_of(w, world):
    c = {k: v for k, v in w.items() if k not in ("steps", "name", "kind", "rank")}
    c["workload"] = w["name"]
    if w.get("split"):
        c["parallelism"] = f"split-trees x{world}"
    elif w.get("job"):
        c["parallelism"] = f"one job, shard_plan by sequence x{world}"
    else:
        c["parallelism"] = f"every rank its own copy x{world}"
    return c


def run_reference(args, w, rank, world):
    """The reference's CPU algorithm (oracle port, all host threads) on bounded samples."""
    if rank != 0:
        return
    reps = max(1, args.steps)
    val, threads, sample, dt = cpu_leg(w, reference_threads=False, reps=reps)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(val, 4), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True,
        "scaling": "strong" if (w.get("job") or args.split_trees) else "weak", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic", "config": config_of(dict(w, split=world) if args.split_trees else w, world),
        "cpu_baseline": {"value": round(val, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample + f", median of {reps} steps", **cpu_host()},
        "e2e": {"value": round(val, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="c5", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--seqs", type=int, default=None, help="override the workload's sequence count")
    ap.add_argument("--layers", type=int, default=None, help="override the workload's layer count (small captures)")
    ap.add_argument("--split-trees", action="store_true",
                    help="N > 1: spread one request's trees over the ranks by position (strong scaling)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    w = dict(WORKLOADS[args.workload])
    if args.seqs:
        w["n_seqs"] = args.seqs
    if args.layers:
        w["n_layers"] = args.layers
    if args.steps is None:
        # about a second of timed work, so the clock sampler sees the region
        args.steps = w["steps"] if args.impl == "ours" else 5

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if w["kind"] == "online":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the reference has no online per-step commit"}))
            return
        if w["kind"] == "capture":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the capture workload times the reference's "
                                  "host-copy capture itself, in its own line"}))
            return
        run_reference(args, w, rank, world)
        return
    if w["kind"] == "capture":
        if world > 1:
            raise SystemExit("the capture workload runs on one GPU")
        run_capture(args, w, local)
        return
    if w["kind"] == "online":
        if world > 1:
            raise SystemExit("the online workload runs on one GPU")
        run_online(args, w, local)
        return

    import torch
    import torch.distributed as dist
    from commitllm_b200 import commit as C

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device(f"cuda:{local}"))
    stream = torch.cuda.Stream(local)
    ctx = C.Context(local, stream)
    if args.split_trees:
        if w["kind"] != "kv" or w["n_seqs"] != 1:
            raise SystemExit("--split-trees needs a one-sequence KV workload (c2)")
        w = dict(w, split=world, rank=rank)
        step = SplitKvStep(w, ctx, stream, local, rank, world)
        args.no_e2e = True
    elif w.get("job"):
        step = KvJobStep(w, ctx, stream, local, rank, world)
    elif w["kind"] == "request":
        if world > 1:
            raise SystemExit("the request workload runs on one GPU")
        step = RequestStep(w, ctx, stream, local, rank, world)
        args.no_e2e = True
    else:
        step = {"kv": KvStep, "kvt": KvtStep, "trace": TraceStep}[w["kind"]](w, ctx, stream, local, rank, world)
    torch.cuda.synchronize()
    # per-rank work of one step (a job's share, or this rank's copy)
    w_rank = dict(w, n_seqs=step.n_local, n_layers=step.n_layers_local) if w.get("job") else w
    blocks, other_blocks, src_bytes, msg_bytes, n_roots = algorithmic(w_rank)

    for _ in range(args.warmup):
        step(False)
    ctx.sync(timeout_ms=600000)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    step.kernel_events.clear()
    if hasattr(step, "exchange_events"):
        step.exchange_events.clear()

    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    # The clock sampler starts (and delivers its first row) before the ranks
    # meet, and the timed region of every rank opens right after one device-side
    # rendezvous on the step stream, so no rank starts its clock early.
    with Clocks(local) as clk:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        if world > 1:
            with torch.cuda.stream(stream):
                dist.all_reduce(torch.ones(1, device=f"cuda:{local}"))
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
    kms = [a.elapsed_time(b) for a, b in step.kernel_events]
    k_avg = sum(kms) / len(kms)               # one launch of the dominant kernel
    k_step = sum(kms) / args.steps            # all its launches of one step

    # the token-level IO chain of the KV workloads' sequences, timed on its own
    # (serial: one warp per sequence; not part of the KV step above)
    io_chain = None
    if w["kind"] in ("kv", "kvt"):
        S, T = w_rank["n_seqs"], w["seq_len"]
        g = torch.Generator(device=f"cuda:{local}")
        g.manual_seed(77)
        leaves = torch.randint(0, 256, (S * T, 32), generator=g, device=f"cuda:{local}", dtype=torch.uint8)
        tok = torch.randint(0, 128256, (S * T,), generator=g, device=f"cuda:{local}", dtype=torch.int32)
        ph = C.prompt_hashes(ctx, [b"synthetic prompt %d" % s for s in range(S)])
        io_out = ctx.empty(S * T, 32)
        off = [s * T for s in range(S + 1)]
        C.io_chain(ctx, leaves, tok, ph, off, out=io_out)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        C.io_chain(ctx, leaves, tok, ph, off, out=io_out)
        b.record(stream)
        torch.cuda.synchronize()
        io_ms = a.elapsed_time(b)
        io_chain = {"chains": S, "tokens_per_chain": T, "ms": round(io_ms, 3),
                    "ns_per_token": round(io_ms * 1e6 / T, 1)}
        if rank == 0 and world == 1 and not args.no_cpu:
            import numpy as np
            from oracle import vco
            lh, th = leaves[:T].cpu().numpy(), tok[:T].cpu().numpy().view(np.uint32)
            t_c = time.perf_counter()
            vco.io_chain(lh, th, b"synthetic prompt 0")
            io_chain["cpu_ms_one_chain"] = round((time.perf_counter() - t_c) * 1e3, 3)
        del leaves, tok, io_out

    # openings: merkle::prove for 1 024 random (sequence, layer, position) leaves of one more commit
    openings = None
    if w["kind"] == "kv" and w.get("job"):
        # 1 024 random (sequence, layer, position) openings of this rank's trees of the last timed step
        import numpy as np
        r_ = np.random.default_rng(99 + rank)
        n_open = 1024
        seqs = r_.integers(0, step.n_local, n_open)
        lays = r_.integers(0, step.n_layers_local, n_open)
        poss = r_.integers(0, w["seq_len"], n_open)
        groups = {}
        for sq, ly, ps in zip(seqs, lays, poss):
            ts, t = step.locate(int(sq), int(ly))
            groups.setdefault(id(ts), (ts, [], []))[1].append(t)
            groups[id(ts)][2].append(int(ps))
        for ts, tl, pl in groups.values():
            ts.prove(tl[:8], pl[:8])
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        depth = 0
        for ts, tl, pl in groups.values():
            _, depths = ts.prove(tl, pl)
            depth = int(depths[0])
        b.record(stream)
        torch.cuda.synchronize()
        openings = {"n": n_open, "ms": round(a.elapsed_time(b), 3), "siblings_each": depth,
                    "what": "merkle::prove of random (sequence, layer, position) leaves of the job's trees, batched, "
                            "device"}
    elif w["kind"] == "kv" and not w.get("split"):
        import numpy as np
        r_ = np.random.default_rng(99 + rank)
        n_open = 1024
        tr_ids = r_.integers(0, w["n_seqs"] * w["n_layers"], n_open).tolist()
        lf_ids = r_.integers(0, w["seq_len"], n_open).tolist()
        _, trees_o = C.kv_commit(ctx, step.view, keep_trees=True, roots_out=step.roots)
        trees_o.prove(tr_ids[:8], lf_ids[:8])
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        sib, depths = trees_o.prove(tr_ids, lf_ids)
        b.record(stream)
        torch.cuda.synchronize()
        openings = {"n": n_open, "ms": round(a.elapsed_time(b), 3), "siblings_each": int(depths[0]),
                    "what": "merkle::prove of random (sequence, layer, position) leaves, batched, device"}
        del sib
        trees_o.free()

    request_phases = step.phases() if w["kind"] == "request" else None

    # integer-ALU peak probe on the same GPU, same run
    peak_ops = C.int_peak(ctx, 0, 4000)
    ctx.sync(timeout_ms=600000)

    # the one-pass kernel's tensor-core work against cuBLAS int8 (torch._int_mm, 8192^3), same GPU,
    # same run, and the two-kernel path (f64 rows through HBM) it replaces
    transcript = None
    if w["kind"] == "kvt":
        T = w["n_seqs"] * w["seq_len"]
        ops = 2.0 * T * 2 * step.kv * w["hidden"] * w["n_layers"]
        t_two, k_two, same = step.two_call()
        with torch.cuda.stream(stream):
            ga = torch.randint(-128, 128, (8192, 8192), device=f"cuda:{local}", dtype=torch.int8)
            gb = torch.randint(-128, 128, (8192, 8192), device=f"cuda:{local}", dtype=torch.int8).t()
            for _ in range(3):
                torch._int_mm(ga, gb)
            ms_l = []
            for _ in range(10):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                torch._int_mm(ga, gb)
                b.record(stream)
                b.synchronize()
                ms_l.append(a.elapsed_time(b))
        int8_peak = 2.0 * 8192 ** 3 / (min(ms_l) * 1e-3) / 1e12
        del ga, gb
        transcript = {"kernel": "kvt_commit_kernel (one pass: int8 MMA + f64 dequant/RoPE + SHA-256 + trees)",
                      "kernel_ms": round(k_avg, 4), "tensor_achieved": round(ops / (k_avg * 1e-3) / 1e12, 1),
                      "tensor_peak": round(int8_peak, 1), "unit": "int8 TOP/s",
                      "tensor_frac": round(ops / (k_avg * 1e-3) / 1e12 / int8_peak, 4),
                      "peak_source": "cuBLAS int8 GEMM (torch._int_mm, 8192^3, best of 10), this GPU, this run",
                      "two_call": {"kv_transcript_ms": round(t_two, 4), "kv_commit_ms": round(k_two, 4),
                                   "total_ms": round(t_two + k_two, 4), "roots_equal": same,
                                   "what": "vc_kv_transcript (f64 rows to HBM) then vc_kv_commit of them"}}

    # end to end through the public API from pinned host memory
    e2e = None
    if not args.no_e2e:
        e2e_note = None
        estep, e_src, e_roots = step, src_bytes, n_roots
        if w["kind"] == "trace":
            # 101.6 GB of captures per step would not fit pinned host memory: the
            # e2e leg commits a 16-sequence slice of the same workload
            w_e = dict(w, n_seqs=16)
            estep = TraceStep(w_e, ctx, stream, local, rank, world=1)
            _, _, e_src, _, e_roots = algorithmic(w_e)
            e2e_note = "16 of 256 sequences per step (same shapes)"
        elif w.get("job"):
            # the job's share from pinned host memory would be up to 344 GB: the e2e leg
            # commits the resident sequences x a layer slice (<= 4 GiB per step, same shapes)
            w_s = dict(w_rank, n_seqs=step.resident, job=False)
            src_s = algorithmic(w_s)[2]
            n_l = max(1, min(w_s["n_layers"], int(w_s["n_layers"] * (4 << 30) // src_s)))
            w_e = dict(w_s, n_layers=n_l)
            estep = KvStep(w_e, ctx, stream, local, rank, world=1)
            _, _, e_src, _, e_roots = algorithmic(w_e)
            e2e_note = (f"{step.resident} of {w['n_seqs']} sequences x {n_l} of {w['n_layers']} layers per step "
                        f"(same shapes)")
        elif src_bytes > (4 << 30):
            # keep the pinned host copy bounded: commit a layer slice of the same workload
            n_l = max(1, int(w["n_layers"] * (4 << 30) // src_bytes))
            w_e = dict(w, n_layers=n_l)
            estep = KvStep(w_e, ctx, stream, local, rank, world=1)
            _, _, e_src, _, e_roots = algorithmic(w_e)
            e2e_note = f"{n_l} of {w['n_layers']} layers per step (same shapes)"
        host = [t.cpu().pin_memory() for t in estep.host_inputs()]
        dev = [torch.empty_like(t) for t in estep.host_inputs()]
        roots_host = torch.empty(e_roots * 32, dtype=torch.uint8).pin_memory()
        h2d = sum(t.numel() * t.element_size() for t in host)

        def e2e_step():
            with torch.cuda.stream(stream):
                return estep.e2e_step(host, dev, roots_host)

        for _ in range(3 if w["kind"] != "trace" else 1):
            e2e_step()
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        n_e2e = max(3, min(args.steps, 10)) if w["kind"] != "trace" else 2
        d2h = 0
        a.record(stream)
        for _ in range(n_e2e):
            d2h = e2e_step()
        b.record(stream)
        torch.cuda.synchronize()
        e_ms = a.elapsed_time(b) / n_e2e
        if world > 1:
            tt = torch.tensor([e_ms], device=f"cuda:{local}")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            e_ms = float(tt.item())
        e2e = {"value": round(e_src * world / (e_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e_ms, 3)}
        if e2e_note:
            e2e["sample"] = e2e_note
        del host, dev, estep

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        val, cores, sample, dt = cpu_leg(w, reference_threads=True)
        cpu = {"value": round(val, 4), "unit": "GB/s", "cores": cores, "kind": "port",
               "sample": sample + f" ({dt:.2f} s); the reference's own threading for this path", **cpu_host()}

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
    alu_achieved = blocks * BLK_OPS / (k_step * 1e-3) / 1e12
    alu_peak = peak_ops / 1e12
    hbm_achieved = src_bytes / (k_step * 1e-3) / 1e9
    # whole-job bytes: one job over all ranks (c5, split trees), or every rank its own copy
    strong = bool(w.get("split") or w.get("job"))
    job_w = {k: v for k, v in w.items() if k not in ("split", "rank")}
    job_bytes = algorithmic(job_w)[2] if strong else src_bytes * world
    job_roots = algorithmic(job_w)[4] if strong else n_roots * world
    # the integer ALU pipe's own rate at the clock seen: 4 sub-partitions x 16 int32 lanes per clock per SM
    clocks = clk.summary()
    n_sm = torch.cuda.get_device_properties(local).multi_processor_count
    pipe_peak = n_sm * 64 * (clocks["sm_mhz"] or 1965.0) * 1e6 / 1e12
    line = {
        "metric": METRIC, "value": round(job_bytes / (ms_step * 1e-3) / 1e9, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "strong" if strong else "weak", "vs_baseline": None,
        "dtype": "u8", "data": "synthetic",
        "config": config_of(w, world),
        "l2": "inputs larger than L2 (%.0f MB read per GPU per step)" % (src_bytes / 1e6),
        "roots_per_s": round(job_roots / (ms_step * 1e-3), 2),
        "hashed_msg_GBps": round(msg_bytes * (job_bytes / src_bytes) / (ms_step * 1e-3) / 1e9, 3),
        "roofline": {"bound": "int_alu", "achieved": round(alu_achieved, 3), "peak": round(alu_peak, 3),
                     "unit": "Tops/s", "frac": round(alu_achieved / alu_peak, 4),
                     "traffic": None,
                     "algorithmic_bytes": src_bytes,
                     "kernel": {"trace": "trace_leaf_kernel", "kvt": "kvt_commit_kernel"}.get(w["kind"],
                                                                                              "kv_commit_kernel"),
                     "kernel_ms": round(k_avg, 4), "launches_per_step": len(kms) // args.steps,
                     "sha_blocks": blocks, "ops_per_block": BLK_OPS,
                     "peak_source": "vc_int_peak SHA-mix probe, this GPU, this run",
                     "alu_pipe": {"peak": round(pipe_peak, 3), "frac": round(alu_achieved / pipe_peak, 4),
                                  "source": "%d SMs x 64 int32 lanes/clk x median SM clock in the timed region; "
                                            "IMADs on the FMA pipe can lift a kernel above it" % n_sm},
                     "hbm": {"achieved": round(hbm_achieved, 1), "peak": hbm, "unit": "GB/s",
                             "frac": round(hbm_achieved / hbm, 4), "peak_source": "MEASURED_PEAKS.json hbm_gbs"}},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "io_chain": io_chain,
        "openings": openings,
        "transcript": transcript,
        "gpu_launches": args.steps * step.launches,
        "clocks": clocks,
    }
    if w["kind"] == "request":
        ops = (blocks + other_blocks) * BLK_OPS / (ms_step * 1e-3) / 1e12
        line["roofline"] = {
            "bound": "latency", "achieved": round(ops, 3), "peak": round(alu_peak, 3), "unit": "Tops/s",
            "frac": round(ops / alu_peak, 4), "traffic": None, "algorithmic_bytes": src_bytes,
            "kernel": "commit_request (trace_leaf_kernel, io_chain_kernel, tree_commit_kernel, kv_commit_kernel)",
            "note": "one request: %d serial SHA chains for the trace leaves (%d blocks each with the logits "
                    "wrap), then the IO chain, 2 dependent blocks per token; the KV trees run on a second stream "
                    "beside them" % (w["seq_len"], sha_blocks(14 + w["n_layers"] * (w["hidden"] + 5))
                                     + sha_blocks(53 + 4 * w["vocab"]))}
        ph = request_phases
        line["phases_ms"] = ph
        line["io_chain_share"] = round(ph["io_chain"] / ms_step, 3)
        line["serial_floor_ms"] = round(ph["trace_leaves"] + ph["io_chain"], 3)
    if w.get("job"):
        xs = [a.elapsed_time(b) for a, b in step.exchange_events]
        line["step_breakdown_ms"] = {
            "kv_commit_kernels": round(k_step, 3),
            "exchange": round(sum(xs) / len(xs), 3) if xs else 0.0,
            "what": "per step on rank 0: the commit launches, then the NCCL all-gather of the 32-byte roots and the "
                    "root-of-roots tree; the rest of ms_per_step is launch gaps and the wait for the slowest rank"}
    if w["kind"] in ("kv", "kvt"):
        line["kv_roots_per_s"] = line["roots_per_s"]
    if w["kind"] == "kvt":
        line["config"]["source_bytes"] = "f64 KvEntry rows committed (16 B per K/V element pair)"
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
