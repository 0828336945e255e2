"""Online (per decode step) commitment of a batch of requests.

The reference commits once, after generation (``commit_minimal``,
crates/verilm-prover/src/lib.rs:336-499): trace leaves for every token, the
serial IO chain, then the trace and IO trees.  Here the same values are built
while the requests decode: after a forward pass, the new tokens'
retained-state leaves are hashed and each request's IO chain is extended by
its new tokens on the GPU; closing a request builds its two trees.  The roots
equal the offline commit of the same captures, bit for bit, so the receipts
are unchanged -- only the time at which the hashing happens moves.

SHA-256 is serial within a message, so one pass of B tokens is B independent
chains: a decode step of 256 long leaves (logits wraps of 8 017 blocks) is
latency-bound on a few SMs.  ``defer_tokens`` trades latency for parallelism:
passes are queued and hashed together once that many tokens are pending (or
at ``flush`` / ``close``).  Deferring is the default (``DEFAULT_DEFER_TOKENS``,
8 192 tokens: 32 decode steps of a 256-sequence batch), which keeps both the
long leaves and the serial IO chain off the decode step and off the
post-generation critical path; ``defer_tokens=0`` hashes every pass as it is
stepped.  Deferred passes are read at flush time, so their capture buffers
must stay valid until then: a caller that reuses capture buffers keeps at
least ``ceil(defer_tokens / tokens per pass)`` of them in a ring, or calls
``flush`` before overwriting one.  Wrap tensors (logits, final residuals, lp
hidden) are read in place when every queued pass uses the same tensor (a ring
buffer with per-token rows), and gathered otherwise.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

from . import commit as C
from ._lib import check, lib

DEFAULT_DEFER_TOKENS = 8192


@dataclass
class _Pass:
    slots: List[int]
    layout: C.TraceLayout
    token_ids: torch.Tensor


def _runs(slots: Sequence[int]):
    """(slot, first index, count) of each slot's consecutive tokens; a slot may
    appear in one run only."""
    runs = []
    for i, s in enumerate(slots):
        s = int(s)
        if runs and runs[-1][0] == s:
            runs[-1][2] += 1
        else:
            if any(r[0] == s for r in runs):
                raise ValueError(f"tokens of slot {s} are not consecutive")
            runs.append([s, i, 1])
    return runs


def _merge_wrap(ctx, passes: List[_Pass], tensor_attr: str, rows_attr: str):
    """One wrap tensor + per-token rows for the concatenated passes."""
    tens = [getattr(p.layout, tensor_attr) for p in passes]
    if all(t is None for t in tens):
        return None, None
    rows_all: List[int] = []
    first = next(t for t in tens if t is not None)
    same = all(t is None or (t.data_ptr() == first.data_ptr() and t.shape == first.shape
                             and t.stride() == first.stride()) for t in tens)
    if same:
        for p, t in zip(passes, tens):
            n = len(p.layout.tok_fwd)
            rows = getattr(p.layout, rows_attr)
            rows_all += list(rows) if (t is not None and rows is not None) else [-1] * n
        return first, rows_all
    # different tensors per pass: gather the referenced rows into one tensor
    picks = []
    for p, t in zip(passes, tens):
        n = len(p.layout.tok_fwd)
        rows = getattr(p.layout, rows_attr)
        for j in range(n):
            r = int(rows[j]) if (t is not None and rows is not None) else -1
            if r < 0:
                rows_all.append(-1)
            else:
                rows_all.append(len(picks))
                picks.append(t[r])
    with torch.cuda.stream(ctx.stream):
        merged = torch.stack(picks) if picks else None
    return merged, rows_all


def _merge_layouts(ctx, passes: List[_Pass]) -> C.TraceLayout:
    l0 = passes[0].layout
    fwd_rows, tok_fwd, tok_row, a_rows, scale_a, x_rows, scale_x = [], [], [], [], [], [], []
    has_x = l0.x_attn_rows is not None
    for p in passes:
        lay = p.layout
        if (lay.n_layers, lay.hidden, lay.scale_stride, lay.scale_x_stride) != \
                (l0.n_layers, l0.hidden, l0.scale_stride, l0.scale_x_stride) or (lay.x_attn_rows is not None) != has_x:
            raise ValueError("deferred passes must share n_layers, hidden, scale strides and x_attn presence")
        base = len(fwd_rows)
        fwd_rows += list(lay.fwd_rows)
        tok_fwd += [base + int(f) for f in lay.tok_fwd]
        tok_row += list(lay.tok_row)
        a_rows += [list(r) for r in lay.a_rows]
        scale_a += [list(r) for r in lay.scale_a]
        if has_x:
            x_rows += [list(r) for r in lay.x_attn_rows]
            scale_x += [list(r) for r in lay.scale_x_attn]
    fr, fr_rows = _merge_wrap(ctx, passes, "final_residual", "tok_fr_row")
    lp, lp_rows = _merge_wrap(ctx, passes, "lp_hidden", "tok_lp_row")
    lg, lg_rows = _merge_wrap(ctx, passes, "logits", "tok_logits_row")
    return C.TraceLayout(n_layers=l0.n_layers, hidden=l0.hidden, fwd_rows=fwd_rows, tok_fwd=tok_fwd,
                         tok_row=tok_row, a_rows=a_rows, scale_a=scale_a, scale_stride=l0.scale_stride,
                         x_attn_rows=x_rows if has_x else None, scale_x_attn=scale_x if has_x else None,
                         scale_x_stride=l0.scale_x_stride, final_residual=fr, tok_fr_row=fr_rows,
                         lp_hidden=lp, tok_lp_row=lp_rows, logits=lg, tok_logits_row=lg_rows)


class OnlineCommitter:
    """Per-request histories of trace leaves and IO values, held on the device.

    ``max_slots`` requests can be open at once, each with at most
    ``max_tokens`` committed tokens (``token_ids = all_ids[1:]`` in the
    reference, i.e. one per forward-pass row).  ``defer_tokens``: N > 0
    queues passes until N tokens are pending (default
    ``DEFAULT_DEFER_TOKENS``; see the module docstring for the capture
    lifetime this requires); 0 hashes every pass when it is stepped.
    """

    def __init__(self, ctx: C.Context, max_slots: int, max_tokens: int, defer_tokens: int = DEFAULT_DEFER_TOKENS):
        self.ctx = ctx
        self.max_slots, self.max_tokens = int(max_slots), int(max_tokens)
        self.defer_tokens = int(defer_tokens)
        self.leaves = ctx.empty(self.max_slots, self.max_tokens, 32)
        self.io = ctx.empty(self.max_slots, self.max_tokens, 32)
        self.prev = ctx.empty(self.max_slots, 32)
        self.count = [0] * self.max_slots        # tokens hashed into each slot's history
        self.queued = [0] * self.max_slots       # tokens of each slot waiting in deferred passes
        self.pending: List[_Pass] = []
        self.n_pending = 0
        self.open_slots: Dict[int, dict] = {}

    def open(self, slot: int, prompt: bytes, sampling_seed: bytes, n_prompt_tokens: Optional[int] = None) -> None:
        """Start a request: prompt hash, seed commitment and the IO chain's genesis."""
        if not 0 <= slot < self.max_slots or slot in self.open_slots:
            raise ValueError(f"slot {slot} is out of range or already open")
        seed = bytes(sampling_seed)
        if len(seed) != 32:
            raise ValueError("sampling_seed must be exactly 32 bytes")
        ph = C.prompt_hashes(self.ctx, [bytes(prompt)])
        check(lib().vc_io_genesis(self.ctx.handle, 1, ctypes.c_void_p(ph.data_ptr()),
                                  ctypes.c_void_p(self.prev[slot].data_ptr())))
        sc = C.seed_commitments(self.ctx, self.ctx.to_device(np.frombuffer(seed, np.uint8).reshape(1, 32)))
        self.count[slot] = 0
        self.queued[slot] = 0
        self.open_slots[slot] = {"prompt_hash": ph, "seed_commitment": sc, "n_prompt_tokens": n_prompt_tokens}

    def step(self, slots: Sequence[int], layout: C.TraceLayout, token_ids: torch.Tensor) -> None:
        """Commit one forward pass: token i of ``layout`` belongs to request ``slots[i]``.

        A request's tokens in the pass must be consecutive (a prefill chunk or
        one decode row) and in sequence order; ``token_ids`` (int32, on the
        device) are the tokens the rows produced.
        """
        n = len(slots)
        if n != len(layout.tok_fwd) or token_ids.numel() != n:
            raise ValueError("slots, layout and token_ids must describe the same tokens")
        runs = _runs(slots)
        for s, _i, k in runs:
            if s not in self.open_slots:
                raise ValueError(f"slot {s} is not open")
            if self.count[s] + self.queued[s] + k > self.max_tokens:
                raise ValueError(f"slot {s} exceeds max_tokens")
        for s, _i, k in runs:
            self.queued[s] += k
        self.pending.append(_Pass([int(s) for s in slots], layout, token_ids))
        self.n_pending += n
        if self.n_pending >= self.defer_tokens:
            self.flush()

    def flush(self) -> None:
        """Hash every queued pass: leaves in one launch, each request's IO chain
        extended by its queued tokens in order, histories updated."""
        if not self.pending:
            return
        ctx = self.ctx
        passes, self.pending = self.pending, []
        self.n_pending = 0
        layout = passes[0].layout if len(passes) == 1 else _merge_layouts(ctx, passes)
        slots = [s for p in passes for s in p.slots]
        n = len(slots)
        leaves = C.trace_leaves(ctx, layout)
        # slot-major order (each request's tokens in pass order) for the IO chains
        first_seen: Dict[int, int] = {}
        for i, s in enumerate(slots):
            first_seen.setdefault(s, i)
        order = sorted(range(n), key=lambda i: (first_seen[slots[i]], i))
        runs = _runs([slots[i] for i in order])
        with torch.cuda.stream(ctx.stream):
            tok = torch.cat([p.token_ids.reshape(-1).to(torch.int32) for p in passes]) if len(passes) > 1 \
                else passes[0].token_ids.reshape(-1).to(torch.int32)
            if order != list(range(n)):
                o = torch.tensor(order, dtype=torch.long).to(leaves.device, non_blocking=True)
                leaves = leaves[:n].index_select(0, o)
                tok = tok.index_select(0, o)
            tok = tok.contiguous()
            idx = torch.tensor([r[0] for r in runs], dtype=torch.long, device=self.prev.device)
            prev = self.prev.index_select(0, idx).contiguous()
        step_io = ctx.empty(n, 32)
        tok_off = [r[1] for r in runs] + [n]
        check(lib().vc_io_extend(ctx.handle, len(runs), C._i64(tok_off), ctypes.c_void_p(leaves.data_ptr()),
                                 ctypes.c_void_p(tok.data_ptr()), ctypes.c_void_p(prev.data_ptr()),
                                 ctypes.c_void_p(step_io.data_ptr())))
        # each token's place in its request's history: one indexed scatter per buffer
        row, col = [], []
        for s, _i, k in runs:
            row += [s] * k
            col += range(self.count[s], self.count[s] + k)
        with torch.cuda.stream(ctx.stream):
            self.prev.index_copy_(0, idx, prev)
            r = torch.tensor(row, dtype=torch.long).to(self.leaves.device, non_blocking=True)
            c = torch.tensor(col, dtype=torch.long).to(self.leaves.device, non_blocking=True)
            self.leaves[r, c] = leaves[:n]
            self.io[r, c] = step_io
        for s, _i, k in runs:
            self.count[s] += k
            self.queued[s] -= k

    def close(self, slot: int) -> dict:
        """Finish a request: build its trace and IO trees (flushing queued passes
        first).  Returns device digests (``merkle_root``, ``io_root``,
        ``prompt_hash``, ``seed_commitment``) and ``n_tokens``; the slot can be
        reopened afterwards."""
        if slot not in self.open_slots:
            raise ValueError(f"slot {slot} is not open")
        if self.queued[slot]:
            self.flush()
        n = self.count[slot]
        if n == 0:
            raise ValueError("need at least one leaf")
        ctx = self.ctx
        with torch.cuda.stream(ctx.stream):
            both = torch.empty(2 * n, 32, dtype=torch.uint8, device=self.leaves.device)
            both[:n].copy_(self.leaves[slot, :n])
            both[n:].copy_(self.io[slot, :n])
        roots, _ = C.build_trees(ctx, both, [0, n, 2 * n], keep_trees=False)
        meta = self.open_slots.pop(slot)
        return {"merkle_root": roots[0], "io_root": roots[1], "prompt_hash": meta["prompt_hash"][0],
                "seed_commitment": meta["seed_commitment"][0], "n_tokens": n,
                "n_prompt_tokens": meta["n_prompt_tokens"], "_keep": both}
