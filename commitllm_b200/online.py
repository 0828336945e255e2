"""Online (per decode step) commitment of a batch of requests.

The reference commits once, after generation (``commit_minimal``,
crates/verilm-prover/src/lib.rs:336-499): trace leaves for every token, the
serial IO chain, then the trace and IO trees.  Here the same values are built
step by step while the requests decode: after each forward pass, the new
tokens' retained-state leaves are hashed and each request's IO chain is
extended by its new tokens on the GPU; closing a request builds its two trees.
The roots equal the offline commit of the same captures, bit for bit, so the
receipts are unchanged -- only the time at which the hashing happens moves
(into the decode loop, overlapped with it, instead of after it).
"""
from __future__ import annotations

import ctypes
from typing import Dict, Optional, Sequence

import numpy as np
import torch

from . import commit as C
from ._lib import check, lib


class OnlineCommitter:
    """Per-request histories of trace leaves and IO values, held on the device.

    ``max_slots`` requests can be open at once, each with at most
    ``max_tokens`` committed tokens (``token_ids = all_ids[1:]`` in the
    reference, i.e. one per forward-pass row).
    """

    def __init__(self, ctx: C.Context, max_slots: int, max_tokens: int):
        self.ctx = ctx
        self.max_slots, self.max_tokens = int(max_slots), int(max_tokens)
        self.leaves = ctx.empty(self.max_slots, self.max_tokens, 32)
        self.io = ctx.empty(self.max_slots, self.max_tokens, 32)
        self.prev = ctx.empty(self.max_slots, 32)
        self.count = [0] * self.max_slots
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
        runs = []          # (slot, first token in this pass, count)
        for i, s in enumerate(slots):
            s = int(s)
            if s not in self.open_slots:
                raise ValueError(f"slot {s} is not open")
            if runs and runs[-1][0] == s:
                runs[-1][2] += 1
            else:
                if any(r[0] == s for r in runs):
                    raise ValueError(f"tokens of slot {s} are not consecutive")
                runs.append([s, i, 1])
        for s, _i, k in runs:
            if self.count[s] + k > self.max_tokens:
                raise ValueError(f"slot {s} exceeds max_tokens")
        ctx = self.ctx
        step_leaves = C.trace_leaves(ctx, layout)
        # the active requests' chains, compacted in pass order
        step_io = ctx.empty(n, 32)
        tok_off = [r[1] for r in runs] + [n]
        with torch.cuda.stream(ctx.stream):
            idx = torch.tensor([r[0] for r in runs], dtype=torch.long, device=self.prev.device)
            prev = self.prev.index_select(0, idx).contiguous()
            tok = token_ids.to(torch.int32).contiguous()
        check(lib().vc_io_extend(ctx.handle, len(runs), C._i64(tok_off), ctypes.c_void_p(step_leaves.data_ptr()),
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
            self.leaves[r, c] = step_leaves[:n]
            self.io[r, c] = step_io
        for s, _i, k in runs:
            self.count[s] += k

    def close(self, slot: int) -> dict:
        """Finish a request: build its trace and IO trees.  Returns device digests
        (``merkle_root``, ``io_root``, ``prompt_hash``, ``seed_commitment``) and
        ``n_tokens``; the slot can be reopened afterwards."""
        if slot not in self.open_slots:
            raise ValueError(f"slot {slot} is not open")
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
