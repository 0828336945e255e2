"""Sharding the KV commitment across GPUs and the root-of-roots exchange.

Trees are independent per (sequence, layer) -- the reference builds one per
layer of each request (crates/verilm-prover/src/lib.rs:449-482) -- so each
rank commits its own shard with no communication.  The one exchange step is
an all-gather of the 32-byte roots (NCCL over NVLink), after which every
rank holds every request's ``kv_roots`` and, as an additive extension the
reference does not have, the root-of-roots: ``build_tree`` over all gathered
roots in (sequence, layer) order.

Shard plan: sequences are dealt to ranks in contiguous ranges; with fewer
sequences than ranks, each sequence's layers are split into contiguous
layer ranges across the ranks that share it.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Tuple

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class Shard:
    seq_begin: int
    seq_end: int
    layer_begin: int
    layer_end: int

    @property
    def n_trees(self) -> int:
        return (self.seq_end - self.seq_begin) * (self.layer_end - self.layer_begin)


def shard_plan(n_seqs: int, n_layers: int, world: int) -> List[Shard]:
    """Split (sequence, layer) trees over ``world`` ranks, sequence-major."""
    if n_seqs < 1 or n_layers < 1 or world < 1:
        raise ValueError("n_seqs, n_layers and world must be >= 1")
    out = []
    if world <= n_seqs:
        for r in range(world):
            b = n_seqs * r // world
            e = n_seqs * (r + 1) // world
            out.append(Shard(b, e, 0, n_layers))
        return out
    # more ranks than sequences: ranks_per_seq ranks share each sequence's layers
    for r in range(world):
        s = r * n_seqs // world
        first = -(-s * world // n_seqs)             # first rank of sequence s
        last = -(-(s + 1) * world // n_seqs)        # one past its last rank
        k, m = r - first, last - first
        lb = n_layers * k // m
        le = n_layers * (k + 1) // m
        out.append(Shard(s, s + 1, lb, le))
    return out


def tree_order(plan: List[Shard], n_layers: int) -> List[Tuple[int, int]]:
    """(sequence, layer) of each tree in the concatenation of all ranks' shards."""
    order = []
    for sh in plan:
        for s in range(sh.seq_begin, sh.seq_end):
            for l in range(sh.layer_begin, sh.layer_end):
                order.append((s, l))
    return order


def gather_roots(local: torch.Tensor, plan: List[Shard], n_seqs: int, n_layers: int,
                 group=None) -> torch.Tensor:
    """All-gather every rank's ``[n_trees_r, 32]`` roots into ``[n_seqs, n_layers, 32]``.

    Ranks hold different tree counts; each contributes a buffer padded to the
    largest shard, so one all_gather_into_tensor suffices.
    """
    world = len(plan)
    width = max(sh.n_trees for sh in plan)
    rank = dist.get_rank(group)
    buf = torch.zeros(width, 32, dtype=torch.uint8, device=local.device)
    buf[: plan[rank].n_trees].copy_(local.reshape(-1, 32))
    out = torch.empty(world * width, 32, dtype=torch.uint8, device=local.device)
    dist.all_gather_into_tensor(out, buf, group=group)
    full = torch.empty(n_seqs, n_layers, 32, dtype=torch.uint8, device=local.device)
    for r, sh in enumerate(plan):
        got = out[r * width: r * width + sh.n_trees].view(sh.seq_end - sh.seq_begin, sh.layer_end - sh.layer_begin, 32)
        full[sh.seq_begin:sh.seq_end, sh.layer_begin:sh.layer_end].copy_(got)
    return full
