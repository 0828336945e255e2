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


def _row_major(plan: List[Shard], n_seqs: int, n_layers: int) -> bool:
    """True when the shards, concatenated in rank order, are the (sequence,
    layer) grid in row-major order: then the gathered buffer needs no reordering."""
    return tree_order(plan, n_layers) == [(s, l) for s in range(n_seqs) for l in range(n_layers)]


def gather_roots(local: torch.Tensor, plan: List[Shard], n_seqs: int, n_layers: int,
                 group=None) -> torch.Tensor:
    """All-gather every rank's ``[n_trees_r, 32]`` roots into ``[n_seqs, n_layers, 32]``.

    Ranks hold different tree counts; each contributes a buffer padded to the
    largest shard, so one all_gather_into_tensor suffices.
    """
    world = len(plan)
    width = max(sh.n_trees for sh in plan)
    rank = dist.get_rank(group)
    uniform = all(sh.n_trees == width for sh in plan) and _row_major(plan, n_seqs, n_layers)
    if uniform:
        buf = local.reshape(-1, 32).contiguous()
    else:
        buf = torch.zeros(width, 32, dtype=torch.uint8, device=local.device)
        buf[: plan[rank].n_trees].copy_(local.reshape(-1, 32))
    out = torch.empty(world * width, 32, dtype=torch.uint8, device=local.device)
    dist.all_gather_into_tensor(out, buf, group=group)
    if uniform:
        # shard_plan's shards tile the (sequence, layer) grid in row-major order, so
        # without padding the gathered concatenation already is the result
        return out.view(n_seqs, n_layers, 32)
    full = torch.empty(n_seqs, n_layers, 32, dtype=torch.uint8, device=local.device)
    for r, sh in enumerate(plan):
        got = out[r * width: r * width + sh.n_trees].view(sh.seq_end - sh.seq_begin, sh.layer_end - sh.layer_begin, 32)
        full[sh.seq_begin:sh.seq_end, sh.layer_begin:sh.layer_end].copy_(got)
    return full


# ---------------------------------------------------------------------------
# Split trees: one request's per-layer trees spread over the ranks by position
# ---------------------------------------------------------------------------

@dataclass(frozen=True)
class SplitRange:
    """Rank ``rank``'s part of a tree of ``n_leaves`` positions split over
    ``world`` ranks: positions ``[begin, begin + count)`` (``count`` may be 0
    past the end), inside the aligned subtree of ``2**sub_log2`` leaves that
    starts at ``begin``; ``top_log2`` levels sit above the subtrees."""
    rank: int
    begin: int
    count: int
    sub_log2: int
    top_log2: int


def split_ranges(n_leaves: int, world: int) -> List[SplitRange]:
    """Aligned power-of-two position ranges of ``n_pad / world`` leaves.

    ``build_tree`` (merkle.rs:11-48) pads only level 0 with zero leaves, so the
    tree over ``n_pad = next_pow2(n_leaves)`` leaves is the ``world`` subtrees
    of ``n_pad / world`` leaves with ``log2 world`` levels of ``hash_pair`` on
    top.  ``world`` must be a power of two no larger than ``n_pad``.
    """
    if n_leaves < 1:
        raise ValueError("a tree needs at least one leaf")
    if world < 1 or world & (world - 1):
        raise ValueError("the number of ranks must be a power of two")
    lp = (n_leaves - 1).bit_length()
    top = (world - 1).bit_length()
    if top > lp:
        raise ValueError(f"{world} ranks exceed the {1 << lp} padded leaves of the tree")
    sub = lp - top
    size = 1 << sub
    return [SplitRange(r, r * size, max(0, min(size, n_leaves - r * size)), sub, top) for r in range(world)]


def split_view(view, rng: SplitRange):
    """``view`` (this rank's rows of one sequence, local row 0 = position
    ``rng.begin``) with the subtree fields set for ``commit.kv_commit``."""
    from dataclasses import replace
    return replace(view, seq_lens=[rng.count], pos_base=[rng.begin], tree_log2=rng.sub_log2)


def combine_subtree_roots(ctx, gathered: torch.Tensor, n_layers: int, keep_trees: bool = False):
    """Top levels of split trees: ``gathered`` is ``[world, n_layers, 32]``
    (rank r's subtree roots); per layer, ``build_tree`` over the ``world``
    subtree roots gives the layer's kv_root.  Returns ``(roots [n_layers, 32], top trees or None)``."""
    from . import commit as C
    world = gathered.shape[0]
    leaves = gathered.permute(1, 0, 2).contiguous().view(-1, 32)      # [layer][rank]
    return C.build_trees(ctx, leaves, [l * world for l in range(n_layers + 1)], keep_trees=keep_trees)


def split_kv_commit(ctx, view, rng: SplitRange, n_layers: int, group=None, keep_trees: bool = False):
    """Commit this rank's subtrees and exchange them: every rank gets the
    request's ``kv_roots`` ``[n_layers, 32]``, equal to a single-GPU commit.

    ``view`` holds this rank's rows (one sequence).  Returns
    ``(kv_roots, local subtree TreeSet or None, top TreeSet or None)``.
    """
    from . import commit as C
    if rng.count == 0 and rng.sub_log2 == 0:
        # a single zero padding leaf (build_tree pads level 0 with [0; 32])
        with torch.cuda.stream(ctx.stream):
            local = torch.zeros(n_layers, 32, dtype=torch.uint8, device=f"cuda:{ctx.device}")
        trees = None
    else:
        local, trees = C.kv_commit(ctx, split_view(view, rng), keep_trees=keep_trees)
    with torch.cuda.stream(ctx.stream):
        gathered = gather_subtree_roots(local, n_layers, group)
    roots, top = combine_subtree_roots(ctx, gathered, n_layers, keep_trees=keep_trees)
    return roots, trees, top


def gather_subtree_roots(local: torch.Tensor, n_layers: int, group=None) -> torch.Tensor:
    """The exchange of split trees: every rank's ``[n_layers, 32]`` subtree
    roots, all-gathered into ``[world, n_layers, 32]`` in rank (= position) order."""
    world = dist.get_world_size(group)
    out = torch.empty(world * n_layers, 32, dtype=torch.uint8, device=local.device)
    dist.all_gather_into_tensor(out, local.reshape(-1, 32).contiguous(), group=group)
    return out.view(world, n_layers, 32)
