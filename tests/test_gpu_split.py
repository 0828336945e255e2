"""Split trees: one request's per-layer KV trees spread over ranks by aligned
power-of-two position ranges (each rank commits its subtrees; the gathered
subtree roots give the top levels).  Emulated here on one GPU, rank by rank:
roots, node arrays and proofs must equal the single-GPU commit bit for bit."""
from dataclasses import replace

import numpy as np
import pytest
import torch

from commitllm_b200 import commit as C
from commitllm_b200 import dist as D
from tests import kvref

pytestmark = pytest.mark.gpu


def level_off(lp, k):
    return sum(1 << (lp - j) for j in range(k))


def rank_commit(ctx, view, rng, n_layers, keep_trees=True, paged=False):
    if rng.count == 0 and rng.sub_log2 == 0:
        return torch.zeros(n_layers, 32, dtype=torch.uint8, device="cuda"), None
    if paged:
        # this rank's pages: its own block-table row, starting at page begin / block
        bs = view.k_layers[0].shape[1]
        bt = view.block_tables[:, rng.begin // bs:].contiguous()
        rv = replace(view, block_tables=bt, seq_lens=[rng.count], pos_base=[rng.begin], tree_log2=rng.sub_log2)
    else:
        rv = replace(view, seq_row_offset=[rng.begin], seq_lens=[rng.count], pos_base=[rng.begin],
                     tree_log2=rng.sub_log2)
    roots, trees = C.kv_commit(ctx, rv, keep_trees=keep_trees)
    return roots[0], trees


CASES = [(4096, 8), (5000, 8), (37, 4), (300, 2), (3, 2), (8, 8), (5, 8), (1000, 1)]


@pytest.mark.parametrize("n,world", CASES)
def test_split_trees_equal_single_gpu(ctx, n, world):
    L, nh, hd = 3, 2, 64
    tr = kvref.contiguous(n * 7 + world, L, [n], nh, hd)
    view = tr.view()
    full, full_trees = C.kv_commit(ctx, view, keep_trees=True)
    ranges = D.split_ranges(n, world)
    local, trees = [], []
    for rng in ranges:
        r, t = rank_commit(ctx, view, rng, L)
        local.append(r)
        trees.append(t)
    roots, top = D.combine_subtree_roots(ctx, torch.stack(local), L, keep_trees=True)
    ctx.sync(30000)
    assert torch.equal(roots.cpu(), full[0].cpu())
    lp = (n - 1).bit_length()
    sub = ranges[0].sub_log2
    for l in range(L):
        fn = full_trees.nodes(l).cpu()
        for rng, t in zip(ranges, trees):
            if t is None:
                continue
            tn = t.nodes(l).cpu()
            for k in range(sub + 1):
                lo = level_off(lp, k) + (rng.begin >> k)
                assert torch.equal(tn[level_off(sub, k):level_off(sub, k) + (1 << (sub - k))],
                                   fn[lo:lo + (1 << (sub - k))]), (l, rng.rank, k)
    # proofs: the local subtree's siblings, then the top tree's, equal merkle::prove on the full tree
    rng_ = np.random.default_rng(n)
    for p in sorted(set(rng_.integers(0, n, 6).tolist() + [0, n - 1])):
        r = p >> sub
        l = int(rng_.integers(0, L))
        want, _ = full_trees.prove([l], [p])
        parts = []
        if trees[r] is not None and sub > 0:
            s, _ = trees[r].prove([l], [p - ranges[r].begin])
            parts.append(s[0].cpu())
        if world > 1:
            s, _ = top.prove([l], [r])
            parts.append(s[0].cpu())
        got = torch.cat(parts) if parts else torch.zeros(0, 32, dtype=torch.uint8)
        assert torch.equal(got, want[0].cpu()), (p, l)


def test_split_trees_paged(ctx):
    n, world, L = 1000, 4, 2
    tr = kvref.paged(11, L, [n], 2, 64, block_size=16)
    view = tr.view()
    full, _ = C.kv_commit(ctx, view, keep_trees=False)
    ranges = D.split_ranges(n, world)      # 256-position ranges, multiples of the 16-token block
    local = [rank_commit(ctx, view, rng, L, keep_trees=False, paged=True)[0] for rng in ranges]
    roots, _ = D.combine_subtree_roots(ctx, torch.stack(local), L)
    assert torch.equal(roots.cpu(), full[0].cpu())


def test_split_tree_validation(ctx):
    tr = kvref.contiguous(3, 1, [40], 2, 64)
    view = tr.view()
    with pytest.raises(ValueError):
        C.kv_commit(ctx, replace(view, tree_log2=5))                    # 40 leaves do not fit 2^5
    with pytest.raises(ValueError):
        C.kv_commit(ctx, replace(view, pos_base=[(1 << 32) - 10]))      # positions beyond u32
    with pytest.raises(ValueError):
        D.split_ranges(40, 3)
    with pytest.raises(ValueError):
        D.split_ranges(4, 8)
