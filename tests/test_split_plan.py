"""Split-tree arithmetic on the CPU: build_tree over all leaves equals the
subtrees of the aligned ranges with build_tree over their roots on top."""
import hashlib

import numpy as np
import pytest

from commitllm_b200 import dist as D
from oracle import commit_oracle as O


def subtree_root(leaves, begin, count, sub_log2):
    """Root of the 2^sub_log2-leaf subtree starting at begin (zero leaves past the end)."""
    lv = [leaves[begin + i] if i < count else bytes(32) for i in range(1 << sub_log2)]
    while len(lv) > 1:
        lv = [O.hash_pair(lv[2 * i], lv[2 * i + 1]) for i in range(len(lv) // 2)]
    return lv[0]


@pytest.mark.parametrize("n", [1, 2, 3, 5, 8, 37, 300, 1000, 1025])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_split_equals_build_tree(n, world):
    pad = 1 << (n - 1).bit_length()
    if world > pad:
        with pytest.raises(ValueError):
            D.split_ranges(n, world)
        return
    leaves = [hashlib.sha256(b"leaf %d" % i).digest() for i in range(n)]
    ranges = D.split_ranges(n, world)
    assert sum(r.count for r in ranges) == n
    assert all(r.begin == r.rank << r.sub_log2 for r in ranges)
    roots = [subtree_root(leaves, r.begin, r.count, r.sub_log2) for r in ranges]
    assert O.build_tree(roots).root == O.build_tree(leaves).root
    # ranges past the end are the padding constants Z_k
    z = O.zero_subtree_roots(ranges[0].sub_log2)
    for r, root in zip(ranges, roots):
        if r.count == 0:
            assert root == z[r.sub_log2]
