"""A bounded device wait that runs out: the failure path every waiting kernel
of this library shares (kv_transcript_kernel, kvt_commit_kernel,
trace_leaf_split_kernel).  The probe's wait on an mbarrier that nothing
arrives at gives up after its limit and flags the context; the host sees
VC_ETIMEDOUT at the next sync, the flag is cleared, and the context commits
correctly afterwards.  No GPU fault, trap or hang is involved."""
import numpy as np
import pytest

from commitllm_b200 import commit as C
from oracle import commit_oracle as O

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_stays_usable(ctx):
    C.wait_probe(ctx, 50_000_000)          # 50 ms
    with pytest.raises(Exception, match="bounded wait"):
        ctx.sync(20000)
    ctx.sync(20000)                        # the flag was cleared
    # the same context still commits correctly
    rng = np.random.default_rng(5)
    leaves = [rng.integers(0, 256, 32, dtype=np.uint8).tobytes() for _ in range(37)]
    dev = ctx.to_device(np.frombuffer(b"".join(leaves), dtype=np.uint8).reshape(37, 32))
    roots, trees = C.build_trees(ctx, dev, [0, 37], keep_trees=True)
    ctx.sync(20000)
    assert bytes(roots[0].cpu().numpy()) == O.build_tree(leaves).root
    trees.free()


def test_wait_probe_rejects_unbounded_limits(ctx):
    with pytest.raises(Exception):
        C.wait_probe(ctx, 0)
    with pytest.raises(Exception):
        C.wait_probe(ctx, 3_000_000_000)
