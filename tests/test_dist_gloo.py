"""Sharding and the root exchange across ranks, on CPU with gloo (world size 2-4).

Each rank computes its shard's kv_roots with the oracle (the stand-in for
the GPU commit in this CPU test), the ranks all-gather them through
``commitllm_b200.dist.gather_roots``, and every rank must end up with the
single-process roots in (sequence, layer) order and the same root-of-roots.
A rank that fails before the exchange makes the others fail fast (short
process-group timeout) instead of hanging.
"""
import multiprocessing as mp
import os
import socket
import traceback

import numpy as np
import pytest

from commitllm_b200 import dist as D


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_plan_covers_every_tree_once():
    for S, L, W in [(1, 32, 1), (1, 32, 2), (1, 32, 8), (3, 5, 4), (32, 80, 8), (4, 80, 8), (5, 2, 3), (2, 3, 8)]:
        plan = D.shard_plan(S, L, W)
        assert len(plan) == W
        seen = D.tree_order(plan, L)
        assert sorted(seen) == [(s, l) for s in range(S) for l in range(L)]
        assert len(seen) == len(set(seen))


def test_uniform_shard_plans_are_row_major():
    """gather_roots returns the gathered buffer as is when every shard has the
    same size: those plans must tile (sequence, layer) in row-major order."""
    for S, L, W in [(1, 32, 8), (8, 4, 4), (32, 80, 8), (2, 6, 4), (4, 80, 8), (1, 32, 2)]:
        plan = D.shard_plan(S, L, W)
        if all(sh.n_trees == plan[0].n_trees for sh in plan):
            assert D.tree_order(plan, L) == [(s, l) for s in range(S) for l in range(L)]


def _worker(rank, world, port, S, L, fail_rank, q, plan=None):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import datetime

        import torch
        import torch.distributed as dist
        from tests import kvref
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
        plan = plan or D.shard_plan(S, L, world)
        sh = plan[rank]
        tr = kvref.contiguous(55, L, [9 + 3 * s for s in range(S)], 2, 8)
        if rank == fail_rank:
            raise RuntimeError("injected failure before the exchange")
        # this rank's shard: sequences [b, e), layers [lb, le)
        roots_all, _ = tr.oracle(n_threads=1, with_nodes=False)
        local = torch.from_numpy(np.ascontiguousarray(roots_all[sh.seq_begin:sh.seq_end, sh.layer_begin:sh.layer_end]))
        full = D.gather_roots(local.reshape(-1, 32), plan, S, L)
        from oracle import commit_oracle as O
        ror = O.compute_root([bytes(x) for x in full.reshape(-1, 32).numpy()])
        q.put((rank, "ok", bytes(full.numpy().tobytes()), ror, bytes(roots_all.tobytes())))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        q.put((rank, "err", f"{type(e).__name__}: {e}", traceback.format_exc(), None))


def _run(world, S, L, fail_rank=-1, timeout=120, plan=None):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, S, L, fail_rank, q, plan)) for r in range(world)]
    for p in ps:
        p.start()
    out = []
    for _ in range(world):
        out.append(q.get(timeout=timeout))
    for p in ps:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return sorted(out, key=lambda x: x[0])


@pytest.mark.parametrize("world,S,L", [(2, 1, 6), (2, 3, 4), (4, 2, 5)])
def test_gather_roots_reassembles_single_process_roots(world, S, L):
    res = _run(world, S, L)
    assert all(r[1] == "ok" for r in res), res
    want = res[0][4]
    for r in res:
        assert r[2] == want              # every rank holds every kv_root, in order
        assert r[3] == res[0][3]         # and the same root-of-roots


def test_gather_roots_equal_shards_in_another_order():
    """A caller's plan with equal shards that do not tile the grid row-major
    (2 sequences x 4 ranks, each sequence's layers in halves, sequences
    interleaved) must still come back in (sequence, layer) order."""
    S, L = 2, 4
    plan = [D.Shard(0, 1, 0, 2), D.Shard(1, 2, 0, 2), D.Shard(0, 1, 2, 4), D.Shard(1, 2, 2, 4)]
    assert D.tree_order(plan, L) != [(s, l) for s in range(S) for l in range(L)]
    res = _run(4, S, L, plan=plan)
    assert all(r[1] == "ok" for r in res), res
    for r in res:
        assert r[2] == res[0][4]
        assert r[3] == res[0][3]


def test_failed_rank_does_not_hang_the_others():
    res = _run(2, 2, 2, fail_rank=1, timeout=180)
    assert res[1][1] == "err" and "injected" in res[1][2]
    assert res[0][1] == "err"            # rank 0's collective ended with an error, not a hang


def _split_worker(rank, world, port, n, L, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import datetime

        import torch
        import torch.distributed as dist
        from oracle import commit_oracle as O
        from tests import kvref
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
        rng = D.split_ranges(n, world)[rank]
        tr = kvref.contiguous(77, L, [n], 2, 8)
        kf = [O.bf16_to_f64(tr.k[l].reshape(n, -1)) for l in range(L)]
        vf = [O.bf16_to_f64(tr.v[l].reshape(n, -1)) for l in range(L)]
        local = np.zeros((L, 32), np.uint8)
        for l in range(L):
            # this rank's subtree: its leaves, zero leaves past the end (the GPU commit in production)
            lv = [O.hash_kv_entry(l, rng.begin + i, kf[l][rng.begin + i], vf[l][rng.begin + i]) if i < rng.count
                  else bytes(32) for i in range(1 << rng.sub_log2)]
            while len(lv) > 1:
                lv = [O.hash_pair(lv[2 * i], lv[2 * i + 1]) for i in range(len(lv) // 2)]
            local[l] = np.frombuffer(lv[0], np.uint8)
        gathered = D.gather_subtree_roots(torch.from_numpy(local), L).numpy()
        roots = [O.build_tree([bytes(gathered[r, l]) for r in range(world)]).root for l in range(L)]
        full = [O.kv_tree_for_layer(l, kf[l], vf[l]).root for l in range(L)]
        q.put((rank, "ok", roots == full, None))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, "err", f"{type(e).__name__}: {e}", traceback.format_exc()))


@pytest.mark.parametrize("world,n", [(2, 37), (4, 100), (4, 9)])
def test_split_tree_exchange_gives_single_process_roots(world, n):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_split_worker, args=(r, world, port, n, 3, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = sorted((q.get(timeout=120) for _ in range(world)), key=lambda x: x[0])
    for p in ps:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert all(r[1] == "ok" and r[2] is True for r in res), res
