"""Online per-step commitment (commitllm_b200.online) equals the offline commit.

A continuous batch: requests prefill in chunks, decode one token per step,
join and leave at different steps; logits bind only to generated tokens.
Each request's merkle_root / io_root / prompt hash / seed commitment must
equal commit_minimal's (the oracle's) over the same captures.
"""
import numpy as np
import pytest
import torch

from commitllm_b200 import commit as C
from commitllm_b200.online import OnlineCommitter
from oracle import commit_oracle as O
from tests import synth

pytestmark = pytest.mark.gpu

L, H, V = 3, 40, 97


@pytest.mark.parametrize("defer,ring", [(0, False), (3, False), (1000, False), (1000, True)])
def test_online_equals_offline(ctx, defer, ring):
    """ring: every pass writes its logits into one shared tensor (read in place at flush)."""
    schedule = [  # per step: list of (slot, rows)
        [(0, 3), (1, 2)],
        [(0, 1), (1, 1)],
        [(0, 1), (1, 1), (2, 4)],
        [(1, 1), (2, 1)],
        [(2, 1)],
    ]
    closes = {2: [0], 3: [1], 4: [2]}            # slots closed after a step
    prompts = {0: b"alpha", 1: b"", 2: b"gamma prompt"}
    n_prompt = {0: 3, 1: 2, 2: 4}
    oc = OnlineCommitter(ctx, max_slots=4, max_tokens=16, defer_tokens=defer)
    held = []                                     # deferred passes are read at flush: keep captures alive
    hist = {s: [] for s in prompts}               # per slot: (a [L,H], scales [L], logits or None, token)
    results = {}
    rng = np.random.default_rng(5)
    ring_t = ctx.empty(64, V, dtype=torch.float32) if ring else None
    ring_used = 0
    for k, rows in enumerate(schedule):
        for s, _ in rows:
            if s not in oc.open_slots and not hist[s]:
                oc.open(s, prompts[s], bytes([s]) * 32, n_prompt_tokens=n_prompt[s])
        n = sum(r for _, r in rows)
        a = rng.integers(-128, 128, size=(L, n, H), dtype=np.int8)
        sc = rng.random((L, n), dtype=np.float32)
        toks = rng.integers(0, 1000, size=n).astype(np.int32)
        slots, logit_rows, logits = [], [], []
        i = 0
        for s, r in rows:
            for j in range(r):
                pos = len(hist[s])                          # this token's index in its request
                gen = pos >= n_prompt[s] - 1                # gen_start = n_prompt_tokens - 1
                lg = rng.standard_normal(V).astype(np.float32) if gen else None
                logit_rows.append(len(logits) if gen else -1)
                if gen:
                    logits.append(lg)
                hist[s].append((a[:, i].copy(), sc[:, i].copy(), lg, int(toks[i])))
                slots.append(s)
                i += 1
        ad, sd = ctx.to_device(a), ctx.to_device(sc)
        held.append((ad, sd))
        ld = ctx.to_device(np.stack(logits)) if logits else None
        if ring and ld is not None:
            ring_t[ring_used:ring_used + ld.shape[0]].copy_(ld)
            logit_rows = [r + ring_used if r >= 0 else -1 for r in logit_rows]
            ring_used += ld.shape[0]
            ld = ring_t
        lay = C.TraceLayout(n_layers=L, hidden=H, fwd_rows=[n], tok_fwd=[0] * n, tok_row=list(range(n)),
                            a_rows=[[ad.data_ptr() + l * n * H for l in range(L)]],
                            scale_a=[[sd.data_ptr() + 4 * l * n for l in range(L)]], scale_stride=1,
                            logits=ld, tok_logits_row=logit_rows if ld is not None else None)
        oc.step(slots, lay, ctx.to_device(toks))
        for s in closes.get(k, []):
            results[s] = oc.close(s)
    ctx.sync(timeout_ms=60000)
    for s, r in results.items():
        retained = [[O.RetainedLayerState(h[0][l].tobytes(), float(h[1][l])) for l in range(L)] for h in hist[s]]
        gen_logits = [h[2] for h in hist[s] if h[2] is not None]
        com = O.commit_minimal(retained, [h[3] for h in hist[s]], prompts[s], bytes([s]) * 32,
                               captured_logits_f32=gen_logits, n_prompt_tokens=n_prompt[s])
        assert bytes(r["merkle_root"].cpu().numpy()) == com.merkle_root, s
        assert bytes(r["io_root"].cpu().numpy()) == com.io_root, s
        assert bytes(r["prompt_hash"].cpu().numpy()) == com.prompt_hash
        assert bytes(r["seed_commitment"].cpu().numpy()) == com.seed_commitment
        assert r["n_tokens"] == len(hist[s])


def test_online_rejects_bad_steps(ctx):
    oc = OnlineCommitter(ctx, max_slots=2, max_tokens=2)
    with pytest.raises(ValueError):
        oc.open(0, b"p", b"short")
    oc.open(0, b"p", b"\0" * 32)
    with pytest.raises(ValueError):
        oc.open(0, b"p", b"\0" * 32)            # already open
    a = ctx.to_device(np.zeros((1, 3, 4), np.int8))
    s = ctx.to_device(np.ones((1, 3), np.float32))
    lay = C.TraceLayout(n_layers=1, hidden=4, fwd_rows=[3], tok_fwd=[0] * 3, tok_row=[0, 1, 2],
                        a_rows=[[a.data_ptr()]], scale_a=[[s.data_ptr()]])
    with pytest.raises(ValueError):
        oc.step([0, 0, 0], lay, ctx.to_device(np.zeros(3, np.int32)))   # exceeds max_tokens
    with pytest.raises(ValueError):
        oc.step([0, 1, 0], lay, ctx.to_device(np.zeros(3, np.int32)))   # slot 1 not open


def test_deferred_default_with_a_capture_ring(ctx):
    """The capture-lifetime contract of deferred mode: a decode loop that reuses
    ceil(defer_tokens / tokens per pass) capture buffers in a ring never has one
    overwritten before the flush that reads it, so the roots equal the offline
    commit; the default committer (DEFAULT_DEFER_TOKENS) defers every pass."""
    from commitllm_b200 import online
    assert OnlineCommitter(ctx, max_slots=1, max_tokens=1).defer_tokens == online.DEFAULT_DEFER_TOKENS > 0
    B, steps, defer = 4, 11, 12                  # 3 passes per flush
    depth = -(-defer // B)
    oc = OnlineCommitter(ctx, max_slots=B, max_tokens=steps, defer_tokens=defer)
    for s in range(B):
        oc.open(s, b"ring %d" % s, bytes([s + 1]) * 32, n_prompt_tokens=1)
    ring_a = [ctx.empty(L, B, H, dtype=torch.int8) for _ in range(depth)]
    ring_s = [ctx.empty(L, B, dtype=torch.float32) for _ in range(depth)]
    ring_l = ctx.empty(depth * B, V, dtype=torch.float32)   # logits rows of the ring's passes
    rng = np.random.default_rng(11)
    hist = {s: [] for s in range(B)}
    for k in range(steps):
        slot = k % depth
        a = rng.integers(-128, 128, size=(L, B, H), dtype=np.int8)
        sc = rng.random((L, B), dtype=np.float32)
        lg = rng.standard_normal((B, V)).astype(np.float32)
        toks = rng.integers(0, 1000, size=B).astype(np.int32)
        with torch.cuda.stream(ctx.stream):
            ring_a[slot].copy_(torch.from_numpy(a))
            ring_s[slot].copy_(torch.from_numpy(sc))
            ring_l[slot * B:(slot + 1) * B].copy_(torch.from_numpy(lg))
        for s in range(B):
            hist[s].append((a[:, s].copy(), sc[:, s].copy(), lg[s].copy(), int(toks[s])))
        lay = C.TraceLayout(n_layers=L, hidden=H, fwd_rows=[B], tok_fwd=[0] * B, tok_row=list(range(B)),
                            a_rows=[[ring_a[slot].data_ptr() + l * B * H for l in range(L)]],
                            scale_a=[[ring_s[slot].data_ptr() + 4 * l * B for l in range(L)]], scale_stride=1,
                            logits=ring_l, tok_logits_row=[slot * B + s for s in range(B)])
        oc.step(list(range(B)), lay, ctx.to_device(toks))
    res = {s: oc.close(s) for s in range(B)}
    ctx.sync(timeout_ms=60000)
    for s in range(B):
        retained = [[O.RetainedLayerState(h[0][l].tobytes(), float(h[1][l])) for l in range(L)] for h in hist[s]]
        com = O.commit_minimal(retained, [h[3] for h in hist[s]], b"ring %d" % s, bytes([s + 1]) * 32,
                               captured_logits_f32=[h[2] for h in hist[s]], n_prompt_tokens=1)
        assert bytes(res[s]["merkle_root"].cpu().numpy()) == com.merkle_root
        assert bytes(res[s]["io_root"].cpu().numpy()) == com.io_root
