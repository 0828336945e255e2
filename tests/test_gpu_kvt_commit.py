"""The transcript committed in one pass (vc_kv_transcript_commit) against the oracle
and against the two-call path (vc_kv_transcript, then vc_kv_commit of its f64 rows).

The one-pass kernel never stores the f64 K/V rows: each position's
hash_kv_entry message is absorbed as its channels leave the tensor cores.
Its kv_roots, and every node of every tree, must equal those of the oracle's
compute_kv_transcript + build_tree (crates/verilm-prover/src/lib.rs:207-329,
449-482) and of the two-call GPU path, bit for bit: shapes with head_dim 64 and
128 run fused, the others through the two-call fallback inside the entry.
"""
import numpy as np
import pytest
import torch

from commitllm_b200 import commit as C
from oracle import commit_oracle as O
from tests.test_gpu_kv_transcript import gpu_inputs, make_case, oracle_of

pytestmark = pytest.mark.gpu

CASES = [
    # n_tok, layers, hidden, kv heads, head_dim, mode        (fused when head_dim is 64 or 128)
    (150, 2, 256, 2, 64, "toy"),           # the toy clamp path, fused
    (5, 2, 16, 2, 2, "toy"),               # the reference's toy shape: two-call fallback
    (200, 2, 272, 2, 64, "tensor"),        # ragged positions, hidden not a multiple of 128
    (130, 3, 256, 4, 128, "channel_bias"),
    (64, 2, 128, 3, 96, "mixed"),          # head_dim 96: fallback
    (300, 1, 512, 8, 128, "tensor"),       # Llama kv_dim 1024
    (160, 2, 3584, 4, 128, "channel_bias"),  # Qwen2.5-7B shapes
    (129, 1, 8192, 8, 128, "tensor"),      # Llama-70B hidden
    (1, 2, 128, 8, 128, "tensor"),         # one position: the root is the leaf
    (7, 2, 128, 2, 64, "mixed"),           # a chunk smaller than 128 leaves
    (70, 1, 512, 2, 256, "channel_bias"),  # head_dim 256: fallback
]


@pytest.mark.parametrize("case", CASES, ids=[f"{c[-1]}-{c[0]}x{c[2]}-h{c[3]}x{c[4]}" for c in CASES])
def test_one_pass_roots_match_oracle_and_two_call_path(ctx, case):
    n_tok, L, hidden, nh, hd, mode = case
    c = make_case(n_tok * 1000 + hidden + nh * 7 + hd, n_tok, L, hidden, nh, hd, mode)
    k_ref, v_ref = oracle_of(c)
    inp, _keep = gpu_inputs(ctx, c, token_major=(n_tok % 2 == 0))
    base = 3
    roots, trees = C.kv_transcript_commit(ctx, inp, layer_base=base, keep_trees=True)
    k, v = C.kv_transcript(ctx, inp)
    roots2, trees2 = C.kv_commit(ctx, C.kv_transcript_view(k, v, layer_base=base), keep_trees=True)
    ctx.sync(60000)
    got = roots.cpu().numpy()
    assert np.array_equal(got, roots2.cpu().numpy().reshape(L, 32))
    for l in range(L):
        want = O.build_tree([O.hash_kv_entry(base + l, p, k_ref[l][p], v_ref[l][p]) for p in range(n_tok)])
        assert bytes(got[l]) == want.root, f"layer {l}"
        assert torch.equal(trees.nodes(l), trees2.nodes(l))
        assert [bytes(x) for x in trees.nodes(l).cpu().numpy()] == list(want.nodes)
    trees.free()
    trees2.free()


def test_one_pass_llama8b_full_size(ctx):
    """Llama-3-8B shapes, 4 096 positions x 32 layers, per-tensor scales, llama3 RoPE:
    every kv_root of the one-pass commit equals the two-call path's (which the
    tests above and test_gpu_kv_transcript pin to the oracle bit for bit)."""
    g = torch.Generator(device=f"cuda:{ctx.device}")
    g.manual_seed(4242)
    dev = f"cuda:{ctx.device}"
    T, L, H, nh, hd = 4096, 32, 4096, 8, 128
    kv = nh * hd
    with torch.cuda.stream(ctx.stream):
        x = torch.randint(-128, 128, (T, L, H), generator=g, device=dev, dtype=torch.int8)
        sx = torch.rand(T, L, generator=g, device=dev) * 0.05 + 1e-3
        wk = [torch.randint(-128, 128, (kv, H), generator=g, device=dev, dtype=torch.int8) for _ in range(L)]
        wv = [torch.randint(-128, 128, (kv, H), generator=g, device=dev, dtype=torch.int8) for _ in range(L)]
    inp = C.KvTranscriptInputs(x_attn=[x[:, l] for l in range(L)], wk=wk, wv=wv, scale_x=sx, n_kv_heads=nh,
                               head_dim=hd, per_tensor=[(0.0021 + 1e-5 * l, 0.0017 + 1e-5 * l) for l in range(L)],
                               rope=C.RopeConfig(theta=500000.0, scaling="llama3"))
    roots, _ = C.kv_transcript_commit(ctx, inp, keep_trees=False)
    k, v = C.kv_transcript(ctx, inp)
    roots2, _ = C.kv_commit(ctx, C.kv_transcript_view(k, v), keep_trees=False)
    ctx.sync(120000)
    assert torch.equal(roots, roots2.view(L, 32))


def test_one_pass_needs_a_position(ctx):
    c = make_case(9, 4, 1, 128, 2, 64, "tensor")
    inp, _ = gpu_inputs(ctx, c, token_major=False)
    inp.x_attn = [inp.x_attn[0][:0]]
    inp.scale_x = inp.scale_x[:0]
    from commitllm_b200._lib import VcValueError
    with pytest.raises(VcValueError, match="at least one position"):
        C.kv_transcript_commit(ctx, inp)
