"""Parity at the benchmark sizes.

* Llama-3.1-8B shape (32 layers x 8 x 128, 4096 tokens): all 32 kv_roots
  against the oracle's C restatement.
* Qwen2.5-7B shape, paged (28 layers x 4 x 128, 16 x 8192 tokens in permuted
  16-token pages): the paged commit equals the commit of the same rows
  gathered into a contiguous layout (a size-independent property); a few
  trees are checked against the oracle directly; 1024 random openings verify
  against their roots.
* Llama-3.1-70B sequence length (32 768 positions) and 32 769 (padded to
  65 536): kv_roots against the C oracle, openings at both ends verify.
"""
import numpy as np
import pytest
import torch

from commitllm_b200 import commit as C
from commitllm_b200._lib import VC_DTYPE_BF16
from oracle import commit_oracle as O
from tests import kvref, synth

pytestmark = pytest.mark.gpu


def test_llama8b_shape_kv_roots_match_oracle(ctx):
    L, H, D, N = 32, 8, 128, 4096
    k, v = synth.kv_rows_bf16(8, L, N, H, D)
    tr = kvref.Transcript(k, v, [N], VC_DTYPE_BF16)
    view = tr.view(ctx.device)
    roots, trees = C.kv_commit(ctx, view, keep_trees=True)
    ctx.sync(timeout_ms=120000)
    oroots, _ = tr.oracle(n_threads=32, with_nodes=False)
    assert np.array_equal(roots.cpu().numpy(), oroots)
    # a few full node arrays too
    for l in (0, 17, 31):
        ref = kvref.Transcript(k[l:l + 1], v[l:l + 1], [N], VC_DTYPE_BF16, layer_base=l).oracle(n_threads=1)[1][0]
        assert np.array_equal(trees.nodes(l).cpu().numpy(), ref)


def test_qwen7b_shape_paged_equals_contiguous_and_oracle(ctx):
    L, H, D, S, N, bs = 28, 4, 128, 16, 8192, 16
    dev = f"cuda:{ctx.device}"
    g = torch.Generator(device=dev)
    g.manual_seed(77)
    pages = S * N // bs
    k = [torch.randn(pages, bs, H, D, generator=g, device=dev, dtype=torch.bfloat16) for _ in range(L)]
    v = [torch.randn(pages, bs, H, D, generator=g, device=dev, dtype=torch.bfloat16) for _ in range(L)]
    bt = torch.randperm(pages, generator=g, device=dev).to(torch.int32).view(S, N // bs).contiguous()
    paged = C.KvCacheView(k, v, [N] * S, block_tables=bt)
    r_paged, trees = C.kv_commit(ctx, paged, keep_trees=True)
    # gather rows in (sequence, position) order
    idx = bt.long().view(-1)
    kc = [t[idx].reshape(S * N, H, D) for t in k]
    vc = [t[idx].reshape(S * N, H, D) for t in v]
    r_cont, _ = C.kv_commit(ctx, C.KvCacheView(kc, vc, [N] * S), keep_trees=False)
    ctx.sync(timeout_ms=300000)
    assert torch.equal(r_paged, r_cont)
    rp = r_paged.cpu().numpy()
    # oracle on two (sequence, layer) trees
    for s, l in ((0, 0), (S - 1, L - 1)):
        kh = kc[l][s * N:(s + 1) * N].view(torch.int16).cpu().numpy().view(np.uint16)[None]
        vh = vc[l][s * N:(s + 1) * N].view(torch.int16).cpu().numpy().view(np.uint16)[None]
        o, _ = kvref.Transcript(kh, vh, [N], VC_DTYPE_BF16, layer_base=l).oracle(n_threads=16, with_nodes=False)
        assert bytes(o[0, 0]) == bytes(rp[s, l])
    # 1024 random openings verify against their kv_roots
    rng = np.random.default_rng(3)
    tsel = rng.integers(0, S * L, 1024)
    psel = rng.integers(0, N, 1024)
    sib, depth = trees.prove(list(tsel), list(psel))
    sib = sib.cpu().numpy()
    for i in range(1024):
        t, p = int(tsel[i]), int(psel[i])
        leaf = bytes(trees.nodes(t)[p].cpu().numpy())
        proof = O.MerkleProof(p, [bytes(x) for x in sib[i, :depth[i]]])
        assert O.verify(bytes(rp[t // L, t % L]), leaf, proof)


@pytest.mark.parametrize("n", [32768, 32769])
def test_llama70b_sequence_length_roots_and_deep_openings(ctx, n):
    """C5's sequence length (32 768 positions: 256 chunks per tree, 15 levels)
    and one more (padded to 65 536: half the tree is padding): kv_roots against
    the oracle's C restatement, and openings at both ends verify."""
    L, H, D = 2, 8, 128
    k, v = synth.kv_rows_bf16(n % 97, L, n, H, D)
    tr = kvref.Transcript(k, v, [n], VC_DTYPE_BF16)
    view = tr.view(ctx.device)
    roots, trees = C.kv_commit(ctx, view, keep_trees=True)
    ctx.sync(timeout_ms=120000)
    oroots, _ = tr.oracle(n_threads=L, with_nodes=False)
    assert np.array_equal(roots.cpu().numpy(), oroots)
    pos = [0, 1, n // 2, n - 2, n - 1]
    sib, depth = trees.prove([1] * len(pos), pos)
    sib = sib.cpu().numpy()
    kf = O.bf16_to_f64(k[1].reshape(n, -1))
    vf = O.bf16_to_f64(v[1].reshape(n, -1))
    for i, p in enumerate(pos):
        assert depth[i] == (n - 1).bit_length()
        proof = O.MerkleProof(leaf_index=p, siblings=[bytes(x) for x in sib[i, :depth[i]]])
        assert O.verify(bytes(oroots[0, 1]), O.hash_kv_entry(1, p, kf[p], vf[p]), proof)
