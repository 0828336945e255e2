"""KV commitment on the GPU vs the oracle: kv_roots, tree nodes and openings.

Mirrors the reference's KV tests (crates/verilm-verify/tests/canonical.rs:
3096-3400: hash_kv_entry sensitivity, kv_commit_e2e_toy_autoregressive,
kv_open_produces_valid_merkle_proofs) and merkle.rs:608-666 (tree sizes).
All comparisons are bit-exact.
"""
import json
import os

import numpy as np
import pytest

from commitllm_b200 import commit as C
from commitllm_b200._lib import VC_DTYPE_BF16, VC_DTYPE_F32, VC_DTYPE_F64, VcValueError
from oracle import commit_oracle as O
from tests import kvref
from tests.golden.make_c1_golden import C1, c1_inputs

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "c1_golden.json")


def _gpu(ctx, tr, keep=True):
    view = tr.view(ctx.device)
    roots, trees = C.kv_commit(ctx, view, keep_trees=keep)
    ctx.sync(timeout_ms=60000)
    return roots.cpu().numpy(), trees


def test_c1_kv_roots_and_openings_match_golden(ctx):
    g = json.load(open(GOLDEN))
    k, v, *_ = c1_inputs()
    tr = kvref.Transcript(k, v, [C1["n_tokens"]], VC_DTYPE_BF16)
    roots, trees = _gpu(ctx, tr)
    assert [bytes(r).hex() for r in roots[0]] == g["kv_roots"]
    for o in g["kv_openings"]:
        sib, depth = trees.prove([o["layer"]], [o["pos"]])
        got = [bytes(x).hex() for x in sib[0, :depth[0]].cpu().numpy()]
        assert got == o["siblings"]
        leaf = bytes(trees.nodes(o["layer"])[o["pos"]].cpu().numpy())
        assert leaf.hex() == o["leaf"]
        pr = O.MerkleProof(o["pos"], [bytes.fromhex(s) for s in got])
        assert O.verify(bytes.fromhex(g["kv_roots"][o["layer"]]), leaf, pr)


@pytest.mark.parametrize("n", [1, 2, 3, 5, 8, 13, 28, 32, 127, 128, 129, 255, 256, 257, 1000])
def test_tree_sizes_nodes_match_build_tree(ctx, n):
    tr = kvref.contiguous(100 + n, 2, [n], 2, 16)
    roots, trees = _gpu(ctx, tr)
    oroots, onodes = tr.oracle()
    assert np.array_equal(roots, oroots)
    for t in range(2):
        assert np.array_equal(trees.nodes(t).cpu().numpy(), onodes[t])


def test_python_oracle_agrees_with_c_oracle_and_gpu(ctx):
    tr = kvref.contiguous(7, 3, [37], 2, 8, layer_base=5)
    roots, _ = _gpu(ctx, tr, keep=False)
    oroots, _ = tr.oracle(with_nodes=False)
    assert np.array_equal(roots, oroots)
    for l in range(3):
        kf = O.bf16_to_f64(tr.k[l].reshape(37, -1))
        vf = O.bf16_to_f64(tr.v[l].reshape(37, -1))
        leaves = [O.hash_kv_entry(5 + l, p, kf[p], vf[p]) for p in range(37)]
        assert bytes(roots[0, l]) == O.compute_root(leaves)


def test_paged_multi_sequence_ragged(ctx):
    lens = [1, 16, 17, 200, 128, 300, 3]
    tr = kvref.paged(11, 3, lens, 4, 32, block_size=16)
    roots, trees = _gpu(ctx, tr)
    oroots, onodes = tr.oracle()
    assert np.array_equal(roots, oroots)
    for t in range(len(lens) * 3):
        assert np.array_equal(trees.nodes(t).cpu().numpy(), onodes[t])


@pytest.mark.parametrize("dtype", [VC_DTYPE_F32, VC_DTYPE_F64])
def test_wide_dtypes(ctx, dtype):
    tr = kvref.contiguous(21, 2, [45, 130], 2, 64, dtype=dtype)
    roots, _ = _gpu(ctx, tr, keep=False)
    oroots, _ = tr.oracle(with_nodes=False)
    assert np.array_equal(roots, oroots)


def test_f64_entries_match_reference_hash_kv_entry(ctx):
    # kv_hash_* tests of canonical.rs use arbitrary f64 values (e.g. 4.1)
    k = np.array([[[[1.0, 2.0, 3.0, 4.1, 5.5, -6.25, 7.0, 8.0]]],
                  [[[0.1, 0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8]]]], dtype=np.float64).reshape(1, 2, 1, 8)
    v = (k * -3.0).copy()
    tr = kvref.Transcript(k, v, [2], VC_DTYPE_F64)
    roots, trees = _gpu(ctx, tr)
    leaves = [O.hash_kv_entry(0, p, k[0, p, 0], v[0, p, 0]) for p in range(2)]
    assert bytes(roots[0, 0]) == O.compute_root(leaves)
    assert bytes(trees.nodes(0)[1].cpu().numpy()) == leaves[1]


def test_special_values_bf16(ctx):
    # zeros, negative zero, subnormals, infinities, NaNs (quiet and signalling)
    special = np.array([0x0000, 0x8000, 0x0001, 0x8001, 0x007F, 0x0040, 0x7F80, 0xFF80, 0x7FC0, 0x7F81,
                        0xFFC1, 0x0080, 0x7F7F, 0xFF7F, 0x3F80, 0xBF80], dtype=np.uint16)
    tr = kvref.contiguous(5, 1, [64], 2, 16)
    flat_k = tr.k.reshape(-1)
    flat_v = tr.v.reshape(-1)
    rng = np.random.default_rng(0)
    idx = rng.choice(flat_k.size, 600, replace=False)
    flat_k[idx] = special[rng.integers(0, special.size, 600)]
    flat_v[idx[:300]] = special[rng.integers(0, special.size, 300)]
    flat_k[:32] = special[np.arange(32) % special.size]   # a whole row of specials
    roots, _ = _gpu(ctx, tr, keep=False)
    oroots, _ = tr.oracle(with_nodes=False)
    assert np.array_equal(roots, oroots)
    # and the Python oracle's widening rule agrees with the C oracle's
    kf = O.bf16_to_f64(tr.k[0].reshape(64, -1))
    vf = O.bf16_to_f64(tr.v[0].reshape(64, -1))
    assert O.compute_root([O.hash_kv_entry(0, p, kf[p], vf[p]) for p in range(64)]) == bytes(oroots[0, 0])


def test_special_values_f32(ctx):
    tr = kvref.contiguous(6, 1, [33], 1, 16, dtype=VC_DTYPE_F32)
    bits = tr.k.view(np.uint32).reshape(-1)
    vals = np.array([0, 0x80000000, 1, 0x807FFFFF, 0x00400000, 0x7F800000, 0xFF800000, 0x7FC00000, 0x7F800001,
                     0x00800000, 0x7F7FFFFF], dtype=np.uint32)
    bits[: vals.size * 3] = np.tile(vals, 3)
    roots, _ = _gpu(ctx, tr, keep=False)
    oroots, _ = tr.oracle(with_nodes=False)
    assert np.array_equal(roots, oroots)


@pytest.mark.parametrize("heads,hd", [(2, 2), (1, 4), (3, 12), (1, 1), (5, 24)])
def test_generic_shapes(ctx, heads, hd):
    # kv_dim not a multiple of 8 takes the element-wise kernel (the reference's
    # toy model has kv_dim 4, constants.rs:232-246)
    tr = kvref.contiguous(31, 2, [3, 9], heads, hd)
    roots, trees = _gpu(ctx, tr)
    oroots, onodes = tr.oracle()
    assert np.array_equal(roots, oroots)
    for t in range(4):
        assert np.array_equal(trees.nodes(t).cpu().numpy(), onodes[t])


def test_hnd_layout_strides(ctx):
    # [pages, heads, block, dim] (head stride = block * dim)
    tr = kvref.paged(41, 2, [40, 70], 4, 16, block_size=16)
    k_hnd = np.ascontiguousarray(tr.k.transpose(0, 1, 3, 2, 4))
    v_hnd = np.ascontiguousarray(tr.v.transpose(0, 1, 3, 2, 4))
    import torch
    kd = torch.from_numpy(k_hnd.view(np.int16)).cuda()
    vd = torch.from_numpy(v_hnd.view(np.int16)).cuda()
    kv = [kd[l].permute(0, 2, 1, 3) for l in range(2)]   # logical [pages, block, heads, dim]
    vv = [vd[l].permute(0, 2, 1, 3) for l in range(2)]
    view = C.KvCacheView(kv, vv, tr.seq_lens, block_tables=torch.from_numpy(tr.block_tables).cuda())
    roots, _ = C.kv_commit(ctx, view, keep_trees=False)
    oroots, _ = tr.oracle(with_nodes=False)
    assert np.array_equal(roots.cpu().numpy(), oroots)


def test_leaf_sensitivity(ctx):
    # canonical.rs kv_hash_different_{k,v,layer,position}
    tr = kvref.contiguous(9, 1, [4], 1, 8)
    base, _ = _gpu(ctx, tr, keep=False)
    tr2 = kvref.contiguous(9, 1, [4], 1, 8)
    tr2.k[0, 2, 0, 3] ^= 1
    r2, _ = _gpu(ctx, tr2, keep=False)
    tr3 = kvref.contiguous(9, 1, [4], 1, 8)
    tr3.v[0, 0, 0, 7] ^= 0x100
    r3, _ = _gpu(ctx, tr3, keep=False)
    tr4 = kvref.contiguous(9, 1, [4], 1, 8, layer_base=1)
    r4, _ = _gpu(ctx, tr4, keep=False)
    assert len({bytes(x[0, 0]) for x in (base, r2, r3, r4)}) == 4


def test_roots_only_matches_with_trees(ctx):
    tr = kvref.paged(13, 2, [1000, 129, 1], 2, 64)
    a, _ = _gpu(ctx, tr, keep=False)
    b, _ = _gpu(ctx, tr, keep=True)
    assert np.array_equal(a, b)


def test_openings_every_level(ctx):
    tr = kvref.contiguous(17, 2, [300], 2, 8)
    roots, trees = _gpu(ctx, tr)
    pos = list(range(0, 300, 7)) + [299]
    sib, depth = trees.prove([1] * len(pos), pos)
    sib = sib.cpu().numpy()
    nodes = trees.nodes(1).cpu().numpy()
    otree = O.MerkleTree([bytes(x) for x in nodes], 300, 512, bytes(nodes[-1]))
    for i, p in enumerate(pos):
        ref = O.prove(otree, p)
        assert [bytes(x) for x in sib[i, :depth[i]]] == ref.siblings
        assert O.verify(bytes(roots[0, 1]), bytes(nodes[p]), ref)


def test_prove_rejects_out_of_range(ctx):
    tr = kvref.contiguous(19, 1, [5], 1, 8)
    _, trees = _gpu(ctx, tr)
    with pytest.raises(VcValueError):
        trees.prove([0], [5])
    with pytest.raises(VcValueError):
        trees.prove([1], [0])


def test_bad_page_id_is_reported_not_faulted(ctx):
    tr = kvref.paged(23, 1, [40], 1, 8, block_size=16)
    tr.block_tables[0, 1] = 10 ** 6      # outside the cache: the kernel skips it and flags
    view = tr.view(ctx.device)
    C.kv_commit(ctx, view, keep_trees=False)
    with pytest.raises(VcValueError):
        ctx.sync(timeout_ms=60000)
    ctx.sync(timeout_ms=60000)           # the flag is cleared


def test_invalid_arguments(ctx):
    tr = kvref.contiguous(3, 1, [4], 1, 8)
    view = tr.view(ctx.device)
    view.seq_lens = [0]
    with pytest.raises(VcValueError):
        C.kv_commit(ctx, view)
    view.seq_lens = [5]   # more rows than the buffer holds
    with pytest.raises(VcValueError):
        C.kv_commit(ctx, view)


@pytest.mark.parametrize("paged_case", [False, True])
def test_host_buffer_commit_matches_device_commit(ctx, paged_case):
    """kv_commit_host pipelines layer groups from host memory; roots and proofs equal kv_commit's."""
    import torch
    tr = kvref.paged(71, 5, [40, 300], 2, 64) if paged_case else kvref.contiguous(72, 5, [333], 4, 32)
    view = tr.view(ctx.device)
    want, wtrees = C.kv_commit(ctx, view, keep_trees=True)
    host_k = [t.cpu().pin_memory() for t in view.k_layers]
    host_v = [t.cpu().pin_memory() for t in view.v_layers]
    got, groups = C.kv_commit_host(ctx, host_k, host_v, tr.seq_lens, block_tables=view.block_tables, n_groups=3)
    ctx.sync(timeout_ms=60000)
    assert torch.equal(got, want)
    s, l = len(tr.seq_lens) - 1, 4
    sib, depth = groups.prove(s, l, [0, 7, tr.seq_lens[s] - 1])
    sib2, depth2 = wtrees.prove([s * 5 + l] * 3, [0, 7, tr.seq_lens[s] - 1])
    assert depth == depth2 and torch.equal(sib, sib2)
    groups.free()


def test_kv_openings_verify_like_the_verifier(ctx):
    """open_v4's KV part: every returned KvEntry re-hashes (hash_kv_entry) to a leaf whose
    proof verifies against kv_roots[layer] -- verify_kv_entry_provenance's check."""
    tr = kvref.paged(81, 4, [150], 2, 32, block_size=16)
    view = tr.view(ctx.device)
    roots, trees = C.kv_commit(ctx, view, keep_trees=True)
    layers, t = [3, 0], 149
    ent, sib, depth = C.kv_open(ctx, view, trees, 0, layers, t + 1)
    ctx.sync(timeout_ms=60000)
    ent, sib, roots = ent.cpu().numpy(), sib.cpu().numpy(), roots.cpu().numpy()
    assert depth == 8 and ent.shape == (2, 150, 2, 64)
    for i, l in enumerate(layers):
        for p in range(0, t + 1, 7):
            leaf = O.hash_kv_entry(l, p, ent[i, p, 0], ent[i, p, 1])
            assert O.verify(bytes(roots[0, l]), leaf, O.MerkleProof(p, [bytes(x) for x in sib[i, p]]))
        # entries are the cache rows widened exactly
        pg = tr.block_tables[0, 5 // 16]
        want = O.bf16_to_f64(tr.k[l, pg, 5 % 16].reshape(-1))
        assert np.array_equal(ent[i, 5, 0].view(np.uint64), want.view(np.uint64))


def test_audit_kv_encodings(ctx):
    """kv_entries / kv_proofs in serde_json (f64 hex) and bincode form, via the drop-in handle."""
    import struct
    from commitllm_b200 import verilm_rs as V
    tr = kvref.contiguous(82, 2, [9], 1, 8)
    view = tr.view(ctx.device)
    a = np.zeros((9, 2, 4), np.int8)
    h = V.commit_minimal_from_captures([a[t, l] for t in range(9) for l in range(2)],
                                       np.ones(9 * 2 * 4, np.float32), 2, [1] * 9, list(range(9)), b"p", b"\0" * 32,
                                       kv_cache=view, ctx=ctx)
    js = json.loads(h.audit_kv_json(4, [1]))
    assert len(js["kv_entries"]) == 1 and len(js["kv_entries"][0]) == 5
    e = js["kv_entries"][0][4]
    k = np.frombuffer(bytes.fromhex("".join(e["k_roped"])), dtype="<f8")
    v = np.frombuffer(bytes.fromhex("".join(e["v_deq"])), dtype="<f8")
    leaf = O.hash_kv_entry(1, 4, k, v)
    pr = js["kv_proofs"][0][4]
    assert O.verify(bytes.fromhex(h.kv_roots_hex()[1]), leaf, O.MerkleProof(pr["leaf_index"], [bytes(s) for s in pr["siblings"]]))
    b = h.audit_kv_bincode(4, [1])
    # Some(vec of 1 layer) of 5 entries, first entry's k_roped length 8
    assert b[0] == 1 and struct.unpack_from("<QQQ", b, 1) == (1, 5, 8)
    k0 = bytes.fromhex("".join(js["kv_entries"][0][0]["k_roped"]))
    assert b[25:25 + 64] == k0                                   # entry 0's k_roped, raw f64 LE
