"""The oracle against the reference's golden vectors and tree identities (CPU).

Pins: golden_conformance.rs:253-261 (merkle_root / io_root), the frozen
receipts v4_audit_{canonical,fullbridge}.bin (roots, prompt hash, seed
commitment, genesis), FIPS 180-4 SHA-256 test vectors, and the structural
identities of merkle.rs:608-666.
"""
import hashlib
import json
import os
import struct

import numpy as np
import pytest

from oracle import commit_oracle as O
from oracle import vco

HERE = os.path.dirname(__file__)
PINS = json.load(open(os.path.join(HERE, "golden", "reference_pins.json")))


def _layers(name):
    return [O.RetainedLayerState(bytes.fromhex(l["a"]), struct.unpack("<f", struct.pack("<I", l["scale_a_bits"]))[0])
            for l in PINS[name]["retained_layers"]]


def test_sha256_standard_vectors():
    assert O.sha256(b"abc").hex() == "ba7816bf8f01cfea414140de5dae2223b00361a396177a9cb410ff61f20015ad"
    assert O.sha256(b"").hex() == "e3b0c44298fc1c149afbf4c8996fb92427ae41e4649b934ca495991b7852b855"
    msg = b"abcdbcdecdefdefgefghfghighijhijkijkljklmklmnlmnomnopnopq"
    assert O.sha256(msg).hex() == "248d6a61d20638b8e5c026930c3e6039a33ce45964ff2167f6ecedd419db06c1"


def test_golden_e2e_verify_pins():
    g = PINS["golden_e2e_verify"]
    com = O.commit_minimal([_layers(g["retained_from"])], g["token_ids"], g["prompt"].encode(), bytes([7] * 32),
                           n_prompt_tokens=g["n_prompt_tokens"])
    assert com.merkle_root.hex() == g["merkle_root"]
    assert com.io_root.hex() == g["io_root"]


@pytest.mark.parametrize("name", ["v4_audit_canonical.bin", "v4_audit_fullbridge.bin"])
def test_frozen_receipts(name):
    r = PINS[name]
    c = r["commitment"]
    com = O.commit_minimal([_layers(name)], [r["token_id"]], r["prompt"].encode(), bytes.fromhex(r["sampling_seed"]),
                           n_prompt_tokens=c["n_prompt_tokens"])
    assert com.merkle_root.hex() == c["merkle_root"]
    assert com.io_root.hex() == c["io_root"]
    assert com.prompt_hash.hex() == c["prompt_hash"]
    assert com.seed_commitment.hex() == c["seed_commitment"]
    assert O.io_genesis_v4(O.hash_prompt(r["prompt"].encode())).hex() == r["prev_io_hash"]
    assert r["merkle_proof"]["siblings"] == [] and r["io_proof"]["siblings"] == []


def test_single_leaf_root_is_leaf():
    leaf = O.hash_leaf(b"hello")
    t = O.build_tree([leaf])
    assert t.root == leaf and O.verify(t.root, leaf, O.prove(t, 0))


def test_two_and_five_leaves_and_tamper():
    leaves = [O.hash_leaf(bytes([i])) for i in range(5)]
    t = O.build_tree(leaves)
    for i, leaf in enumerate(leaves):
        assert O.verify(t.root, leaf, O.prove(t, i))
    p = O.prove(t, 0)
    assert not O.verify(t.root, leaves[1], p)
    p.siblings[0] = bytes([p.siblings[0][0] ^ 0xFF]) + p.siblings[0][1:]
    assert not O.verify(t.root, leaves[0], p)


@pytest.mark.parametrize("n", [1, 2, 3, 5, 8, 13, 28, 32])
def test_compute_root_matches_build_tree(n):
    leaves = [O.hash_leaf(bytes([i])) for i in range(n)]
    assert O.build_tree(leaves).root == O.compute_root(leaves)


def test_padding_only_at_level_zero():
    leaves = [O.hash_leaf(b"x")] * 3
    t = O.build_tree(leaves)
    z = O.zero_subtree_roots(3)
    assert t.nodes[3] == bytes(32)                       # padded leaf
    assert t.nodes[5] == O.hash_pair(leaves[2], z[0])    # parent of a leaf and a pad
    t5 = O.build_tree([O.hash_leaf(b"y")] * 5)
    assert t5.nodes[8 + 3] == z[1]                       # parent of two pads = H(0^64), not zero


def test_kv_entry_encoding():
    k = np.array([1.0, 2.0, 3.0, 4.0])
    v = np.array([5.0, 6.0, 7.0, 8.0])
    msg = b"vi-kv-v1" + struct.pack("<II", 3, 9) + k.astype("<f8").tobytes() + v.astype("<f8").tobytes()
    assert O.hash_kv_entry(3, 9, k, v) == hashlib.sha256(msg).digest()
    assert O.hash_kv_entry(0, 0, k, v) != O.hash_kv_entry(0, 1, k, v)
    assert O.hash_kv_entry(0, 5, k, v) != O.hash_kv_entry(1, 5, k, v)
    assert O.hash_kv_entry(0, 0, [1.0, 2.0, 3.0, 4.1], v) != O.hash_kv_entry(0, 0, k, v)


def test_bf16_widening_is_exact():
    bits = np.arange(0, 1 << 16, dtype=np.uint32).astype(np.uint16)
    d = O.bf16_to_f64(bits)
    f = (bits.astype(np.uint32) << 16).view(np.float32)
    fin = np.isfinite(f)
    assert np.array_equal(d[fin], f[fin].astype(np.float64))
    nan = np.isnan(f)
    u = d[nan].view(np.uint64)
    assert np.all((u >> 51) & 0xFFF == 0xFFF)            # exponent all ones, quiet bit set


def test_c_oracle_matches_python_oracle():
    rng = np.random.default_rng(1)
    for n in (1, 2, 3, 5, 9, 33, 100):
        leaves = rng.integers(0, 256, size=(n, 32), dtype=np.uint8)
        t = O.build_tree([bytes(x) for x in leaves])
        nodes = vco.build_tree(leaves)
        assert [bytes(x) for x in nodes] == t.nodes
        assert vco.compute_root(leaves) == t.root
    leaves = rng.integers(0, 256, size=(17, 32), dtype=np.uint8)
    toks = rng.integers(0, 1 << 32, size=17, dtype=np.uint64).astype(np.uint32)
    io = vco.io_chain(leaves, toks, b"prompt")
    assert [bytes(x) for x in io] == O.io_chain([bytes(x) for x in leaves], [int(x) for x in toks], b"prompt")


def test_c1_golden_reproduces_with_c_oracle():
    from tests import kvref
    from commitllm_b200._lib import VC_DTYPE_BF16
    from tests.golden.make_c1_golden import C1, c1_inputs
    g = json.load(open(os.path.join(HERE, "golden", "c1_golden.json")))
    k, v, *_ = c1_inputs()
    roots, trees = kvref.Transcript(k, v, [C1["n_tokens"]], VC_DTYPE_BF16).oracle(n_threads=2)
    assert [bytes(r).hex() for r in roots[0]] == g["kv_roots"]
    for o in g["kv_openings"]:
        nodes = trees[o["layer"]]
        t = O.MerkleTree([bytes(x) for x in nodes], C1["n_tokens"], 128, bytes(nodes[-1]))
        assert [s.hex() for s in O.prove(t, o["pos"]).siblings] == o["siblings"]


def test_c_oracle_paged_matches_contiguous():
    from tests import kvref
    tr = kvref.paged(3, 2, [20, 1, 40], 2, 8, block_size=4)
    roots_p, _ = tr.oracle(with_nodes=False)
    # gather the pages into a contiguous layout and commit again
    rows_k, rows_v = [], []
    for s, n in enumerate(tr.seq_lens):
        for p in range(n):
            pg = tr.block_tables[s, p // 4]
            rows_k.append(tr.k[:, pg, p % 4])
            rows_v.append(tr.v[:, pg, p % 4])
    k = np.stack(rows_k, axis=1)
    v = np.stack(rows_v, axis=1)
    roots_c, _ = kvref.Transcript(k, v, tr.seq_lens, tr.dtype).oracle(with_nodes=False)
    assert np.array_equal(roots_p, roots_c)
