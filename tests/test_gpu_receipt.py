"""The drop-in as the reference's server calls it, manifest included, and the
audit receipts it opens, checked the way the verifier checks them.

The call has the shape of sidecar/verilm/server.py:1162-1177 (per-(pass,
layer) o_proj captures, drain-order scales, token_ids = all_ids[1:], prompt,
seed, manifest, n_prompt_tokens, captured logits) plus the request's KV cache.
The receipt (``audit_v4_binary``: "VV4A" || zstd(bincode)) is decoded with the
golden generator's independent bincode reader and every digest in it is
recomputed with the oracle: the retained leaf and its proof against
merkle_root, the IO chain replayed from genesis over the prefix leaves
(canonical.rs:407-441), every prefix proof, and every KV entry's leaf and
proof against kv_roots[layer] (canonical.rs:3344-3540).
"""
import json
import struct

import numpy as np
import pytest

from commitllm_b200 import manifest as M
from commitllm_b200 import verilm_rs as V
from commitllm_b200._lib import VC_DTYPE_BF16
from oracle import commit_oracle as O
from tests import kvref
from tests.golden import make_golden as G
from tests.golden.make_c1_golden import C1, c1_inputs
from tests.test_gpu_trace import _drain_scales

pytestmark = pytest.mark.gpu

MANIFEST = {
    "tokenizer_hash": "11" * 32, "temperature": 0.6, "top_k": 20, "top_p": 0.9, "eos_policy": "stop",
    "weight_hash": "22" * 32, "quant_hash": "33" * 32, "system_prompt_hash": "44" * 32, "repetition_penalty": 1.0,
    "frequency_penalty": 0.0, "presence_penalty": 0.0, "logit_bias": [[5, 1.25]], "bad_word_ids": [7, 3],
    "guided_decoding": "", "stop_sequences": ["</s>"], "max_tokens": 256, "chat_template_hash": "55" * 32,
    "rope_config_hash": None, "rmsnorm_eps": 1e-5, "sampler_version": "chacha20-vi-sample-v1",
    "bos_eos_policy": "add_bos", "truncation_policy": None, "special_token_policy": None, "padding_policy": None,
    "decode_mode": "sampled", "adapter_hash": None, "attn_backend": "sdpa", "attn_mode": "stock",
    "attn_dtype": "bfloat16", "quant_family": "W8A8", "scale_derivation": "absmax", "quant_block_size": None,
    "kv_dim": 256, "ffn_dim": None, "d_head": 64, "n_q_heads": 16, "n_kv_heads": 4, "rope_theta": 10000.0,
    "min_tokens": 0, "ignore_eos": False, "detokenization_policy": "default", "eos_token_id": 2,
}


def _commit(ctx, n_prompt_tokens=3):
    k, v, tok, pos, a, sc = c1_inputs()
    n, L = C1["n_tokens"], C1["n_layers"]
    rng = np.random.default_rng(808)
    gen = n - (n_prompt_tokens - 1)
    logits = [rng.standard_normal(50, dtype=np.float32) * 3 for _ in range(gen)]
    view = kvref.Transcript(k, v, [n], VC_DTYPE_BF16).view(ctx.device)
    h = V.commit_minimal_from_captures([a[t, l] for t in range(n) for l in range(L)], _drain_scales(L, [1] * n, sc),
                                       L, [1] * n, [int(x) for x in tok], C1["prompt"].encode(),
                                       bytes.fromhex(C1["sampling_seed"]), manifest=MANIFEST,
                                       n_prompt_tokens=n_prompt_tokens, captured_logits_f32=logits, kv_cache=view,
                                       ctx=ctx)
    return h, (k, v, tok, a, sc, logits)


def test_manifest_bound_like_the_reference(ctx):
    h, _ = _commit(ctx)
    m = M.from_dict(MANIFEST)
    om = dict(m)
    c = json.loads(h.commitment_json())
    assert bytes(c["manifest_hash"]) == O.hash_manifest(om)
    assert bytes(c["input_spec_hash"]) == O.hash_input_spec(om)
    assert bytes(c["model_spec_hash"]) == O.hash_model_spec(om)
    assert bytes(c["decode_spec_hash"]) == O.hash_decode_spec(om)
    assert bytes(c["output_spec_hash"]) == O.hash_output_spec(om)
    assert h.manifest_hash_hex() == O.hash_manifest(om).hex()
    with pytest.raises(ValueError, match="missing tokenizer_hash"):
        V.commit_minimal_from_captures([b"\x01"], np.ones(4, np.float32), 1, [1], [1], b"p", bytes(32),
                                       manifest={"temperature": 0.0}, ctx=ctx)


def _retained_leaf(rec, logits_row):
    layers = [O.RetainedLayerState(bytes.fromhex(l["a"]), struct.unpack("<f", struct.pack("<I", l["scale_a_bits"]))[0])
              for l in rec["retained_layers"]]
    return O.hash_retained_with_captured_logits(layers, None, None, logits_row)


def _proof(p):
    return O.MerkleProof(p["leaf_index"], [bytes.fromhex(s) for s in p["siblings"]])


@pytest.mark.parametrize("t", [0, 1, 2, 57, 127])
def test_audit_receipt_verifies(ctx, t):
    n_prompt = 3
    h, (k, v, tok, a, sc, logits) = _commit(ctx, n_prompt)
    gen_start = n_prompt - 1
    blob = h.audit_v4_binary(t, layer_indices=[1, 0], output_text="out")
    assert blob[:4] == b"VV4A"
    raw = G.zstd_decompress(blob[4:])
    rec = G.read_v4_audit_prefix(blob)
    r = G.Bincode(raw)
    r.o = G._prefix_len(blob)
    G.read_v4_audit_rest(r, rec)                      # consumes the whole receipt
    c = rec["commitment"]
    assert c == {**c, "merkle_root": h.merkle_root_hex(), "io_root": h.io_root_hex(), "kv_roots": h.kv_roots_hex()}
    assert c["manifest_hash"] == h.manifest_hash_hex()
    m = {kk: (bytes.fromhex(vv) if vv is not None and M.KIND[kk].endswith("b32") else vv)
         for kk, vv in rec["manifest"].items()}
    assert O.hash_manifest(m).hex() == c["manifest_hash"]
    assert rec["token_index"] == t and rec["token_id"] == int(tok[t]) and rec["output_text"] == "out"
    assert bytes.fromhex(rec["prompt_field"]) == C1["prompt"].encode() and rec["n_prompt_tokens"] == n_prompt
    assert rec["shell_opening"] is None
    # retained leaf and its proof (canonical.rs:365-366)
    leaf = _retained_leaf(rec, logits[t - gen_start] if t >= gen_start else None)
    assert [bytes.fromhex(l["a"]) for l in rec["retained_layers"]] == [a[t, l].tobytes() for l in range(C1["n_layers"])]
    root = bytes.fromhex(c["merkle_root"])
    assert O.verify(root, leaf, _proof(rec["merkle_proof"]))
    # prefix leaves and proofs, IO chain from genesis (canonical.rs:389-441)
    assert len(rec["prefix_leaf_hashes"]) == t and rec["prefix_token_ids"] == [int(x) for x in tok[:t]]
    prev = O.io_genesis_v4(O.hash_prompt(C1["prompt"].encode()))
    for j, (lh, p) in enumerate(zip(rec["prefix_leaf_hashes"], rec["prefix_merkle_proofs"])):
        assert O.verify(root, bytes.fromhex(lh), _proof(p))
        prev = O.io_hash_v4(bytes.fromhex(lh), rec["prefix_token_ids"][j], prev)
    assert prev.hex() == rec["prev_io_hash"]
    io_t = O.io_hash_v4(leaf, rec["token_id"], prev)
    assert O.verify(bytes.fromhex(c["io_root"]), io_t, _proof(rec["io_proof"]))
    # KV provenance of the challenged layers, positions 0..=t (canonical.rs:3379-3388)
    assert len(rec["kv_entries"]) == 2 and all(len(e) == t + 1 for e in rec["kv_entries"])
    for layer, ents, prfs in zip([1, 0], rec["kv_entries"], rec["kv_proofs"]):
        kf = O.bf16_to_f64(k[layer].reshape(C1["n_tokens"], -1))
        vf = O.bf16_to_f64(v[layer].reshape(C1["n_tokens"], -1))
        for p, (e, pr) in enumerate(zip(ents, prfs)):
            kr = np.frombuffer(bytes.fromhex(e["k_roped"]), "<f8")
            vr = np.frombuffer(bytes.fromhex(e["v_deq"]), "<f8")
            assert np.array_equal(kr.view(np.uint64), kf[p].view(np.uint64))
            assert np.array_equal(vr.view(np.uint64), vf[p].view(np.uint64))
            assert O.verify(bytes.fromhex(c["kv_roots"][layer]), O.hash_kv_entry(layer, p, kr, vr), _proof(pr))
    # the JSON form carries the same receipt
    d = json.loads(h.audit_v4(t, layer_indices=[1, 0], output_text="out"))
    assert bytes(d["commitment"]["merkle_root"]).hex() == c["merkle_root"]
    assert d["token_index"] == t and len(d["prefix_leaf_hashes"]) == t


def test_audit_without_kv_and_bad_index(ctx):
    h, _ = _commit(ctx)
    from commitllm_b200 import receipt as R
    resp = R.deserialize_v4_audit(h.audit_v4_binary(4, include_kv=False))
    assert resp["kv_entries"] is None and resp["kv_proofs"] is None
    with pytest.raises(ValueError, match="out of range"):
        h.audit_v4_binary(C1["n_tokens"])


def test_commit_request_equals_the_from_captures_commit(ctx):
    """commit_request (whole tensors, KV trees on a second stream) makes the same
    commitment and the same receipts as commit_minimal_from_captures."""
    import torch
    from commitllm_b200 import receipt as R
    h1, (k, v, tok, a, sc, logits) = _commit(ctx)
    n = C1["n_tokens"]
    view = kvref.Transcript(k, v, [n], VC_DTYPE_BF16).view(ctx.device)
    A = ctx.to_device(np.ascontiguousarray(a)).view(torch.int8)
    S = ctx.to_device(np.ascontiguousarray(sc, dtype=np.float32))
    LG = ctx.to_device(np.stack(logits).astype(np.float32))
    T = ctx.to_device(np.asarray(tok, dtype=np.int32))
    h2 = V.commit_request(A, S, T, C1["prompt"].encode(), bytes.fromhex(C1["sampling_seed"]), n_prompt_tokens=3,
                          captured_logits_f32=LG, kv_cache=view, manifest=MANIFEST, ctx=ctx)
    assert h2.commitment_json() == h1.commitment_json()
    for t in (0, 77):
        r1 = R.zstd_decompress(h1.audit_v4_binary(t, layer_indices=[0])[4:])
        r2 = R.zstd_decompress(h2.audit_v4_binary(t, layer_indices=[0])[4:])
        assert r1 == r2


@pytest.mark.parametrize("where", ["cuda", "cpu"])
def test_retained_kv_survives_cache_reuse(ctx, where):
    """After retain_kv, the receipts (KV entries and proofs included) do not
    change when the engine overwrites the request's cache pages."""
    import torch
    h, _ = _commit(ctx)
    before = {t: h.audit_v4_binary(t, layer_indices=[0, 1]) for t in (0, 9, C1["n_tokens"] - 1)}
    cache = h._kv_view
    h.retain_kv(where)
    with torch.cuda.stream(ctx.stream):
        for t in list(cache.k_layers) + list(cache.v_layers):
            t.zero_()                       # the engine reuses the pages
    ctx.sync()
    for t, b in before.items():
        assert h.audit_v4_binary(t, layer_indices=[0, 1]) == b
    h.retain_kv(where)                      # a second call keeps what was retained
    assert h.audit_v4_binary(9, layer_indices=[0, 1]) == before[9]


def test_retained_kv_from_a_paged_cache(ctx):
    """retain_kv gathers the rows of a paged cache (permuted pages): the
    receipts before and after the pages are overwritten are identical, and
    equal to those of the same request committed from a contiguous cache."""
    import torch
    from commitllm_b200.commit import KvCacheView
    h_c, (k, v, tok, a, sc, logits) = _commit(ctx)
    cont = h_c._kv_view
    n, L, bs = C1["n_tokens"], C1["n_layers"], 16
    nb = (n + bs - 1) // bs
    perm = torch.randperm(nb + 3, generator=torch.Generator().manual_seed(3))[:nb]

    def paged(t):
        p = torch.zeros(nb + 3, bs, *t.shape[1:], dtype=t.dtype, device=t.device)
        for b in range(nb):
            rows = t[b * bs:(b + 1) * bs]
            p[int(perm[b]), : rows.shape[0]] = rows
        return p

    view = KvCacheView([paged(t) for t in cont.k_layers], [paged(t) for t in cont.v_layers], [n],
                       block_tables=perm.to(torch.int32).cuda(ctx.device)[None].contiguous())
    h = V.commit_minimal_from_captures([a[t, l] for t in range(n) for l in range(L)], _drain_scales(L, [1] * n, sc),
                                       L, [1] * n, [int(x) for x in tok], C1["prompt"].encode(),
                                       bytes.fromhex(C1["sampling_seed"]), manifest=MANIFEST, n_prompt_tokens=3,
                                       captured_logits_f32=logits, kv_cache=view, ctx=ctx)
    assert h.kv_roots_hex() == h_c.kv_roots_hex()
    want = h_c.audit_v4_binary(11, layer_indices=[0, 1])
    h.retain_kv()
    with torch.cuda.stream(ctx.stream):
        for t in list(view.k_layers) + list(view.v_layers):
            t.fill_(7)
    ctx.sync()
    assert h.audit_v4_binary(11, layer_indices=[0, 1]) == want


def test_witnessed_scores_ride_in_the_receipt(ctx):
    """set_witnessed_scores (verilm-py/src/lib.rs:623-648): the scores are in
    every receipt that includes the KV openings, and absent otherwise."""
    from commitllm_b200 import receipt as R
    h, _ = _commit(ctx)
    rng = np.random.default_rng(4)
    scores = [rng.standard_normal(4 * 9).astype(np.float32) for _ in range(C1["n_layers"])]
    h.set_witnessed_scores(scores, n_q_heads=4)
    resp = R.deserialize_v4_audit(h.audit_v4_binary(8))
    got = resp["witnessed_scores"]
    assert len(got) == len(scores)
    for g_, s in zip(got, scores):
        assert g_["n_q_heads"] == 4 and g_["seq_len"] == 9 and np.array_equal(np.asarray(g_["scores"]), s)
    assert R.deserialize_v4_audit(h.audit_v4_binary(8, include_kv=False))["witnessed_scores"] is None
    assert json.loads(h.audit_v4(8))["witnessed_scores"][0]["seq_len"] == 9
    with pytest.raises(ValueError, match="not divisible"):
        h.set_witnessed_scores([np.zeros(10, np.float32)], n_q_heads=4)
    assert h.deep_prefix is False and h.use_captured_x_attn is False
    h.deep_prefix = True                     # accepted; no bridge weights here, as in the reference without them
    assert R.deserialize_v4_audit(h.audit_v4_binary(8))["prefix_retained"] is None
