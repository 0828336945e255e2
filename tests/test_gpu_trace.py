"""Trace (retained-state) leaves, IO chain, trees and the verilm_rs drop-in on
the GPU vs the oracle and the reference's own golden vectors."""
import json
import os
import struct

import numpy as np
import pytest
import torch

from commitllm_b200 import commit as C
from commitllm_b200 import verilm_rs as V
from oracle import commit_oracle as O
from oracle import vco
from tests import synth
from tests.golden.make_c1_golden import C1, c1_inputs

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(__file__)
PINS = json.load(open(os.path.join(HERE, "golden", "reference_pins.json")))


def _pin_layers(name):
    r = PINS[name]
    return r, [(bytes.fromhex(l["a"]), l["scale_a_bits"]) for l in r["retained_layers"]]


def _drain_scales(n_layers, fwd_batch_sizes, scale_a):
    """Flat drain-order scales: per (fwd, layer) [B qkv | B o_proj | B gate | B down]."""
    out = []
    t0 = 0
    for bs in fwd_batch_sizes:
        for l in range(n_layers):
            out += [0.5] * bs
            out += [scale_a[t0 + b][l] for b in range(bs)]
            out += [0.25] * bs + [0.125] * bs
        t0 += bs
    return np.asarray(out, dtype=np.float32)


@pytest.mark.parametrize("name,prompt_key", [("v4_audit_canonical.bin", None), ("v4_audit_fullbridge.bin", None),
                                             ("v4_audit_canonical.bin", "golden")])
def test_reference_golden_roots_through_gpu(ctx, name, prompt_key):
    """golden_conformance.rs:253-261 and the frozen receipts, via the drop-in API."""
    r, layers = _pin_layers(name)
    a_list = [np.frombuffer(a, dtype=np.int8) for a, _ in layers]
    scale_a = [[struct.unpack("<f", struct.pack("<I", s))[0] for _, s in layers]]
    prompt = r["prompt"] if prompt_key is None else PINS["golden_e2e_verify"]["prompt"]
    h = V.commit_minimal_from_captures(a_list, _drain_scales(len(layers), [1], scale_a), len(layers), [1],
                                       [r["token_id"]], prompt.encode(), bytes.fromhex(r["sampling_seed"]),
                                       n_prompt_tokens=1, ctx=ctx)
    want = r["commitment"] if prompt_key is None else PINS["golden_e2e_verify"]
    assert h.merkle_root_hex() == want["merkle_root"]
    assert h.io_root_hex() == want["io_root"]
    if prompt_key is None:
        cj = json.loads(h.commitment_json())
        assert bytes(cj["prompt_hash"]).hex() == r["commitment"]["prompt_hash"]
        assert bytes(cj["seed_commitment"]).hex() == r["commitment"]["seed_commitment"]
        assert cj["n_tokens"] == 1 and cj["version"] == "V4" and cj["kv_roots"] == []
        assert bytes(h.io_hashes()[0].cpu().numpy()) == bytes.fromhex(r["commitment"]["io_root"])


def test_c1_io_chain_and_trace_root_match_golden(ctx):
    g = json.load(open(os.path.join(HERE, "golden", "c1_golden.json")))
    k, v, tok, pos, a, sc = c1_inputs()
    n, L = C1["n_tokens"], C1["n_layers"]
    # one forward pass per token (decode-shaped captures)
    a_list = [a[t, l] for t in range(n) for l in range(L)]
    scales = _drain_scales(L, [1] * n, sc)
    from tests import kvref
    from commitllm_b200._lib import VC_DTYPE_BF16
    view = kvref.Transcript(k, v, [n], VC_DTYPE_BF16).view(ctx.device)
    h = V.commit_minimal_from_captures(a_list, scales, L, [1] * n, [int(x) for x in tok], C1["prompt"].encode(),
                                       bytes.fromhex(C1["sampling_seed"]), n_prompt_tokens=1, kv_cache=view, ctx=ctx)
    assert h.merkle_root_hex() == g["merkle_root"]
    assert h.io_root_hex() == g["io_root"]
    assert h.kv_roots_hex() == g["kv_roots"]
    io = h.io_hashes().cpu().numpy()
    assert [bytes(x).hex() for x in io[:4]] == g["io_hashes_head"]
    assert bytes(io[-1]).hex() == g["io_hashes_last"]
    # openings against the committed roots
    for t in (0, 5, 127):
        p = h.retained_proof(t)
        leaf = bytes(h.leaf_hashes()[t].cpu().numpy())
        assert O.verify(bytes.fromhex(g["merkle_root"]), leaf, O.MerkleProof(t, [bytes.fromhex(s) for s in p["siblings"]]))
        p = h.io_proof(t)
        assert O.verify(bytes.fromhex(g["io_root"]), bytes(io[t]), O.MerkleProof(t, [bytes.fromhex(s) for s in p["siblings"]]))
    for o in g["kv_openings"][:4]:
        p = h.kv_proof(o["layer"], o["pos"])
        assert p["siblings"] == o["siblings"]


@pytest.mark.parametrize("hidden", [1, 3, 5, 16, 61, 64, 100, 4096])
@pytest.mark.parametrize("n_layers", [1, 3])
def test_retained_leaves_alignments(ctx, hidden, n_layers):
    """Layer records of hidden + 5 bytes put a_i8 rows at every alignment."""
    fwd = [3, 1, 2]
    n = sum(fwd)
    a = synth.activations_i8(hidden * 7 + n_layers, (n, n_layers, hidden))
    sc = synth.scales_f32(hidden, n * n_layers).reshape(n, n_layers)
    a_list = []
    t0 = 0
    for bs in fwd:
        for l in range(n_layers):
            a_list.append(np.ascontiguousarray(a[t0:t0 + bs, l]).reshape(-1))
        t0 += bs
    toks = list(range(100, 100 + n))
    h = V.commit_minimal_from_captures(a_list, _drain_scales(n_layers, fwd, sc), n_layers, fwd, toks, b"p",
                                       b"\x01" * 32, ctx=ctx)
    retained = [[O.RetainedLayerState(a[t, l].tobytes(), float(sc[t, l])) for l in range(n_layers)] for t in range(n)]
    com = O.commit_minimal(retained, toks, b"p", b"\x01" * 32)
    assert [bytes(x) for x in h.leaf_hashes().cpu().numpy()] == com.trace_leaves
    assert h.merkle_root_hex() == com.merkle_root.hex()
    assert h.io_root_hex() == com.io_root.hex()


def test_wraps_and_gen_start(ctx):
    """final_residual / lp_hidden / captured_logits binding (merkle.rs:170-241),
    logits offset by gen_start = n_prompt_tokens - 1 (prover/src/lib.rs:367-390)."""
    L, H, n = 2, 24, 7
    fwd = [4, 1, 1, 1]
    a = synth.activations_i8(3, (n, L, H))
    sc = synth.scales_f32(4, n * L).reshape(n, L)
    a_list = []
    t0 = 0
    for bs in fwd:
        for l in range(L):
            a_list.append(np.ascontiguousarray(a[t0:t0 + bs, l]).reshape(-1))
        t0 += bs
    fr = [synth.logits_f32(10 + t, 13) for t in range(n)]
    lp = [synth.activations_i8(20 + t, 18).view(np.uint8).astype(np.uint16) * 257 for t in range(5)]  # only 5 tokens
    logits = [synth.logits_f32(30 + t, 1001) for t in range(3)]                  # 3 generated tokens
    toks = [9, 8, 7, 6, 5, 4, 3]
    h = V.commit_minimal_from_captures(a_list, _drain_scales(L, fwd, sc), L, fwd, toks, b"wrap prompt", b"\x02" * 32,
                                       final_residuals=fr, n_prompt_tokens=5, lp_hidden_bf16=lp,
                                       captured_logits_f32=logits, ctx=ctx)
    retained = [[O.RetainedLayerState(a[t, l].tobytes(), float(sc[t, l])) for l in range(L)] for t in range(n)]
    com = O.commit_minimal(retained, toks, b"wrap prompt", b"\x02" * 32, final_residuals=fr, lp_hidden_bf16=lp,
                           captured_logits_f32=logits, n_prompt_tokens=5)
    assert [bytes(x) for x in h.leaf_hashes().cpu().numpy()] == com.trace_leaves
    assert h.merkle_root_hex() == com.merkle_root.hex()


def test_packed_equals_unpacked(ctx):
    """prover/src/lib.rs:2035-2083: packed and unpacked commits give equal roots."""
    L, H = 3, 40
    fwd = [5, 1, 1, 2]
    n = sum(fwd)
    a = synth.activations_i8(8, (n, L, H))
    sc = synth.scales_f32(9, n * L).reshape(n, L)
    a_list, packed = [], []
    t0 = 0
    for bs in fwd:
        for l in range(L):
            blk = np.ascontiguousarray(a[t0:t0 + bs, l]).reshape(-1)
            a_list.append(blk)
            packed.append(blk)
        t0 += bs
    scales = _drain_scales(L, fwd, sc)
    toks = list(range(n))
    fr = synth.logits_f32(99, (n, 6))
    h1 = V.commit_minimal_from_captures(a_list, scales, L, fwd, toks, b"x", b"\x03" * 32,
                                        final_residuals=list(fr), ctx=ctx)
    h2 = V.commit_minimal_packed(np.concatenate(packed), scales, L, H, fwd, toks, b"x", b"\x03" * 32,
                                 packed_final_res=fr.tobytes(), final_res_dim=6, ctx=ctx)
    assert h1.merkle_root_hex() == h2.merkle_root_hex()
    assert h1.io_root_hex() == h2.io_root_hex()


def test_x_attn_some_encoding(ctx):
    """The 0x01 || x_attn_i8 || f32le(scale_x_attn) branch of merkle.rs:151-157."""
    L, H, n = 2, 33, 5
    a = synth.activations_i8(40, (n, L, H))
    x = synth.activations_i8(41, (n, L, H))
    sa = synth.scales_f32(42, n * L).reshape(n, L)
    sx = synth.scales_f32(43, n * L).reshape(n, L)
    ad = ctx.to_device(a)
    xd = ctx.to_device(x)
    sad = ctx.to_device(sa)
    sxd = ctx.to_device(sx)
    # one forward pass of n rows; row stride is L*H for a/x and L for scales
    lay = C.TraceLayout(n_layers=L, hidden=H, fwd_rows=[n], tok_fwd=[0] * n, tok_row=list(range(n)),
                        a_rows=[[ad.data_ptr() + l * H for l in range(L)]], scale_a=[[sad.data_ptr() + 4 * l for l in range(L)]],
                        scale_stride=L, x_attn_rows=[[xd.data_ptr() + l * H for l in range(L)]],
                        scale_x_attn=[[sxd.data_ptr() + 4 * l for l in range(L)]], scale_x_stride=L)
    # a row of token t, layer l sits at t*L*H + l*H: pass stride via hidden trick is not possible,
    # so lay the rows out per layer instead
    a_pl = ctx.to_device(np.ascontiguousarray(a.transpose(1, 0, 2)))
    x_pl = ctx.to_device(np.ascontiguousarray(x.transpose(1, 0, 2)))
    lay.a_rows = [[a_pl.data_ptr() + l * n * H for l in range(L)]]
    lay.x_attn_rows = [[x_pl.data_ptr() + l * n * H for l in range(L)]]
    leaves = C.trace_leaves(ctx, lay)
    ctx.sync(timeout_ms=60000)
    retained = [[O.RetainedLayerState(a[t, l].tobytes(), float(sa[t, l]), x[t, l].tobytes(), float(sx[t, l]))
                 for l in range(L)] for t in range(n)]
    assert [bytes(v) for v in leaves.cpu().numpy()] == [O.hash_retained_state_direct(r) for r in retained]


@pytest.mark.parametrize("n", [1, 2, 3, 5, 8, 13, 28, 32, 129, 1000, 4097])
def test_build_trees_matches_oracle(ctx, n):
    rng = np.random.default_rng(n)
    leaves = rng.integers(0, 256, size=(n, 32), dtype=np.uint8)
    d = ctx.to_device(leaves)
    roots, trees = C.build_trees(ctx, d, [0, n])
    ctx.sync(timeout_ms=60000)
    nodes = vco.build_tree(leaves)
    assert bytes(roots[0].cpu().numpy()) == bytes(nodes[-1]) == vco.compute_root(leaves)
    assert np.array_equal(trees.nodes(0).cpu().numpy(), nodes)
    r2, _ = C.build_trees(ctx, d, [0, n], keep_trees=False)
    assert bytes(r2[0].cpu().numpy()) == bytes(nodes[-1])


def test_many_trees_one_launch(ctx):
    lens = [1, 7, 128, 129, 3000, 2]
    off = np.cumsum([0] + lens)
    leaves = np.random.default_rng(5).integers(0, 256, size=(off[-1], 32), dtype=np.uint8)
    roots, trees = C.build_trees(ctx, ctx.to_device(leaves), list(off))
    ctx.sync(timeout_ms=60000)
    for i in range(len(lens)):
        assert bytes(roots[i].cpu().numpy()) == vco.compute_root(leaves[off[i]:off[i + 1]])


def test_io_chain_multi_sequence(ctx):
    lens = [5, 0, 300, 1]
    off = np.cumsum([0] + lens)
    leaves = np.random.default_rng(6).integers(0, 256, size=(off[-1], 32), dtype=np.uint8)
    toks = synth.token_ids(7, int(off[-1]), 128256)
    prompts = [b"", b"a", b"prompt three" * 30, b"\x00\xff"]
    ph = C.prompt_hashes(ctx, prompts)
    io = C.io_chain(ctx, ctx.to_device(leaves), ctx.to_device(toks.view(np.int32)), ph, list(off))
    ctx.sync(timeout_ms=60000)
    io = io.cpu().numpy()
    for s in range(len(lens)):
        assert bytes(ph[s].cpu().numpy()) == O.hash_prompt(prompts[s])
        want = O.io_chain([bytes(x) for x in leaves[off[s]:off[s + 1]]], [int(t) for t in toks[off[s]:off[s + 1]]],
                          prompts[s])
        assert [bytes(x) for x in io[off[s]:off[s + 1]]] == want


def test_seed_commitments(ctx):
    seeds = np.random.default_rng(8).integers(0, 256, size=(9, 32), dtype=np.uint8)
    out = C.seed_commitments(ctx, ctx.to_device(seeds))
    ctx.sync(timeout_ms=60000)
    assert [bytes(x) for x in out.cpu().numpy()] == [O.hash_seed(bytes(s)) for s in seeds]


def test_verilm_rs_argument_errors(ctx):
    with pytest.raises(ValueError, match="sampling_seed"):
        V.commit_minimal_from_captures([b"\0" * 4], np.zeros(4, np.float32), 1, [1], [1], b"p", b"short", ctx=ctx)
    with pytest.raises(ValueError, match="scales"):
        V.commit_minimal_from_captures([b"\0" * 4], np.zeros(3, np.float32), 1, [1], [1], b"p", b"\0" * 32, ctx=ctx)
    with pytest.raises(ValueError, match="token_ids"):
        V.commit_minimal_from_captures([b"\0" * 4], np.zeros(4, np.float32), 1, [1], [1, 2], b"p", b"\0" * 32, ctx=ctx)
    with pytest.raises(ValueError, match="packed_a"):
        V.commit_minimal_packed(b"\0" * 5, np.zeros(4, np.float32), 1, 4, [1], [1], b"p", b"\0" * 32, ctx=ctx)
    with pytest.raises(ValueError, match="manifest missing tokenizer_hash"):   # extract_manifest, lib.rs:174-178
        V.commit_minimal_from_captures([b"\0" * 4], np.zeros(4, np.float32), 1, [1], [1], b"p", b"\0" * 32,
                                       manifest={"x": 1}, ctx=ctx)


def test_c4_shape_retained_leaves_through_trace_plan(ctx):
    """Full-width sampled-decode leaves (32 layers x 4096 a_i8 + x_attn, 128 256 f32 logits)
    laid out as the benchmark lays them ([step, layer, batch, hidden]), vs the oracle."""
    L, H, B, T, V = 32, 4096, 3, 4, 128256
    a = synth.activations_i8(61, (T, L, B, H))
    x = synth.activations_i8(62, (T, L, B, H))
    sa = synth.scales_f32(63, T * L * B).reshape(T, L, B)
    sx = synth.scales_f32(64, T * L * B).reshape(T, L, B)
    logits = synth.logits_f32(65, (B * T, V))
    ad, xd, sad, sxd, ld = (ctx.to_device(v) for v in (a, x, sa, sx, logits))
    t = np.arange(B * T)
    lay = C.TraceLayout(
        n_layers=L, hidden=H, fwd_rows=[B] * T, tok_fwd=t % T, tok_row=t // T,
        a_rows=[[ad.data_ptr() + ((k * L + l) * B) * H for l in range(L)] for k in range(T)],
        scale_a=[[sad.data_ptr() + 4 * ((k * L + l) * B) for l in range(L)] for k in range(T)], scale_stride=1,
        x_attn_rows=[[xd.data_ptr() + ((k * L + l) * B) * H for l in range(L)] for k in range(T)],
        scale_x_attn=[[sxd.data_ptr() + 4 * ((k * L + l) * B) for l in range(L)] for k in range(T)],
        scale_x_stride=1, logits=ld, tok_logits_row=t)
    plan = C.TracePlan(lay)
    out = ctx.empty(B * T, 32)
    plan.run(ctx, out)
    ctx.sync(timeout_ms=60000)
    got = [bytes(v) for v in out.cpu().numpy()]
    for i in range(B * T):
        s, k = i // T, i % T
        layers = [O.RetainedLayerState(a[k, l, s].tobytes(), float(sa[k, l, s]), x[k, l, s].tobytes(),
                                       float(sx[k, l, s])) for l in range(L)]
        assert got[i] == O.hash_retained_with_captured_logits(layers, None, None, logits[i])


def test_trace_kernel_paths_agree_at_their_boundaries(ctx):
    """vc_trace_leaves picks one of three kernels by token count (on 148 SMs:
    the two-warp split kernel up to 2 x 148 x 32 = 9 472 tokens, the
    one-thread kernel with a two-block prefetch below 3 x 148 CTAs of 128,
    the busy kernel above).  The same tokens hashed through each give the same
    leaves, mixed wraps in one warp included (every third token without
    logits, every fifth with a final residual), and a sample of them equals
    the oracle's."""
    n_sm = torch.cuda.get_device_properties(ctx.device).multi_processor_count
    L, H, V_ = 2, 200, 37
    n_big = 3 * n_sm * 128 + 5                                   # busy kernel
    g = torch.Generator(device=f"cuda:{ctx.device}").manual_seed(7)
    dev = f"cuda:{ctx.device}"
    a = torch.randint(-128, 128, (L, n_big, H), generator=g, device=dev, dtype=torch.int8)
    sa = torch.rand(L, n_big, generator=g, device=dev)
    lg = torch.randn(n_big, V_, generator=g, device=dev)
    fr = torch.randn(n_big, 11, generator=g, device=dev)

    def leaves(n):
        lay = C.TraceLayout(n_layers=L, hidden=H, fwd_rows=[n], tok_fwd=[0] * n, tok_row=list(range(n)),
                            a_rows=[[a[l].data_ptr() for l in range(L)]], scale_a=[[sa[l].data_ptr() for l in range(L)]],
                            scale_stride=1, logits=lg, tok_logits_row=[t if t % 3 else -1 for t in range(n)],
                            final_residual=fr, tok_fr_row=[t if t % 5 == 0 else -1 for t in range(n)])
        out = C.trace_leaves(ctx, lay)
        ctx.sync(60000)
        return out.cpu().numpy()

    n_split = 2 * n_sm * 32
    l_split = leaves(n_split)
    l_plain = leaves(n_split + 1)
    l_busy = leaves(n_big)
    assert np.array_equal(l_split, l_plain[:n_split]) and np.array_equal(l_plain, l_busy[: n_split + 1])
    a_h, sa_h, lg_h, fr_h = a.cpu().numpy(), sa.cpu().numpy(), lg.cpu().numpy(), fr.cpu().numpy()
    for t in (0, 1, 3, 5, 31, 32, n_split - 1, n_split, n_big - 1):
        layers = [O.RetainedLayerState(a_h[l, t].tobytes(), float(sa_h[l, t])) for l in range(L)]
        want = O.hash_retained_with_captured_logits(layers, fr_h[t] if t % 5 == 0 else None, None,
                                                    lg_h[t] if t % 3 else None)
        assert bytes(l_busy[t]) == want, t
