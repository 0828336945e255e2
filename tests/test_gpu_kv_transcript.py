"""compute_kv_transcript on the tensor cores vs the oracle, bit for bit.

The oracle restates crates/verilm-prover/src/lib.rs:207-329 with exact i32
accumulators, the reference's f64 operation order and the C library's
cos/sin; the CUDA path must reproduce every f64 bit, and the KV roots over
its rows must equal the oracle's.
"""
import numpy as np
import pytest
import torch

from commitllm_b200 import commit as C
from commitllm_b200._lib import VcValueError
from oracle import commit_oracle as O

pytestmark = pytest.mark.gpu


def make_case(seed, n_tok, n_layers, hidden, n_heads, head_dim, mode):
    rng = np.random.default_rng(seed)
    kv = n_heads * head_dim
    x = rng.integers(-128, 128, (n_tok, n_layers, hidden), dtype=np.int8)
    wk = [rng.integers(-128, 128, (kv, hidden), dtype=np.int8) for _ in range(n_layers)]
    wv = [rng.integers(-128, 128, (kv, hidden), dtype=np.int8) for _ in range(n_layers)]
    sx = (rng.random((n_tok, n_layers), dtype=np.float32) * np.float32(0.05) + np.float32(1e-3)).astype(np.float32)
    per_tensor = per_channel = biases = None
    rope = O.RopeScaling()
    theta = 500000.0
    if mode == "tensor":
        per_tensor = [(np.float32(rng.random() * 0.01), np.float32(rng.random() * 0.01)) for _ in range(n_layers)]
    elif mode == "channel_bias":
        per_channel = [((rng.random(kv, dtype=np.float32) * 0.01).astype(np.float32),
                        (rng.random(kv, dtype=np.float32) * 0.01).astype(np.float32)) for _ in range(n_layers)]
        biases = [(rng.standard_normal(kv).astype(np.float32), rng.standard_normal(kv).astype(np.float32))
                  for _ in range(n_layers)]
        rope, theta = None, 1000000.0
    elif mode == "mixed":
        # per-channel K only on even layers, V never: the rest falls back to per-tensor scales
        per_tensor = [(np.float32(0.003 * (l + 1)), np.float32(0.002)) for l in range(n_layers)]
        per_channel = [((rng.random(kv, dtype=np.float32) * 0.01).astype(np.float32), None) if l % 2 == 0 else None
                       for l in range(n_layers)]
        biases = [(None, rng.standard_normal(kv).astype(np.float32)) for _ in range(n_layers)]
        rope = O.RopeScaling(rope_type="linear", factor=4.0)
    return dict(x=x, wk=wk, wv=wv, sx=sx, n_heads=n_heads, head_dim=head_dim, per_tensor=per_tensor,
                per_channel=per_channel, biases=biases, rope=rope, theta=theta)


def oracle_of(c):
    return O.compute_kv_transcript(c["x"], c["wk"], c["wv"], c["sx"], c["n_heads"], c["head_dim"],
                                   per_tensor=c["per_tensor"], per_channel=c["per_channel"], biases=c["biases"],
                                   rope_theta=c["theta"], rope_scaling=c["rope"])


def gpu_inputs(ctx, c, token_major=True):
    dev = lambda a: None if a is None else ctx.to_device(a)
    if token_major:
        # the captures' order: one [n_tokens, n_layers, hidden] buffer, per-layer strided views
        X = ctx.to_device(c["x"])
        xs = [X[:, l, :] for l in range(X.shape[1])]
    else:
        X = ctx.to_device(np.ascontiguousarray(c["x"].transpose(1, 0, 2)))
        xs = X
    pair = lambda p: None if p is None else (dev(p[0]), dev(p[1]))
    rope = None
    if c["rope"] is not None:
        r = c["rope"]
        rope = C.RopeConfig(theta=c["theta"], scaling=r.rope_type, factor=r.factor,
                            low_freq_factor=r.low_freq_factor, high_freq_factor=r.high_freq_factor,
                            original_max_position_embeddings=r.original_max_position_embeddings)
    else:
        rope = C.RopeConfig(theta=c["theta"])
    return C.KvTranscriptInputs(
        x_attn=xs, wk=[dev(w) for w in c["wk"]], wv=[dev(w) for w in c["wv"]], scale_x=dev(c["sx"]),
        n_kv_heads=c["n_heads"], head_dim=c["head_dim"], per_tensor=c["per_tensor"],
        per_channel=None if c["per_channel"] is None else [pair(p) for p in c["per_channel"]],
        biases=None if c["biases"] is None else [pair(p) for p in c["biases"]], rope=rope), X


def same_bits(a, b):
    return np.array_equal(np.ascontiguousarray(a).view(np.uint64), np.ascontiguousarray(b).view(np.uint64))


CASES = [
    # n_tok, layers, hidden, kv heads, head_dim, mode
    (5, 2, 16, 2, 2, "toy"),              # the reference's toy model shape (hidden 16, kv_dim 4, d_head 2)
    (200, 2, 272, 2, 64, "tensor"),       # ragged positions, hidden not a multiple of 128, kv_dim < 256
    (130, 3, 256, 4, 128, "channel_bias"),
    (64, 2, 128, 3, 96, "mixed"),         # head_dim 96: 192-channel tiles, kv_dim 288
    (300, 1, 512, 8, 128, "tensor"),      # Llama-style kv_dim 1024
    (33, 2, 64, 2, 8, "tensor"),          # small heads: 8-wide RoPE groups
    (160, 2, 3584, 4, 128, "channel_bias"),  # Qwen2.5-7B shapes: hidden 3584, 4 x 128 KV heads, biases
    (129, 1, 8192, 8, 128, "tensor"),     # Llama-70B hidden 8192: 64 K-blocks per tile
    (70, 2, 512, 2, 256, "channel_bias"),  # head_dim 256 (the largest): one head per 256-channel tile
    (1, 2, 128, 8, 128, "tensor"),        # a single position
]


@pytest.mark.parametrize("case", CASES, ids=[f"{c[-1]}-{c[0]}x{c[2]}-h{c[3]}x{c[4]}" for c in CASES])
def test_transcript_matches_oracle(ctx, case):
    n_tok, L, hidden, nh, hd, mode = case
    c = make_case(n_tok * 1000 + hidden + nh * 7 + hd, n_tok, L, hidden, nh, hd, mode)
    k_ref, v_ref = oracle_of(c)
    inp, _keep = gpu_inputs(ctx, c, token_major=(n_tok % 2 == 0))
    k, v = C.kv_transcript(ctx, inp)
    ctx.sync(60000)
    k, v = k.cpu().numpy(), v.cpu().numpy()
    assert same_bits(v, v_ref), "v_deq differs"
    assert same_bits(k, k_ref), "k_roped differs"
    # the KV roots over the transcript equal the oracle's trees
    roots, _ = C.kv_commit(ctx, C.kv_transcript_view(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda()),
                           keep_trees=False)
    roots = roots.cpu().numpy().reshape(L, 32)
    for l in range(L):
        assert bytes(roots[l]) == O.kv_tree_for_layer(l, k_ref[l], v_ref[l]).root


def test_transcript_llama8b_layer_sample(ctx):
    """Llama-3-8B shapes (hidden 4096, 8 x 128 KV heads, llama3 RoPE) for 4096
    positions: two layers, every f64 bit checked on a sample of positions."""
    rng = np.random.default_rng(7)
    n_tok, L, hidden, nh, hd = 4096, 2, 4096, 8, 128
    kv = nh * hd
    x = rng.integers(-128, 128, (L, n_tok, hidden), dtype=np.int8)
    wk = [rng.integers(-128, 128, (kv, hidden), dtype=np.int8) for _ in range(L)]
    wv = [rng.integers(-128, 128, (kv, hidden), dtype=np.int8) for _ in range(L)]
    sx = (rng.random((n_tok, L), dtype=np.float32) * np.float32(0.05)).astype(np.float32)
    pt = [(np.float32(0.0021), np.float32(0.0017)), (np.float32(0.0009), np.float32(0.0013))]
    inp = C.KvTranscriptInputs(x_attn=ctx.to_device(x), wk=[ctx.to_device(w) for w in wk],
                               wv=[ctx.to_device(w) for w in wv], scale_x=ctx.to_device(sx), n_kv_heads=nh,
                               head_dim=hd, per_tensor=pt,
                               rope=C.RopeConfig(theta=500000.0, scaling="llama3"))
    k, v = C.kv_transcript(ctx, inp)
    ctx.sync(60000)
    sel = np.sort(rng.choice(n_tok, 96, replace=False))
    sel[-1] = n_tok - 1
    k_ref, v_ref = O.compute_kv_transcript(x[:, sel].transpose(1, 0, 2), wk, wv, sx[sel], nh, hd, per_tensor=pt,
                                           rope_theta=500000.0, rope_scaling=O.RopeScaling())
    # the oracle numbered the sampled rows 0..95: redo its RoPE at the true positions
    inv = O.scaled_inv_freq(hd, 500000.0, O.RopeScaling())
    cos, sin = O.rope_cos_sin(n_tok, inv)
    k_np, v_np = k.cpu().numpy(), v.cpu().numpy()
    for l in range(L):
        assert same_bits(v_np[l, sel], v_ref[l])
        acc = O.matmul_i32(wk[l], x[l, sel])
        f = acc.astype(np.float64) * (float(pt[l][0]) * sx[sel, l].astype(np.float64)[:, None])
        half = hd // 2
        for h in range(nh):
            lo, hi = f[:, h * hd:h * hd + half], f[:, h * hd + half:(h + 1) * hd]
            c_, s_ = cos[sel], sin[sel]
            assert same_bits(k_np[l, sel, h * hd:h * hd + half], lo * c_ - hi * s_)
            assert same_bits(k_np[l, sel, h * hd + half:(h + 1) * hd], hi * c_ + lo * s_)


def test_transcript_zero_tokens_and_errors(ctx):
    c = make_case(3, 4, 1, 32, 2, 8, "tensor")
    inp, _ = gpu_inputs(ctx, c, token_major=False)
    inp.x_attn = [inp.x_attn[0][:0]]
    inp.scale_x = inp.scale_x[:0]
    k, v = C.kv_transcript(ctx, inp)
    assert k.shape == (1, 0, 16)
    bad = make_case(4, 4, 1, 24, 2, 8, "tensor")      # hidden not a multiple of 16
    inp, _ = gpu_inputs(ctx, bad, token_major=False)
    with pytest.raises(VcValueError):
        C.kv_transcript(ctx, inp)
    ctx.sync(10000)


@pytest.mark.parametrize("mode", ["per_tensor", "per_channel_bias"])
def test_verilm_rs_weight_provider_path(ctx, mode):
    """commit_minimal_from_captures with x_attn_inputs + weight_provider commits the
    recomputed transcript (verilm-py/src/lib.rs:941-970): kv_roots and KV openings
    equal the oracle's compute_kv_transcript + hash_kv_entry trees."""
    from commitllm_b200 import verilm_rs as V
    rng = np.random.default_rng(31)
    L, H, nh, hd = 3, 64, 2, 64
    kv = nh * hd
    fwd = [5, 1, 1, 1]
    n = sum(fwd)
    a = rng.integers(-128, 128, (n, L, H), dtype=np.int8)
    x = rng.integers(-128, 128, (n, L, H), dtype=np.int8)
    sq = (rng.random((n, L), dtype=np.float32) * 0.05 + 1e-3).astype(np.float32)   # qkv block = scale_x_attn
    so = (rng.random((n, L), dtype=np.float32) * 0.05 + 1e-3).astype(np.float32)   # o_proj block = scale_a
    a_list, x_list, scales = [], [], []
    t0 = 0
    for bs in fwd:
        for l in range(L):
            a_list.append(np.ascontiguousarray(a[t0:t0 + bs, l]).reshape(-1))
            x_list.append(ctx.to_device(np.ascontiguousarray(x[t0:t0 + bs, l]).reshape(-1)))
            scales += list(sq[t0:t0 + bs, l]) + list(so[t0:t0 + bs, l]) + [0.5] * bs + [0.25] * bs
        t0 += bs
    wk = [rng.integers(-128, 128, (kv, H), dtype=np.int8) for _ in range(L)]
    wv = [rng.integers(-128, 128, (kv, H), dtype=np.int8) for _ in range(L)]
    scal = dict(rope_type="llama3", factor=8.0, low_freq_factor=1.0, high_freq_factor=4.0,
                original_max_position_embeddings=8192)
    cfg = V.ModelConfig(L, H, nh, hd, 500000.0, scal)
    if mode == "per_tensor":
        ws = [[0.01, 0.002 * (l + 1), 0.003, 0.01, 0.01, 0.01, 0.01] for l in range(L)]
        wp = V.WeightProvider(cfg, [ctx.to_device(w) for w in wk], [ctx.to_device(w) for w in wv], weight_scales=ws)
        ref_kw = dict(per_tensor=[(np.float32(s[1]), np.float32(s[2])) for s in ws])
    else:
        pc = [[None, (rng.random(kv, dtype=np.float32) * 0.01).astype(np.float32),
               (rng.random(kv, dtype=np.float32) * 0.01).astype(np.float32), None, None, None, None]
              for _ in range(L)]
        qb = [[None, rng.standard_normal(kv).astype(np.float32), rng.standard_normal(kv).astype(np.float32)]
              for _ in range(L)]
        wp = V.WeightProvider(cfg, [ctx.to_device(w) for w in wk], [ctx.to_device(w) for w in wv],
                              per_channel_weight_scales=[[None if c is None else ctx.to_device(c) for c in row]
                                                         for row in pc],
                              qkv_biases=qb)
        ref_kw = dict(per_channel=[(row[1], row[2]) for row in pc], biases=[(row[1], row[2]) for row in qb])
    toks = [int(t) for t in rng.integers(0, 128256, n)]
    h = V.commit_minimal_from_captures(a_list, np.array(scales, np.float32), L, fwd, toks, b"kv prompt", b"\x07" * 32,
                                       weight_provider=wp, x_attn_inputs=x_list, ctx=ctx)
    k_ref, v_ref = O.compute_kv_transcript(x, wk, wv, sq, nh, hd, rope_theta=500000.0,
                                           rope_scaling=O.RopeScaling(), **ref_kw)
    assert h.kv_roots_hex() == [O.kv_tree_for_layer(l, k_ref[l], v_ref[l]).root.hex() for l in range(L)]
    # the trace leaves do not contain x_attn (prover/src/lib.rs:162-167)
    retained = [[O.RetainedLayerState(a[t, l].tobytes(), float(so[t, l])) for l in range(L)] for t in range(n)]
    com = O.commit_minimal(retained, toks, b"kv prompt", b"\x07" * 32)
    assert h.merkle_root_hex() == com.merkle_root.hex() and h.io_root_hex() == com.io_root.hex()
    # openings carry the recomputed KvEntry rows
    layers, ent, sib = h.kv_openings(n - 1, [0, 2])
    assert layers == [0, 2]
    for i, l in enumerate(layers):
        assert same_bits(ent[i, :, 0], k_ref[l]) and same_bits(ent[i, :, 1], v_ref[l])
    with pytest.raises(ValueError):
        V.commit_minimal_from_captures(a_list, np.array(scales, np.float32), L, fwd, toks, b"p", b"\x07" * 32,
                                       weight_provider=wp, x_attn_inputs=x_list, ctx=ctx,
                                       kv_cache=C.kv_transcript_view(torch.from_numpy(k_ref).cuda(),
                                                                     torch.from_numpy(v_ref).cuda()))
