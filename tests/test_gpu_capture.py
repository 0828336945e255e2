"""Captures kept on the device (commitllm_b200.capture) commit to the same
roots as the reference's host-copy capture path, and as the oracle.

A model stand-in runs a prefill pass and decode passes, each making four
quantized matmuls per layer (qkv_proj, o_proj, gate_up_proj, down_proj) on the
device through the wrapped op, and a sampler that captures the last logits
row of each pass.  The same calls are also copied to the host as the
reference's hook does (capture.py:733-763; sampler.py:153-154) and committed
through ``commit_minimal_from_captures`` from host buffers, and through the
oracle's ``build_retained_from_captures`` + ``commit_minimal``.  The device
captures are committed in place (``commit_captures``) and through
``drain_minimal`` + ``commit_minimal_from_captures`` with device views.
"""
import json

import numpy as np
import pytest
import torch

from commitllm_b200 import capture as K
from commitllm_b200 import receipt as R
from commitllm_b200 import verilm_rs as V
from oracle import commit_oracle as O
from tests.test_gpu_receipt import MANIFEST

pytestmark = pytest.mark.gpu

PROMPT = b"device capture prompt"
SEED = bytes(range(32))


def _serve(buf, lcap, L, H, passes, vocab, seed):
    """Run the passes; returns the host copies the reference's hook keeps:
    (o_inputs, scales, x_attn_inputs, logits rows)."""
    dev = buf.device
    g = torch.Generator(device=dev).manual_seed(seed)
    op = buf.wrap(lambda a, b, sa, sb, dt, bias: torch.zeros(a.shape[0], 8, dtype=dt, device=a.device))
    calls = []
    for bs in passes:
        for _l in range(L):
            for p in range(K.PROJS_PER_LAYER):
                a = torch.randint(-128, 128, (bs, H), generator=g, device=dev, dtype=torch.int8)
                s = torch.rand(bs, 1, generator=g, device=dev) * 0.05 + 1e-3
                out = op(a, None, s, None, torch.bfloat16, None)
                assert out.shape == (bs, 8)
                calls.append((p, a, s))
        lg = (torch.randn(bs, vocab, generator=g, device=dev) * 4).to(torch.bfloat16)
        lcap.capture(lg)
        calls.append(("logits", lg[-1].float(), None))
    torch.cuda.synchronize()
    o = [c[1].cpu().numpy().reshape(-1) for c in calls if c[0] == K.O_PROJ_IDX]
    x = [c[1].cpu().numpy().reshape(-1) for c in calls if c[0] == K.QKV_PROJ_IDX]
    s = np.concatenate([c[2].cpu().numpy().reshape(-1) for c in calls if c[0] != "logits"]).astype(np.float32)
    lg = [c[1].cpu().numpy() for c in calls if c[0] == "logits"]
    return o, s, x, lg


def _weights(L, H, nh, hd, dev):
    g = torch.Generator(device=dev).manual_seed(77)
    kv = nh * hd
    wk = [torch.randint(-128, 128, (kv, H), generator=g, device=dev, dtype=torch.int8) for _ in range(L)]
    wv = [torch.randint(-128, 128, (kv, H), generator=g, device=dev, dtype=torch.int8) for _ in range(L)]
    cfg = V.ModelConfig(L, H, nh, hd, 500000.0, dict(rope_type="llama3", factor=8.0, low_freq_factor=1.0,
                                                     high_freq_factor=4.0, original_max_position_embeddings=8192))
    ws = [[0.01, 0.002 * (l + 1), 0.003, 0.01, 0.01, 0.01, 0.01] for l in range(L)]
    return V.WeightProvider(cfg, wk, wv, weight_scales=ws)


@pytest.mark.parametrize("L,H,n_prompt,n_dec", [(3, 256, 37, 23), (2, 4096, 130, 5), (4, 272, 1, 9)])
def test_device_captures_commit_like_the_host_captures(ctx, L, H, n_prompt, n_dec):
    vocab = 1000
    passes = [n_prompt] + [1] * n_dec
    n = sum(passes)
    buf = K.DeviceCaptureBuffer(L, H, capacity_tokens=16, device=f"cuda:{ctx.device}")
    lcap = K.DeviceLogitsCapture(vocab, capacity=4, device=f"cuda:{ctx.device}")
    o, s, x, lg = _serve(buf, lcap, L, H, passes, vocab, seed=L * 1000 + n)
    caps, logits = buf.drain(), lcap.drain()
    assert caps.fwd_batch_sizes == passes and caps.n_tokens == n and logits.shape == (len(passes), vocab)
    rng = np.random.default_rng(n)
    ids = [int(t) for t in rng.integers(0, 128256, n + 1)]
    h_dev = K.commit_captures(caps, ids[1:], PROMPT, SEED, n_prompt_tokens=n_prompt, logits=logits,
                              manifest=MANIFEST, ctx=ctx)
    h_host = V.commit_minimal_from_captures(o, s, L, passes, ids[1:], PROMPT, SEED, manifest=MANIFEST,
                                            n_prompt_tokens=n_prompt, captured_logits_f32=lg, ctx=ctx)
    assert h_dev.merkle_root_hex() == h_host.merkle_root_hex()
    assert h_dev.io_root_hex() == h_host.io_root_hex()
    assert json.loads(h_dev.commitment_json()) == json.loads(h_host.commitment_json())
    retained = O.build_retained_from_captures([bytes(e) for e in o], s, L, passes)
    com = O.commit_minimal(retained, ids[1:], PROMPT, SEED, captured_logits_f32=lg, n_prompt_tokens=n_prompt)
    assert h_dev.merkle_root_hex() == com.merkle_root.hex() and h_dev.io_root_hex() == com.io_root.hex()
    # the receipt of a generated token reads the device captures
    t = n - 1
    assert R.zstd_decompress(h_dev.audit_v4_binary(t)[4:]) == R.zstd_decompress(h_host.audit_v4_binary(t)[4:])


def test_drain_minimal_feeds_the_drop_in(ctx):
    L, H, vocab = 3, 128, 64
    passes = [20, 1, 1, 1]
    dev = f"cuda:{ctx.device}"
    buf = K.DeviceCaptureBuffer(L, H, device=dev)
    lcap = K.DeviceLogitsCapture(vocab, device=dev)
    o, s, x, lg = _serve(buf, lcap, L, H, passes, vocab, seed=5)
    o_dev, s_dev, count, x_dev, witnessed = buf.drain_minimal()
    assert witnessed is None and count == len(passes) * L * 4 and len(o_dev) == len(passes) * L
    assert all(t.is_cuda for t in o_dev + x_dev) and s_dev.is_cuda
    ids = list(range(100, 100 + sum(passes) + 1))
    h_dev = V.commit_minimal_from_captures(o_dev, s_dev, L, passes, ids[1:], PROMPT, SEED, n_prompt_tokens=20,
                                           captured_logits_f32=lcap.drain(), ctx=ctx)
    h_host = V.commit_minimal_from_captures(o, s, L, passes, ids[1:], PROMPT, SEED, n_prompt_tokens=20,
                                            captured_logits_f32=lg, ctx=ctx)
    assert h_dev.merkle_root_hex() == h_host.merkle_root_hex() and h_dev.io_root_hex() == h_host.io_root_hex()


def test_device_x_attn_commits_the_reference_kv_transcript(ctx):
    """With a weight provider, K/V are recomputed from the captured x_attn (one
    pass) and the kv_roots equal those of the host-copy path."""
    L, H, nh, hd = 2, 512, 4, 128
    passes = [45, 1, 1, 1, 1]
    dev = f"cuda:{ctx.device}"
    buf = K.DeviceCaptureBuffer(L, H, device=dev)
    lcap = K.DeviceLogitsCapture(32, device=dev)
    o, s, x, lg = _serve(buf, lcap, L, H, passes, 32, seed=9)
    wp = _weights(L, H, nh, hd, dev)
    caps = buf.drain()
    ids = list(range(7, 7 + sum(passes) + 1))
    h_dev = K.commit_captures(caps, ids[1:], PROMPT, SEED, n_prompt_tokens=45, weight_provider=wp, ctx=ctx)
    h_host = V.commit_minimal_from_captures(o, s, L, passes, ids[1:], PROMPT, SEED, n_prompt_tokens=45,
                                            weight_provider=wp, x_attn_inputs=x, ctx=ctx)
    assert h_dev.has_captured_x_attn()
    assert h_dev.kv_roots_hex() == h_host.kv_roots_hex() and len(h_dev.kv_roots_hex()) == L
    assert h_dev.merkle_root_hex() == h_host.merkle_root_hex()
    sx = np.array([s[i] for i in caps.scale_index(K.QKV_PROJ_IDX).reshape(-1)], np.float32).reshape(-1, L)
    xa = np.stack([np.concatenate([x[f * L + l].reshape(-1, H) for f in range(len(passes))]) for l in range(L)], 1)
    k_ref, v_ref = O.compute_kv_transcript(xa, [w.cpu().numpy() for w in wp._w["Wk"]],
                                           [w.cpu().numpy() for w in wp._w["Wv"]], sx, nh, hd,
                                           rope_theta=500000.0, rope_scaling=O.RopeScaling(),
                                           per_tensor=[(np.float32(r[1]), np.float32(r[2]))
                                                       for r in wp.weight_scales()])
    assert h_dev.kv_roots_hex() == [O.kv_tree_for_layer(l, k_ref[l], v_ref[l]).root.hex() for l in range(L)]
    with pytest.raises(ValueError, match="x_attn"):
        K.commit_captures(K.DeviceCaptures(a=caps.a, x_attn=None, scales=caps.scales,
                                           fwd_batch_sizes=caps.fwd_batch_sizes, call_count=caps.call_count,
                                           n_layers=L), ids[1:], PROMPT, SEED, weight_provider=wp, ctx=ctx)


def test_trailing_eos_pass_trimmed(ctx):
    """The server drops a trailing pass that produced no committed token
    (server.py:916-935); the trimmed device captures commit like the trimmed
    host lists."""
    L, H, vocab = 2, 64, 40
    passes = [6, 1, 1, 1]
    dev = f"cuda:{ctx.device}"
    buf = K.DeviceCaptureBuffer(L, H, device=dev)
    lcap = K.DeviceLogitsCapture(vocab, device=dev)
    o, s, x, lg = _serve(buf, lcap, L, H, passes, vocab, seed=13)
    caps = buf.drain().trim_last_pass()
    logits = lcap.drain()[:-1]
    n = sum(passes) - 1
    ids = list(range(3, 3 + n + 1))
    h_dev = K.commit_captures(caps, ids[1:], PROMPT, SEED, n_prompt_tokens=6, logits=logits, ctx=ctx)
    h_host = V.commit_minimal_from_captures(o[:-L], s[: s.size - 4 * L], L, passes[:-1], ids[1:], PROMPT, SEED,
                                            n_prompt_tokens=6, captured_logits_f32=lg[:-1], ctx=ctx)
    assert h_dev.merkle_root_hex() == h_host.merkle_root_hex() and h_dev.io_root_hex() == h_host.io_root_hex()


@pytest.mark.parametrize("defer", [0, 3, 8192])
@pytest.mark.parametrize("chunks", [[9], [5, 4]], ids=["prefill", "chunked-prefill"])
def test_online_capture_matches_the_offline_commit(ctx, defer, chunks):
    """The request hashed pass by pass while it decodes (OnlineCapture) has the
    roots of the offline commit of the same captures, and of the oracle.  Small
    slabs make both the capture and the logits slab grow mid-request, which
    flushes the deferred passes first."""
    from commitllm_b200.online import OnlineCommitter
    L, H, vocab, n_dec = 3, 256, 500, 12
    n_prompt = sum(chunks)
    dev = f"cuda:{ctx.device}"
    buf = K.DeviceCaptureBuffer(L, H, capacity_tokens=4, device=dev)
    lcap = K.DeviceLogitsCapture(vocab, capacity=2, device=dev)
    oc = OnlineCommitter(ctx, max_slots=2, max_tokens=64, defer_tokens=defer)
    onl = K.OnlineCapture(buf, oc, lcap, slot=1)
    rng = np.random.default_rng(17 + defer + len(chunks))
    all_ids = [int(x) for x in rng.integers(0, 32000, n_prompt + n_dec + 1)]
    onl.begin(PROMPT, SEED, all_ids[:n_prompt])
    g = torch.Generator(device=dev).manual_seed(99)
    op = buf.wrap(lambda a, b, sa, sb, dt, bias: None)
    host_o, host_s, host_lg = [], [], []
    done = 0
    for bs in chunks + [1] * n_dec:
        for _l in range(L):
            for p in range(K.PROJS_PER_LAYER):
                a = torch.randint(-128, 128, (bs, H), generator=g, device=dev, dtype=torch.int8)
                s = torch.rand(bs, 1, generator=g, device=dev) * 0.05 + 1e-3
                op(a, None, s, None, torch.bfloat16, None)
                if p == K.O_PROJ_IDX:
                    host_o.append(a.cpu().numpy().reshape(-1))
                host_s.append(s.cpu().numpy().reshape(-1))
        done += bs
        if done < n_prompt:
            onl.after_sampling()                       # a prefill chunk: nothing sampled
            continue
        lg = (torch.randn(1, vocab, generator=g, device=dev) * 4).to(torch.bfloat16)
        lcap.capture(lg)
        host_lg.append(lg[0].float().cpu().numpy())
        onl.after_sampling(torch.tensor([all_ids[done]], device=dev))
    dig, caps = onl.finish()
    logits = lcap.drain()
    off = K.commit_captures(caps, all_ids[1:], PROMPT, SEED, n_prompt_tokens=n_prompt, logits=logits, ctx=ctx)
    ctx.sync(20000)
    assert bytes(dig["merkle_root"].cpu().numpy()).hex() == off.merkle_root_hex()
    assert bytes(dig["io_root"].cpu().numpy()).hex() == off.io_root_hex()
    retained = O.build_retained_from_captures([bytes(e) for e in host_o], np.concatenate(host_s), L,
                                              chunks + [1] * n_dec)
    com = O.commit_minimal(retained, all_ids[1:], PROMPT, SEED, captured_logits_f32=host_lg,
                           n_prompt_tokens=n_prompt)
    assert off.merkle_root_hex() == com.merkle_root.hex() and off.io_root_hex() == com.io_root.hex()
