"""The device capture hook (commitllm_b200.capture) on the CPU: call counting,
token-major slabs, scale order, the drain's checks and the op-table patch,
against the layout the reference's capture path produces
(sidecar/verilm/capture.py:414-480, 863-947; server.py:885-935).

The buffer is torch plumbing and runs on any device; the GPU test
(test_gpu_capture.py) commits the captures and compares the roots."""
import types

import numpy as np
import pytest
import torch

from commitllm_b200 import capture as K


def _request(buf, L, hidden, o_dim, passes, seed=0, real=None):
    """Drive ``passes`` forward passes through the wrapped op; returns the
    per-call inputs in call order: [(pass, layer, proj, a, scale)]."""
    g = torch.Generator().manual_seed(seed)
    calls = []
    op = buf.wrap(real or (lambda a, b, sa, sb, dt, bias: ("out", a.shape[0])))
    for f, bs in enumerate(passes):
        for l in range(L):
            for p in range(K.PROJS_PER_LAYER):
                dim = o_dim if p == K.O_PROJ_IDX else hidden
                a = torch.randint(-128, 128, (bs, dim), generator=g, dtype=torch.int8)
                s = torch.rand(bs, 1, generator=g) + 0.01
                out = op(a, None, s, None, torch.bfloat16, None)
                assert out == ("out", bs)          # the real kernel's output, unchanged
                calls.append((f, l, p, a, s))
    return calls


def test_token_major_slabs_and_drain_order():
    L, H, O = 3, 16, 12
    passes = [5, 1, 1, 2, 1]
    buf = K.DeviceCaptureBuffer(L, H, o_dim=O, capacity_tokens=2, device="cpu")   # forces two growths
    calls = _request(buf, L, H, O, passes)
    caps = buf.drain()
    n = sum(passes)
    assert caps.n_tokens == n and caps.fwd_batch_sizes == passes
    assert caps.call_count == len(calls) == len(passes) * L * 4
    # scales: every call's rows, in call order (the reference's drain order)
    assert torch.equal(caps.scales, torch.cat([c[4].reshape(-1) for c in calls]))
    t0 = {f: sum(passes[:f]) for f in range(len(passes))}
    for f, l, p, a, s in calls:
        rows = slice(t0[f], t0[f] + passes[f])
        if p == K.O_PROJ_IDX:
            assert torch.equal(caps.a[rows, l], a)
        if p == K.QKV_PROJ_IDX:
            assert torch.equal(caps.x_attn[rows, l], a)
    # per-projection scales, token-major
    for proj in (K.O_PROJ_IDX, K.QKV_PROJ_IDX):
        got = caps.proj_scales(proj)
        for f, l, p, a, s in calls:
            if p == proj:
                assert torch.equal(got[t0[f]:t0[f] + passes[f], l], s.reshape(-1))
    # drain_minimal's entry order: (pass, layer)
    o = caps.o_inputs()
    assert len(o) == len(passes) * L
    want = [c[3] for c in calls if c[2] == K.O_PROJ_IDX]
    assert all(torch.equal(x, y) for x, y in zip(o, want))
    assert len(caps.x_attn_inputs()) == len(passes) * L


def test_scale_index_matches_the_reference_split():
    """scale_index reproduces commit_minimal_from_captures' split of the flat
    scales (o_proj block at cursor + bs of each entry, cursor += 4 bs)."""
    L = 4
    passes = [7, 1, 3, 1]
    caps = K.DeviceCaptures(a=torch.zeros(sum(passes), L, 8, dtype=torch.int8), x_attn=None,
                            scales=torch.zeros(sum(passes) * 4 * L), fwd_batch_sizes=passes,
                            call_count=len(passes) * 4 * L, n_layers=L)
    idx = caps.scale_index(K.O_PROJ_IDX)
    cursor, t0 = 0, 0
    for bs in passes:
        for l in range(L):
            for r in range(bs):
                assert idx[t0 + r, l] == cursor + bs + r
            cursor += 4 * bs
        t0 += bs
    assert cursor == caps.scales.numel()


def test_trim_last_pass():
    L, H = 2, 8
    passes = [4, 1, 1]
    buf = K.DeviceCaptureBuffer(L, H, device="cpu")
    calls = _request(buf, L, H, H, passes, seed=3)
    caps = buf.drain()
    t = caps.trim_last_pass()
    assert t.fwd_batch_sizes == [4, 1] and t.n_tokens == 5
    assert t.call_count == caps.call_count - 4 * L
    assert torch.equal(t.scales, caps.scales[: caps.scales.numel() - 4 * L])
    assert torch.equal(t.a, caps.a[:5]) and torch.equal(t.x_attn, caps.x_attn[:5])
    assert torch.equal(t.proj_scales(K.O_PROJ_IDX), caps.proj_scales(K.O_PROJ_IDX)[:5])


def test_drain_checks_and_counter():
    L, H = 2, 8
    buf = K.DeviceCaptureBuffer(L, H, device="cpu", capture_x_attn=False)
    op = buf.wrap(lambda *a: None)
    a = torch.zeros(3, H, dtype=torch.int8)
    for _ in range(5):                       # a partial pass
        op(a, None, torch.ones(3, 1), None)
    with pytest.raises(RuntimeError, match="not a multiple of calls_per_fwd"):
        buf.drain()
    # counter drift: a pass whose calls disagree on the row count
    buf.reset_counter()
    op(torch.zeros(2, H, dtype=torch.int8), None, torch.ones(2, 1), None)
    for _ in range(4 * L - 1):
        op(torch.zeros(1, H, dtype=torch.int8), None, torch.ones(1, 1), None)
    with pytest.raises(RuntimeError, match="counter drift"):
        buf.drain()
    # per-tensor scales cannot be split per row (server.py:905-913)
    buf.reset_counter()
    for _ in range(4 * L):
        op(torch.zeros(2, H, dtype=torch.int8), None, torch.ones(1), None)
    with pytest.raises(RuntimeError, match="scales count"):
        buf.drain()
    # disabled: nothing recorded, output still returned
    buf.reset_counter()
    buf.enabled = False
    assert buf.wrap(lambda *a: 7)(a, None, torch.ones(3, 1), None) == 7
    assert buf.stats()["buffered"] == 0
    buf.enabled = True
    caps = buf.drain()
    assert caps.n_tokens == 0 and caps.call_count == 0 and caps.x_attn is None
    # wrong row width
    op(torch.zeros(1, H, dtype=torch.int8), None, torch.ones(1, 1), None)
    with pytest.raises(ValueError, match="o_proj input rows"):
        op(torch.zeros(1, H + 1, dtype=torch.int8), None, torch.ones(1, 1), None)


def test_drain_hands_over_the_slabs():
    L, H = 2, 8
    buf = K.DeviceCaptureBuffer(L, H, device="cpu")
    _request(buf, L, H, H, [3, 1], seed=5)
    first = buf.drain()
    keep = first.a.clone()
    _request(buf, L, H, H, [2], seed=6)     # a second request writes fresh slabs
    second = buf.drain()
    assert torch.equal(first.a, keep)
    assert second.n_tokens == 2 and first.a.data_ptr() != second.a.data_ptr()


def test_install_patches_the_op_table():
    L, H = 1, 4
    ops = types.SimpleNamespace(cutlass_scaled_mm=lambda a, b, sa, sb, dt=None, bias=None: "real")
    orig = ops.cutlass_scaled_mm
    buf = K.DeviceCaptureBuffer(L, H, device="cpu")
    buf.install(ops)
    assert ops.cutlass_scaled_mm is not orig
    with pytest.raises(RuntimeError, match="already"):
        K.DeviceCaptureBuffer(L, H, device="cpu").install(ops)
    for _ in range(4):
        assert ops.cutlass_scaled_mm(torch.zeros(1, H, dtype=torch.int8), None, torch.ones(1), None) == "real"
    buf.uninstall()
    assert ops.cutlass_scaled_mm is orig
    assert buf.drain().fwd_batch_sizes == [1]


def test_request_bookkeeping():
    buf = K.DeviceCaptureBuffer(1, 4, device="cpu")
    assert buf.end_request() is None
    buf.begin_request("r1", [1, 2, 3])
    assert buf.stats()["in_request"]
    out = buf.end_request([9])
    assert out["request_id"] == "r1" and out["prompt_token_ids"] == [1, 2, 3]
    assert out["generated_token_ids"] == [9] and out["ended_at"] >= out["started_at"]
    buf.set_sync_mode("event")
    with pytest.raises(ValueError):
        buf.set_sync_mode("bogus")
    buf.wait_for_transfers()


def test_layer_count_and_configure_from_model():
    class Layer(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.o_proj = torch.nn.Linear(2, 2)

    class Model(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.model = torch.nn.Module()
            self.model.layers = torch.nn.ModuleList([Layer() for _ in range(5)])
            self.config = types.SimpleNamespace(hidden_size=64, num_attention_heads=4, head_dim=8)

    m = Model()
    assert K.layer_count(m) == 5
    buf = K.configure_from_model(m, device="cpu")
    assert (buf.n_layers, buf.hidden, buf.o_dim) == (5, 64, 32)
    assert K.layer_count(torch.nn.Linear(2, 2)) == 0


def test_logits_capture_keeps_float32_rows():
    cap = K.DeviceLogitsCapture(vocab=10, capacity=1, device="cpu")
    g = torch.Generator().manual_seed(1)
    rows = [torch.randn(3, 10, generator=g).to(torch.bfloat16) for _ in range(5)]
    for r in rows:
        cap.capture(r)
    cap.capture(torch.randn(10, generator=g))
    assert len(cap) == 6
    out = cap.drain()
    assert out.dtype == torch.float32 and out.shape == (6, 10)
    for i, r in enumerate(rows):
        assert torch.equal(out[i], r[-1].float())     # what the sampler's .float() keeps
    assert len(cap) == 0 and cap.drain().shape == (0, 10)
    with pytest.raises(ValueError):
        cap.capture(torch.zeros(11))


class _FakeCommitter:
    """Records what OnlineCapture hands an OnlineCommitter (CPU: no hashing)."""

    def __init__(self):
        self.steps, self.flushes, self.opened = [], 0, None
        self.ctx = types.SimpleNamespace(device=None, stream=None)

    def open(self, slot, prompt, seed, n_prompt_tokens=None):
        self.opened = (slot, prompt, n_prompt_tokens)

    def step(self, slots, layout, ids):
        self.steps.append((list(slots), layout, ids.tolist()))

    def flush(self):
        self.flushes += 1

    def close(self, slot):
        return {"slot": slot, "n_tokens": sum(len(s[0]) for s in self.steps)}


def test_online_capture_token_ids_and_rows():
    """Row t of the request commits all_ids[t + 1]: prompt tokens from the
    prompt, the last row of a pass that reaches the end of the prompt the
    sampled token; logits rows bind from gen_start = n_prompt - 1; a growing
    slab flushes the committer first."""
    L, H, vocab = 2, 8, 5
    buf = K.DeviceCaptureBuffer(L, H, capacity_tokens=3, device="cpu")
    lg = K.DeviceLogitsCapture(vocab, capacity=1, device="cpu")
    fc = _FakeCommitter()
    onl = K.OnlineCapture(buf, fc, lg, slot=3)
    prompt_ids = [11, 12, 13, 14, 15, 16]
    onl.begin(b"p", bytes(32), prompt_ids)
    assert fc.opened == (3, b"p", 6)
    op = buf.wrap(lambda *a: None)

    def run_pass(bs):
        for _ in range(L * K.PROJS_PER_LAYER):
            op(torch.zeros(bs, H, dtype=torch.int8), None, torch.ones(bs, 1), None)

    run_pass(4)                                   # prefill chunk ending inside the prompt
    onl.after_sampling()
    assert fc.steps[-1][0] == [3] * 4 and fc.steps[-1][2] == [12, 13, 14, 15]
    run_pass(2)                                   # the prompt's last two rows; the last one samples
    lg.capture(torch.zeros(vocab))
    with pytest.raises(ValueError, match="next_token"):
        onl.after_sampling()
    onl.after_sampling(21)
    assert fc.steps[-1][2] == [16, 21]
    assert fc.steps[-1][1].tok_logits_row == [-1, 0]
    for tok in (22, 23):                          # decode steps
        run_pass(1)
        lg.capture(torch.zeros(vocab))
        onl.after_sampling(tok)
    assert [s[2] for s in fc.steps[2:]] == [[22], [23]]
    assert [s[1].tok_logits_row for s in fc.steps[2:]] == [[1], [2]]
    assert fc.flushes >= 2                        # the capture slab and the logits slab both grew
    out, caps = onl.finish()
    assert out["n_tokens"] == 8 and caps.n_tokens == 8
    with pytest.raises(RuntimeError, match="begin"):
        onl.after_sampling(1)


def test_online_capture_refuses_a_dirty_buffer_and_a_partial_pass():
    buf = K.DeviceCaptureBuffer(1, 4, device="cpu")
    op = buf.wrap(lambda *a: None)
    op(torch.zeros(1, 4, dtype=torch.int8), None, torch.ones(1, 1), None)
    onl = K.OnlineCapture(buf, _FakeCommitter())
    with pytest.raises(RuntimeError, match="drain or reset"):
        onl.begin(b"p", bytes(32), [1, 2])
    buf.reset()
    buf.reset_counter()
    onl.begin(b"p", bytes(32), [1, 2])
    with pytest.raises(RuntimeError, match="no forward pass"):
        onl.after_sampling(5)
    op(torch.zeros(2, 4, dtype=torch.int8), None, torch.ones(2, 1), None)   # one call of a 4-call pass
    with pytest.raises(RuntimeError, match="between forward passes"):
        onl.after_sampling(5)


def test_configure_from_a_transformers_llama():
    """The layer count and geometry of a real module tree (a tiny random
    Llama from transformers), as configure_from_model reads them."""
    transformers = pytest.importorskip("transformers")
    cfg = transformers.LlamaConfig(num_hidden_layers=3, hidden_size=64, intermediate_size=128,
                                   num_attention_heads=4, num_key_value_heads=2, vocab_size=100)
    model = transformers.LlamaForCausalLM(cfg)
    assert K.layer_count(model) == 3
    buf = K.configure_from_model(model, device="cpu")
    assert (buf.n_layers, buf.hidden, buf.o_dim, buf.calls_per_fwd) == (3, 64, 64, 12)


def test_install_on_another_op():
    ops = types.SimpleNamespace(int8_scaled_mm=lambda a, b, sa, sb, dt=None, bias=None: "other")
    buf = K.DeviceCaptureBuffer(1, 4, device="cpu")
    buf.install(ops, name="int8_scaled_mm")
    for _ in range(4):
        assert ops.int8_scaled_mm(torch.zeros(2, 4, dtype=torch.int8), None, torch.ones(2, 1), None) == "other"
    buf.uninstall()
    assert buf.drain().fwd_batch_sizes == [2]


def test_verilm_rs_capture_hook_bookkeeping():
    """verilm_rs.CaptureHook (verilm-py/src/lib.rs:1842-1960): projection index
    by call counting, scales drained in call order (prefill [bs, 1] beside
    decode [1]), counters."""
    from commitllm_b200 import verilm_rs as V
    hook = V.CaptureHook(calls_per_fwd=8, projs_per_layer=4, o_proj_idx=1)
    seen = [hook.record(torch.full((3, 1), float(i))) for i in range(8)]          # a 3-row prefill pass
    seen += [hook.record(torch.full((1,), float(8 + i))) for i in range(8)]       # a decode pass
    assert seen == [0, 1, 2, 3] * 4
    assert (hook.call_counter, hook.total_captured, hook.minimal_call_count) == (16, 16, 16)
    arr, count = hook.drain_scales()
    assert count == 16 and arr.dtype == np.float32
    assert arr.tolist() == [float(i) for i in range(8) for _ in range(3)] + [float(8 + i) for i in range(8)]
    assert hook.minimal_call_count == 0 and hook.drain_scales()[1] == 0
    hook.reset_counter()
    assert hook.record(torch.ones(1)) == 0 and hook.total_captured == 17
    dev, count = hook.drain_scales_device()
    assert count == 1 and isinstance(dev, torch.Tensor) and dev.tolist() == [1.0]
