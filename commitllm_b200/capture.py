"""Device-resident capture of the committed inputs: the hook side of the
reference's capture path, without device-to-host copies.

The reference's vLLM plugin (sidecar/verilm/capture.py:243-947) wraps
``cutlass_scaled_mm``, names each call by counting (every layer makes four
calls in the order qkv_proj, o_proj, gate_up_proj, down_proj;
capture.py:53-58, 912-924), copies every o_proj input, and with x_attn capture
on every qkv_proj input, to a pinned host slab with a non-blocking
device-to-host copy (capture.py:352-373, 733-763), keeps each call's per-row
activation scale as a GPU reference until the drain (capture.py:414-480), and
its sampler pulls each sampled logits row to the host with a synchronous
``.float().cpu()`` (sampler.py:153-154).  The commit then copies all of it
back to a device.

Here the captures stay in HBM, already in the layout the commit kernels read:

* o_proj inputs in a token-major slab ``[tokens, layers, o_dim]`` int8, and
  qkv_proj inputs (x_attn) in ``[tokens, layers, hidden]`` int8: one
  device-to-device copy per captured call, issued on the stream that produced
  the input, so the hook neither synchronises nor touches host memory;
* scales as the reference keeps them, GPU references, concatenated on the
  device at the drain, in the reference's drain order (per forward pass, per
  layer, the qkv, o_proj, gate_up and down blocks of batch-size rows);
* logits rows (:class:`DeviceLogitsCapture`) in a ``[rows, vocab]`` float32
  slab.

:func:`commit_captures` hands the slabs to
:func:`commitllm_b200.verilm_rs.commit_request` in place (the fast path: a
handful of launches per request).  :meth:`DeviceCaptureBuffer.drain_minimal`
returns the reference's tuple, with device views, for
``verilm_rs.commit_minimal_from_captures``.

Like the reference's hook this needs an eagerly executed model: a replayed
CUDA graph runs no Python, so no capture call happens (capture.py:29-32).
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Callable, List, Optional, Sequence

import numpy as np
import torch

# capture.py:53-58
PROJ_SEQUENCE = ("qkv_proj", "o_proj", "gate_up_proj", "down_proj")
PROJS_PER_LAYER = len(PROJ_SEQUENCE)
QKV_PROJ_IDX = 0
O_PROJ_IDX = 1


def layer_count(model) -> int:
    """The layer count ``configure_from_model`` derives (capture.py:116-135):
    one more than the largest integer that follows a ``layers`` component of a
    module name; 0 when no name has one."""
    top = -1
    for name, _ in model.named_modules():
        parts = name.split(".")
        for i, part in enumerate(parts[:-1]):
            if part == "layers":
                try:
                    top = max(top, int(parts[i + 1]))
                except ValueError:
                    pass
    return top + 1


@dataclass
class DeviceCaptures:
    """One request's captures, in device memory.

    a: int8 ``[n_tokens, n_layers, o_dim]``, the o_proj input row of each
    token and layer; x_attn: int8 ``[n_tokens, n_layers, hidden]`` (qkv_proj
    inputs) or None; scales: float32, every captured call's per-row scales
    in the reference's drain order; fwd_batch_sizes: rows of each forward
    pass; call_count: captured matmul calls; ready: an event recorded after
    the last capture (None off CUDA).
    """
    a: torch.Tensor
    x_attn: Optional[torch.Tensor]
    scales: torch.Tensor
    fwd_batch_sizes: List[int]
    call_count: int
    n_layers: int
    ready: Optional[torch.cuda.Event] = None

    @property
    def n_tokens(self) -> int:
        return int(self.a.shape[0])

    def scale_index(self, proj: int) -> np.ndarray:
        """``[n_tokens, n_layers]`` int64: where token t's layer-l scale of
        projection ``proj`` sits in :attr:`scales` (verilm-py/src/lib.rs:859-885:
        entry (pass f, layer l) holds ``[B qkv | B o_proj | B gate_up | B down]``)."""
        bs = np.asarray(self.fwd_batch_sizes, dtype=np.int64)
        n, L = self.n_tokens, self.n_layers
        if int(bs.sum()) != n:
            raise ValueError("fwd_batch_sizes do not add up to the captured tokens")
        pass_base = np.concatenate([[0], np.cumsum(bs * PROJS_PER_LAYER * L)[:-1]]).astype(np.int64)
        tok_pass = np.repeat(np.arange(len(bs)), bs)
        row = np.arange(n, dtype=np.int64) - np.repeat(np.cumsum(bs) - bs, bs)
        lay = np.arange(L, dtype=np.int64)
        return (pass_base[tok_pass][:, None] + (lay[None, :] * PROJS_PER_LAYER + proj) * bs[tok_pass][:, None]
                + row[:, None])

    def proj_scales(self, proj: int) -> torch.Tensor:
        """float32 ``[n_tokens, n_layers]`` on the scales' device: each token's
        per-row scale of projection ``proj`` (:data:`O_PROJ_IDX` for the
        retained state's ``scale_a``, :data:`QKV_PROJ_IDX` for
        ``scale_x_attn``), gathered on the device."""
        idx = torch.from_numpy(self.scale_index(proj).reshape(-1))
        if self.scales.is_cuda:
            idx = idx.pin_memory().to(self.scales.device, non_blocking=True)
        return self.scales.index_select(0, idx).view(self.n_tokens, self.n_layers)

    def trim_last_pass(self) -> "DeviceCaptures":
        """These captures without their last forward pass: the server's
        trailing-EOS trim (server.py:916-935), which drops the pass that
        produced no committed token."""
        if not self.fwd_batch_sizes:
            raise ValueError("no forward pass to trim")
        bs = self.fwd_batch_sizes[-1]
        per_pass = PROJS_PER_LAYER * self.n_layers
        n = self.n_tokens - bs
        return DeviceCaptures(a=self.a[:n], x_attn=None if self.x_attn is None else self.x_attn[:n],
                              scales=self.scales[: self.scales.numel() - per_pass * bs],
                              fwd_batch_sizes=self.fwd_batch_sizes[:-1], call_count=self.call_count - per_pass,
                              n_layers=self.n_layers, ready=self.ready)

    def _entries(self, t: Optional[torch.Tensor]) -> List[torch.Tensor]:
        if t is None:
            return []
        out, t0 = [], 0
        for bs in self.fwd_batch_sizes:
            for l in range(self.n_layers):
                out.append(t[t0:t0 + bs, l])
            t0 += bs
        return out

    def o_inputs(self) -> List[torch.Tensor]:
        """One ``[rows, o_dim]`` device view per (forward pass, layer), the
        order of the reference's ``drain_minimal`` (capture.py:414-480)."""
        return self._entries(self.a)

    def x_attn_inputs(self) -> List[torch.Tensor]:
        """One ``[rows, hidden]`` device view per (forward pass, layer), or []."""
        return self._entries(self.x_attn)


class DeviceCaptureBuffer:
    """The reference's ``CaptureBuffer`` in minimal mode (capture.py:243-845)
    with device slabs in place of the pinned host slab.

    n_layers: transformer layers (four captured calls each); hidden: bytes of a
    qkv_proj input row; o_dim: bytes of an o_proj input row (default hidden);
    capture_x_attn: also keep qkv_proj inputs (the reference's server default);
    capacity_tokens: initial slab rows (the slabs double when a request needs
    more); device: where the slabs live (a CUDA device in serving).

    Call :meth:`record` after each matmul, or :meth:`install` to wrap
    ``vllm._custom_ops.cutlass_scaled_mm``.  :meth:`drain` hands the request's
    slabs to the caller and starts the next request on fresh ones, so the
    committed captures stay valid for later audits.
    """

    def __init__(self, n_layers: int, hidden: int, *, o_dim: Optional[int] = None, capture_x_attn: bool = True,
                 capacity_tokens: int = 4096, device=None):
        if n_layers <= 0 or hidden <= 0:
            raise ValueError("n_layers and hidden must be positive")
        self.n_layers = int(n_layers)
        self.calls_per_fwd = self.n_layers * PROJS_PER_LAYER
        self.hidden = int(hidden)
        self.o_dim = int(o_dim) if o_dim is not None else self.hidden
        self.capture_x_attn = bool(capture_x_attn)
        self._capacity = max(1, int(capacity_tokens))
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device)
        self._enabled = True
        self.total_captured = 0
        self._counter = 0
        self._installed = None
        self.before_grow: Optional[Callable[[], None]] = None
        self._request_id: Optional[str] = None
        self._prompt_ids: List[int] = []
        self._request_start = 0.0
        self._new_request_state()

    def _new_request_state(self):
        self._a = None
        self._x = None
        self._scales: list = []
        self._fwd: List[int] = []
        self._cursor = 0
        self._bs = 0
        self._calls = 0
        self._drift: Optional[str] = None

    # ---------------------------------------------------------------- switches

    @property
    def enabled(self) -> bool:
        return self._enabled

    @enabled.setter
    def enabled(self, value: bool):
        self._enabled = bool(value)

    def set_sync_mode(self, mode: str) -> None:
        """Accepted for the reference's interface (capture.py:324-350); the
        captures make no device-to-host transfer, so there is nothing to sync."""
        if mode not in ("global", "event"):
            raise ValueError(f"unknown sync mode {mode!r}")

    def reset_counter(self) -> None:
        """Realign the call counter before a request (capture.py:765-781)."""
        self._counter = 0

    # ------------------------------------------------------------------ hook

    def _reserve(self, rows: int) -> None:
        if self._a is not None and rows <= self._a.shape[0]:
            return
        if self._a is not None and self.before_grow is not None:
            self.before_grow()          # work that addresses the current slabs runs before they move
        old = 0 if self._a is None else int(self._a.shape[0])
        cap = max(self._capacity, 2 * old, rows)
        a = torch.empty(cap, self.n_layers, self.o_dim, dtype=torch.int8, device=self.device)
        x = (torch.empty(cap, self.n_layers, self.hidden, dtype=torch.int8, device=self.device)
             if self.capture_x_attn else None)
        if self._cursor:
            a[: self._cursor].copy_(self._a[: self._cursor])
            if x is not None:
                x[: self._cursor].copy_(self._x[: self._cursor])
        self._a, self._x = a, x

    def record(self, a: torch.Tensor, scale_a: torch.Tensor) -> None:
        """The capture half of ``_wrapped_cutlass_scaled_mm`` (capture.py:863-947)
        for one matmul: ``a`` its int8 input ``[rows, dim]``, ``scale_a`` its
        per-row activation scales."""
        if not self._enabled:
            return
        idx = self._counter % self.calls_per_fwd
        self._counter += 1
        layer, proj = divmod(idx, PROJS_PER_LAYER)
        rows = int(a.shape[0])
        if idx == 0:
            self._bs = rows
            self._reserve(self._cursor + rows)
        elif rows != self._bs and self._drift is None:
            self._drift = (f"call {self._counter - 1} ({PROJ_SEQUENCE[proj]} of layer {layer}) has {rows} rows, "
                           f"its forward pass {self._bs}: counter drift (reset_counter before each request)")
        self._scales.append(scale_a)
        self._calls += 1
        self.total_captured += 1
        if self._drift is None:
            c = self._cursor
            if proj == O_PROJ_IDX:
                if a.numel() != rows * self.o_dim:
                    raise ValueError(f"o_proj input rows hold {a.numel() // max(rows, 1)} bytes, expected {self.o_dim}")
                self._a[c:c + rows, layer].copy_(a.reshape(rows, self.o_dim).view(torch.int8), non_blocking=True)
            elif proj == QKV_PROJ_IDX and self._x is not None:
                if a.numel() != rows * self.hidden:
                    raise ValueError(f"qkv_proj input rows hold {a.numel() // max(rows, 1)} bytes, "
                                     f"expected {self.hidden}")
                self._x[c:c + rows, layer].copy_(a.reshape(rows, self.hidden).view(torch.int8), non_blocking=True)
        if idx == self.calls_per_fwd - 1:
            self._fwd.append(self._bs)
            self._cursor += self._bs

    def wrap(self, real: Callable) -> Callable:
        """``real`` (``cutlass_scaled_mm``'s signature) followed by :meth:`record`;
        its output is returned unchanged."""
        buf = self

        def wrapped(a, b, scale_a, scale_b, out_dtype=torch.bfloat16, bias=None):
            out = real(a, b, scale_a, scale_b, out_dtype, bias)
            if buf._enabled:
                buf.record(a, scale_a)
            return out

        wrapped.__wrapped__ = real
        wrapped._device_capture = self
        return wrapped

    def install(self, ops=None, name: str = "cutlass_scaled_mm") -> None:
        """Wrap ``ops.<name>`` (``vllm._custom_ops.cutlass_scaled_mm`` by default),
        as the reference's ``register`` does (capture.py:982-1033).  Any op with
        the argument order (a, b, scale_a, scale_b, out_dtype, bias) can be
        wrapped: vLLM's CUTLASS op refuses int8 on SM100, so an engine that runs
        its W8A8 matmuls on B200 through another int8 GEMM installs the wrapper
        on that op."""
        if self._installed is not None:
            raise RuntimeError("this capture buffer is already installed")
        if ops is None:
            import vllm._custom_ops as ops  # the serving engine's op table
        cur = getattr(ops, name)
        if getattr(cur, "_device_capture", None) is not None:
            raise RuntimeError(f"{name} is already wrapped by a capture buffer")
        setattr(ops, name, self.wrap(cur))
        self._installed = (ops, name, cur)

    def uninstall(self) -> None:
        if self._installed is not None:
            ops, name, cur = self._installed
            setattr(ops, name, cur)
            self._installed = None

    # --------------------------------------------------------------- requests

    def begin_request(self, request_id: str, prompt_token_ids: Optional[List[int]] = None) -> None:
        """capture.py:783-790."""
        self._request_id = request_id
        self._prompt_ids = list(prompt_token_ids or [])
        self._request_start = time.monotonic()

    def end_request(self, generated_token_ids: Optional[List[int]] = None) -> Optional[dict]:
        """capture.py:792-812; the captures themselves come from :meth:`drain`."""
        if self._request_id is None:
            return None
        out = {"request_id": self._request_id, "prompt_token_ids": self._prompt_ids,
               "generated_token_ids": list(generated_token_ids or []), "entries": [],
               "started_at": self._request_start, "ended_at": time.monotonic()}
        self._request_id = None
        self._prompt_ids = []
        return out

    def wait_for_transfers(self) -> None:
        """Nothing to wait for: no capture leaves the device (capture.py:814-830)."""

    def stats(self) -> dict:
        return {"buffered": self._cursor, "total_captured": self.total_captured, "enabled": self._enabled,
                "sync_mode": "device", "transfers_pending": False, "in_request": self._request_id is not None}

    def reset(self) -> None:
        """Discard what was captured since the last drain."""
        self._new_request_state()

    def drain(self) -> DeviceCaptures:
        """The request's captures; the slabs now belong to the result and the
        next capture starts on fresh ones.  Call it on the stream that ran the
        forward passes (its ``ready`` event is recorded there).  Raises, as the
        reference's server does (server.py:885-913), when the call count is not
        a whole number of forward passes or the counter drifted."""
        drift, calls, fwd, cursor = self._drift, self._calls, self._fwd, self._cursor
        a, x, scales = self._a, self._x, self._scales
        self._new_request_state()
        if drift is not None:
            raise RuntimeError(drift)
        if calls % self.calls_per_fwd != 0:
            raise RuntimeError(f"Capture count {calls} not a multiple of calls_per_fwd {self.calls_per_fwd}")
        if scales:
            s = torch.cat([t.reshape(-1).to(torch.float32) for t in scales])
        else:
            s = torch.empty(0, dtype=torch.float32, device=self.device)
        expected = sum(bs * PROJS_PER_LAYER * self.n_layers for bs in fwd)
        if s.numel() != expected:
            raise RuntimeError(f"scales count ({s.numel()}) != expected ({expected}): per-row scales expected "
                               f"(fwd_batch_sizes={fwd})")
        if a is None:
            a = torch.empty(0, self.n_layers, self.o_dim, dtype=torch.int8, device=self.device)
            x = (torch.empty(0, self.n_layers, self.hidden, dtype=torch.int8, device=self.device)
                 if self.capture_x_attn else None)
        ready = None
        if self.device.type == "cuda":
            ready = torch.cuda.Event()
            ready.record(torch.cuda.current_stream(self.device))
        return DeviceCaptures(a=a[:cursor], x_attn=None if x is None else x[:cursor], scales=s,
                              fwd_batch_sizes=list(fwd), call_count=calls, n_layers=self.n_layers, ready=ready)

    def drain_minimal(self):
        """The reference's ``drain_minimal`` tuple (capture.py:414-480):
        ``(o_inputs, scales, call_count, x_attn_inputs, witnessed_scores)`` with
        device views and a device scales tensor; witnessed scores (the attention
        score witness) are not captured here and come back None."""
        caps = self.drain()
        return caps.o_inputs(), caps.scales, caps.call_count, caps.x_attn_inputs(), None


def configure_from_model(model, **kw) -> DeviceCaptureBuffer:
    """A capture buffer sized from a model, as ``configure_from_model`` reads
    it (capture.py:116-166): the layer count from module names, ``hidden`` from
    ``config.hidden_size`` and the o_proj row from heads x head_dim."""
    n = layer_count(model)
    if n == 0:
        raise ValueError("could not detect the layer count from the model's module names")
    cfg = getattr(model, "config", None)
    if cfg is None:
        raise ValueError("the model has no config")
    hidden = int(getattr(cfg, "hidden_size", 0))
    heads = int(getattr(cfg, "num_attention_heads", 0))
    head_dim = int(getattr(cfg, "head_dim", 0) or (hidden // heads if heads else 0))
    return DeviceCaptureBuffer(n, hidden, o_dim=heads * head_dim or hidden, **kw)


class DeviceLogitsCapture:
    """The sampler's logits capture (sampler.py:146-154) into a device slab:
    each sampled row (the last row of a 2-D logits tensor) is converted to
    float32 and copied on the device, with no host transfer and no sync."""

    def __init__(self, vocab: int, capacity: int = 4096, device=None):
        self.vocab = int(vocab)
        self._capacity = max(1, int(capacity))
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device)
        self._rows: Optional[torch.Tensor] = None
        self._n = 0
        self.before_grow: Optional[Callable[[], None]] = None

    def __len__(self) -> int:
        return self._n

    def capture(self, logits: torch.Tensor) -> None:
        row = logits[-1] if logits.dim() == 2 else logits
        if row.numel() != self.vocab:
            raise ValueError(f"logits row holds {row.numel()} values, vocab is {self.vocab}")
        if self._rows is None or self._n >= self._rows.shape[0]:
            if self._rows is not None and self.before_grow is not None:
                self.before_grow()
            old = 0 if self._rows is None else int(self._rows.shape[0])
            rows = torch.empty(max(self._capacity, 2 * old), self.vocab, dtype=torch.float32, device=self.device)
            if self._n:
                rows[: self._n].copy_(self._rows[: self._n])
            self._rows = rows
        self._rows[self._n].copy_(row.reshape(-1), non_blocking=True)
        self._n += 1

    def drain(self) -> torch.Tensor:
        """float32 ``[rows, vocab]`` of this request; the slab now belongs to the result."""
        out = (self._rows[: self._n] if self._rows is not None
               else torch.empty(0, self.vocab, dtype=torch.float32, device=self.device))
        self._rows, self._n = None, 0
        return out

    def reset(self) -> None:
        self._rows, self._n = None, 0


def commit_captures(caps: DeviceCaptures, token_ids, prompt, sampling_seed, *, n_prompt_tokens=None,
                    logits: Optional[torch.Tensor] = None, manifest=None, kv_cache=None, weight_provider=None,
                    ctx=None):
    """Commit one request's device captures in place: the commitment
    ``commit_minimal_from_captures`` makes from the same captures
    (verilm-py/src/lib.rs:800-985), through
    :func:`commitllm_b200.verilm_rs.commit_request` with no copy of a, x_attn or
    the logits.  token_ids: ``all_token_ids[1:]`` (one per captured token);
    logits: float32 ``[generated tokens, vocab]`` (:class:`DeviceLogitsCapture`);
    weight_provider: recompute and commit K/V from the captured x_attn, as the
    reference does; kv_cache: commit the device KV cache instead."""
    from . import commit as C
    from . import verilm_rs as V
    if not caps.a.is_cuda:
        raise ValueError("the captures must be in CUDA memory")
    ctx = ctx or C.Context(device=caps.a.device.index)
    if caps.ready is not None:
        ctx.stream.wait_event(caps.ready)
    held = [t for t in (caps.a, caps.x_attn, caps.scales, logits) if t is not None]
    for t in held:
        t.record_stream(ctx.stream)
    with torch.cuda.stream(ctx.stream):
        sa = caps.proj_scales(O_PROJ_IDX)
        sx = None
        if weight_provider is not None:
            if caps.x_attn is None:
                raise ValueError("a weight_provider needs captured x_attn (capture_x_attn=True)")
            sx = caps.proj_scales(QKV_PROJ_IDX)
    return V.commit_request(caps.a, sa, token_ids, prompt, sampling_seed, n_prompt_tokens=n_prompt_tokens,
                            captured_logits_f32=logits, kv_cache=kv_cache, manifest=manifest,
                            x_attn=caps.x_attn if weight_provider is not None else None, scale_x_attn=sx,
                            weight_provider=weight_provider, ctx=ctx)


class OnlineCapture:
    """One request hashed while it decodes, straight from the device captures.

    Joins :class:`DeviceCaptureBuffer` (and optionally
    :class:`DeviceLogitsCapture`) to an
    :class:`commitllm_b200.online.OnlineCommitter`: after each forward pass
    and its sampling, :meth:`after_sampling` hands the pass's captured rows --
    o_proj inputs and scales in place, the logits row of a generated token --
    to the committer, which hashes the retained leaves and extends the IO
    chain (now, or batched with later passes when deferred).  :meth:`finish`
    builds the trace and IO trees, so after generation only the trees remain
    (the reference hashes everything after generation,
    crates/verilm-prover/src/lib.rs:336-499).  The roots equal those of
    :func:`commit_captures` over the same captures.  Deferred passes address
    the slabs, so a slab that has to grow first flushes the committer.
    """

    def __init__(self, buf: DeviceCaptureBuffer, committer, logits: Optional[DeviceLogitsCapture] = None,
                 slot: int = 0):
        self.buf, self.oc, self.logits, self.slot = buf, committer, logits, int(slot)
        buf.before_grow = self._flush
        if logits is not None:
            logits.before_grow = self._flush
        self._open = False

    def _flush(self) -> None:
        # hash the queued passes, and let the capturing stream reuse the old slab's
        # memory only after the committer's stream has read it
        import torch as _t
        self.oc.flush()
        if self.buf.device.type == "cuda":
            _t.cuda.current_stream(self.buf.device).wait_stream(self.oc.ctx.stream)

    def begin(self, prompt: bytes, sampling_seed: bytes, prompt_token_ids: Sequence[int]) -> None:
        """Start the request (the prompt's token ids, as ``all_token_ids[:n_prompt]``)."""
        if not prompt_token_ids:
            raise ValueError("the prompt needs at least one token")
        if self.buf._cursor or self.buf._calls:
            raise RuntimeError("the capture buffer holds another request's captures: drain or reset it first")
        self.oc.open(self.slot, prompt, sampling_seed, n_prompt_tokens=len(prompt_token_ids))
        self.buf.reset_counter()
        self.prompt_ids = [int(t) for t in prompt_token_ids]
        self.n_prompt = len(self.prompt_ids)
        self.done = 0
        self._next_pass = 0
        self._open = True

    def after_sampling(self, next_token=None) -> None:
        """Commit the rows of the forward pass(es) captured since the last call.
        Row t commits ``all_token_ids[t + 1]``: a prompt token, or -- for the
        last row of a pass that reached the end of the prompt -- the token just
        sampled (``next_token``: an int or a one-element CUDA tensor; not
        needed after a prefill chunk that ends inside the prompt)."""
        import torch as _t
        if not self._open:
            raise RuntimeError("begin() first")
        buf = self.buf
        if buf._drift is not None:
            raise RuntimeError(buf._drift)
        if buf._calls % buf.calls_per_fwd != 0:
            raise RuntimeError("after_sampling() between forward passes only")
        t0, t1 = self.done, buf._cursor
        n = t1 - t0
        if n <= 0:
            raise RuntimeError("no forward pass was captured since the last call")
        from . import commit as C
        dev = buf._a.device
        L, H = buf.n_layers, buf.o_dim
        # (pass, row) of the new tokens; the o_proj scale of row r of pass f, layer l
        # is call f * 4L + 4l + O_PROJ_IDX of the request
        rows = []
        for f in range(self._next_pass, len(buf._fwd)):
            rows += [(f, r) for r in range(buf._fwd[f])]
        self._next_pass = len(buf._fwd)
        a_rows, s_rows = [], []
        for i, (f, r) in enumerate(rows):
            t = t0 + i
            a_rows.append([buf._a[t, l].data_ptr() for l in range(L)])
            srow = []
            for l in range(L):
                k = f * buf.calls_per_fwd + PROJS_PER_LAYER * l + O_PROJ_IDX
                sc = buf._scales[k]
                if sc.dtype != _t.float32 or not sc.is_contiguous():
                    sc = buf._scales[k] = sc.to(_t.float32).contiguous()
                srow.append(sc.data_ptr() + 4 * r)
            s_rows.append(srow)
        lay = C.TraceLayout(n_layers=L, hidden=H, fwd_rows=[1] * n, tok_fwd=list(range(n)), tok_row=[0] * n,
                            a_rows=a_rows, scale_a=s_rows, scale_stride=1)
        gen_start = self.n_prompt - 1
        if self.logits is not None and self.logits._rows is not None:
            lay.logits = self.logits._rows
            lay.tok_logits_row = [t - gen_start if gen_start <= t < gen_start + len(self.logits) else -1
                                  for t in range(t0, t1)]
        known = []
        for t in range(t0, t1):
            if t + 1 < self.n_prompt:
                known.append(self.prompt_ids[t + 1])
            elif t != t1 - 1:
                raise RuntimeError("only the last row of a pass can commit a generated token")
        ids = _t.tensor(known, dtype=_t.int32).to(dev, non_blocking=True) if known else None
        if len(known) < n:
            if next_token is None:
                raise ValueError("this pass ends with a generated token: pass next_token")
            last = (next_token.reshape(1).to(device=dev, dtype=_t.int32) if isinstance(next_token, _t.Tensor)
                    else _t.tensor([int(next_token)], dtype=_t.int32).to(dev, non_blocking=True))
            ids = _t.cat([ids, last]) if ids is not None else last
        # the committer's stream reads what the model's stream captured
        if dev.type == "cuda":
            self.oc.ctx.stream.wait_stream(_t.cuda.current_stream(dev))
        self.oc.step([self.slot] * n, lay, ids)
        self.done = t1

    def finish(self):
        """Build the request's trees.  Returns ``(digests, captures)``: the
        committer's device digests (``merkle_root``, ``io_root``, ...) and the
        drained :class:`DeviceCaptures` (for the KV commit and later audits)."""
        if not self._open:
            raise RuntimeError("begin() first")
        if self.done != self.buf._cursor:
            raise RuntimeError("rows were captured after the last after_sampling()")
        out = self.oc.close(self.slot)
        self._open = False
        return out, self.buf.drain()
