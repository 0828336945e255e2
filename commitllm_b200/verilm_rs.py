"""Drop-in for the commit half of the reference's ``verilm_rs`` PyO3 module.

Same entry points, argument meanings and errors as
``crates/verilm-py/src/lib.rs``:

* :func:`commit_minimal_from_captures` (lib.rs:800-985)
* :func:`commit_minimal_packed` (lib.rs:1189-1310)
* handles with ``commitment_json``, ``merkle_root_hex``, ``io_root_hex``,
  ``manifest_hash_hex``, ``n_tokens``, ``kv_roots_hex`` (lib.rs:651-674);
* :class:`CaptureHook` (lib.rs:1842-1960).

The hashing runs on the GPU through libvcommit; inputs may be host buffers
(copied once to the device, and owned by the handle) or CUDA tensors (read in
place: the handle keeps them alive and its audits read them again, so they
must not be overwritten while the handle is open; ``retain_kv`` copies a KV
cache's rows out of the engine's pages).  KV roots come
either, as in the reference, from ``compute_kv_transcript`` when both
``x_attn_inputs`` and a ``weight_provider`` are given (verilm-py/src/lib.rs:
941-955; recomputed on the tensor cores from weights already on the GPU, see
:class:`WeightProvider`), or from the device KV cache (``kv_cache=``),
committing the same leaf encoding ``hash_kv_entry`` (merkle.rs:285-293) over
the cache's values widened to f64.

``manifest=`` binds the deployment manifest exactly as the reference does
(four-spec hashes composed into ``manifest_hash``, prover/src/lib.rs:422-440),
hashed on the host once per request (:mod:`commitllm_b200.manifest`).
``audit_v4`` / ``audit_v4_binary`` return the reference's ``V4AuditResponse``
(JSON, or ``"VV4A" || zstd(bincode)``) built from the GPU trees: retained
state, retained / IO / prefix proofs and the KV entries with their proofs,
as ``open_v4_structural`` plus the KV part of ``open_v4`` build them
(prover/src/lib.rs:1564-1687).  Not provided (outside the commitment path):
the shell opening, whose matrix-product replay from the model weights is
verifier-side math (``shell_opening`` is ``None``), and loading weights from a
safetensors directory.
"""
from __future__ import annotations

import ctypes
import json
import struct
from typing import List, Optional, Sequence

import numpy as np
import torch

from . import commit as C
from . import manifest as _manifest
from . import receipt as _receipt
from ._lib import check, lib

# MatrixType::PER_LAYER order (crates/verilm-core/src/constants.rs:26-34)
MATRIX_TYPES = ("Wq", "Wk", "Wv", "Wo", "Wg", "Wu", "Wd")


class ModelConfig:
    """The fields of ``ModelConfig`` (constants.rs:139-157) that
    ``compute_kv_transcript`` reads.  ``rope_scaling``: None or a dict with
    ``rope_type``, ``factor``, ``low_freq_factor``, ``high_freq_factor``,
    ``original_max_position_embeddings`` (constants.rs:126-137)."""

    def __init__(self, n_layers: int, hidden_dim: int, n_kv_heads: int, d_head: int, rope_theta: float,
                 rope_scaling: Optional[dict] = None):
        self.n_layers, self.hidden_dim = int(n_layers), int(hidden_dim)
        self.n_kv_heads, self.d_head = int(n_kv_heads), int(d_head)
        self.kv_dim = self.n_kv_heads * self.d_head
        self.rope_theta = float(rope_theta)
        self.rope_scaling = rope_scaling


class WeightProvider:
    """The K/V-projection part of the reference's ``WeightProvider``
    (verilm-py/src/lib.rs:530-555; accessors verilm-keygen/src/lib.rs:1202-1232),
    built from tensors a serving engine already holds on the GPU instead of
    loaded from a safetensors directory.

    wk, wv: per layer int8 CUDA tensors ``[kv_dim, hidden]``; weight_scales:
    per layer 7 per-tensor scales in ``MATRIX_TYPES`` order (0.0 for native
    INT8), or empty; per_channel_weight_scales: per layer 7 entries (float32
    ``[out_dim]`` tensors or None; only Wk and Wv are read), or empty;
    qkv_biases: per layer ``[q_bias, k_bias, v_bias]`` (float32 or None), or
    empty.  Empty lists mean what they mean in the reference: no per-tensor /
    per-channel scales (both empty: the toy path), no biases.
    """

    def __init__(self, config: ModelConfig, wk, wv, weight_scales=(), per_channel_weight_scales=(),
                 qkv_biases=()):
        self._config = config
        self._w = {"Wk": list(wk), "Wv": list(wv)}
        self._scales = [list(s) for s in weight_scales]
        self._pc = [list(s) for s in per_channel_weight_scales]
        self._bias = [list(b) for b in qkv_biases]
        if len(self._w["Wk"]) < config.n_layers or len(self._w["Wv"]) < config.n_layers:
            raise ValueError("wk and wv need one tensor per layer")

    def config(self) -> ModelConfig:
        return self._config

    def weight(self, layer: int, mt: str) -> torch.Tensor:
        if mt not in self._w:
            raise ValueError(f"only Wk and Wv are held here, not {mt}")
        return self._w[mt][layer]

    def weight_scales(self):
        return self._scales

    def per_channel_weight_scales(self):
        return self._pc

    def qkv_biases(self):
        return self._bias


def _kv_transcript_from_captures(ctx: C.Context, wp: WeightProvider, x_attn_inputs, scales_d: torch.Tensor,
                                 fwd_batch_sizes, n_layers: int):
    """The inputs of ``compute_kv_transcript`` (prover/src/lib.rs:207-329) from
    the captures: ``build_retained_from_captures``' x_attn (lib.rs:139-181)
    gathered into ``[n_tokens, layers, hidden]`` on the device, scale_x_attn the
    qkv block of each entry's scales (verilm-py/src/lib.rs:859-866), the
    weights, scales, biases and RoPE of the weight provider.  Returns
    ``(KvTranscriptInputs, tensors to keep alive)``."""
    cfg = wp.config()
    n_entries = len(fwd_batch_sizes) * n_layers
    if len(x_attn_inputs) < n_entries:
        raise ValueError("x_attn_inputs must hold one entry per (forward pass, layer)")
    L = min(cfg.n_layers, n_layers)
    n_tok = sum(fwd_batch_sizes)
    H = cfg.hidden_dim
    dev = f"cuda:{ctx.device}"
    with torch.cuda.stream(ctx.stream):
        X = torch.empty(n_tok, L, H, dtype=torch.int8, device=dev)
        sx_idx = torch.empty(n_tok, L, dtype=torch.long)
        t0 = cursor = e = 0
        for bs in fwd_batch_sizes:
            for l in range(n_layers):
                xa = x_attn_inputs[e]
                if isinstance(xa, torch.Tensor) and xa.is_cuda:
                    src = xa.reshape(-1).view(torch.int8)
                else:
                    src = ctx.to_device(_u8_host(xa)).view(torch.int8)
                if src.numel() != bs * H:
                    raise ValueError(f"x_attn entry {e} holds {src.numel()} bytes, expected {bs} x {H}")
                if l < L:
                    X[t0:t0 + bs, l].copy_(src.view(bs, H))
                    sx_idx[t0:t0 + bs, l] = torch.arange(cursor, cursor + bs)     # the qkv block
                cursor += 4 * bs
                e += 1
            t0 += bs
        sx = scales_d.index_select(0, sx_idx.view(-1).to(dev)).view(n_tok, L)
    return _kvt_token_major(ctx, wp, X, sx), [X, sx]


def _kvt_token_major(ctx: C.Context, wp: WeightProvider, X: torch.Tensor, sx: torch.Tensor) -> C.KvTranscriptInputs:
    """``compute_kv_transcript``'s inputs (prover/src/lib.rs:207-329) from x_attn
    already token-major on the device: X int8 ``[n_tokens, layers, hidden]``,
    sx float32 ``[n_tokens, layers]`` (each row's qkv_proj activation scale),
    with the weights, scales, biases and RoPE of the weight provider."""
    cfg = wp.config()
    L = int(X.shape[1])
    if L > cfg.n_layers:
        raise ValueError(f"x_attn holds {L} layers, the model {cfg.n_layers}")
    if int(X.shape[2]) != cfg.hidden_dim:
        raise ValueError(f"x_attn rows hold {int(X.shape[2])} bytes, the model's hidden_dim is {cfg.hidden_dim}")

    def pair(seq, l, conv):
        if not seq or l >= len(seq) or seq[l] is None:
            return None
        row = seq[l]
        k, v = (row[1], row[2]) if len(row) > 2 else (None, None)
        return (conv(k), conv(v))

    def dev_f32(t):
        if t is None:
            return None
        if isinstance(t, torch.Tensor) and t.numel() == 0:
            return None
        if not isinstance(t, torch.Tensor) and len(t) == 0:
            return None
        return ctx.to_device(t if isinstance(t, torch.Tensor) else np.asarray(t, np.float32), dtype=torch.float32)

    ws, pc, qb = wp.weight_scales(), wp.per_channel_weight_scales(), wp.qkv_biases()
    per_tensor = [(float(ws[l][1]) if len(ws[l]) > 1 else 0.0, float(ws[l][2]) if len(ws[l]) > 2 else 0.0)
                  for l in range(min(L, len(ws)))] if ws else None
    per_channel = [pair(pc, l, dev_f32) for l in range(L)] if pc else None
    biases = [pair(qb, l, dev_f32) for l in range(L)] if qb else None
    rs = cfg.rope_scaling
    rope = C.RopeConfig(theta=cfg.rope_theta)
    if rs:
        rope = C.RopeConfig(theta=cfg.rope_theta, scaling=rs.get("rope_type"), factor=rs.get("factor", 8.0),
                            low_freq_factor=rs.get("low_freq_factor", 1.0),
                            high_freq_factor=rs.get("high_freq_factor", 4.0),
                            original_max_position_embeddings=rs.get("original_max_position_embeddings", 8192))
    inp = C.KvTranscriptInputs(x_attn=[X[:, l] for l in range(L)], wk=[wp.weight(l, "Wk") for l in range(L)],
                               wv=[wp.weight(l, "Wv") for l in range(L)], scale_x=sx, n_kv_heads=cfg.n_kv_heads,
                               head_dim=cfg.d_head, per_tensor=per_tensor if per_tensor else None,
                               per_channel=per_channel, biases=biases, rope=rope)
    return inp


def _transcript_subset(inp: C.KvTranscriptInputs, layers: Sequence[int], n_pos: int) -> C.KvTranscriptInputs:
    """The transcript inputs of ``layers`` over positions 0..n_pos-1 (the rows an opening reveals)."""
    pick = lambda seq: None if seq is None else [seq[l] if l < len(seq) else None for l in layers]
    xs = list(inp.x_attn)
    sx = inp.scale_x
    if sx is not None:
        sx = sx[:n_pos][:, list(layers)].contiguous()
    return C.KvTranscriptInputs(x_attn=[xs[l][:n_pos] for l in layers], wk=[inp.wk[l] for l in layers],
                                wv=[inp.wv[l] for l in layers], scale_x=sx, n_kv_heads=inp.n_kv_heads,
                                head_dim=inp.head_dim, per_tensor=pick(inp.per_tensor),
                                per_channel=pick(inp.per_channel), biases=pick(inp.biases), rope=inp.rope)


def _widen(rows: torch.Tensor) -> np.ndarray:
    """K or V rows (bf16 / f32 / f64, or raw bf16 bits as int16 / uint16) as
    f64 [n, kv_dim]: the KvEntry values hash_kv_entry hashes (exact widening)."""
    r = rows.reshape(rows.shape[0], -1)
    if r.dtype in (torch.int16, torch.uint16):
        r = r.view(torch.bfloat16)
    return r.to(torch.float64).numpy()


def _f32_host(x) -> np.ndarray:
    if isinstance(x, torch.Tensor):
        x = x.detach().cpu().numpy()
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32).ravel())


def _u8_host(x) -> np.ndarray:
    if isinstance(x, (bytes, bytearray, memoryview)):
        return np.frombuffer(bytes(x), dtype=np.uint8)
    if isinstance(x, torch.Tensor):
        x = x.detach().cpu().contiguous().view(torch.uint8).numpy() if x.dtype != torch.uint8 else x.detach().cpu().numpy()
    return np.ascontiguousarray(np.asarray(x).view(np.uint8).ravel())


def _rows_tensor(ctx: C.Context, items, dtype_np, dtype_t, name: str):
    """Stack a per-token list into a device [rows, dim] tensor (uniform dim)."""
    if isinstance(items, torch.Tensor) and items.is_cuda:
        t = items if items.dim() == 2 else items.reshape(items.shape[0], -1)
        return t.contiguous(), t.shape[0]
    arrs = []
    for it in items:
        if isinstance(it, torch.Tensor):
            it = it.detach().cpu().contiguous().numpy()
        arrs.append(np.ascontiguousarray(np.asarray(it).view(dtype_np).ravel()))
    if not arrs:
        return None, 0
    dims = {a.size for a in arrs}
    if len(dims) != 1:
        raise ValueError(f"{name}: every token's row must have the same length")
    host = np.stack(arrs)
    return ctx.to_device(host), host.shape[0]


class _Committed:
    """Device results of one request's commit; host copies made on first use."""

    def __init__(self, ctx, n_tokens, token_ids, n_prompt_tokens, digests, trees, kv_roots, kv_trees,
                 n_kv_layers, manifest=None, prompt=b"", seed=bytes(32), layout=None):
        self._ctx = ctx
        self._manifest = manifest        # DeploymentManifest (manifest.from_dict) or None
        self._spec = _manifest.spec_hashes(manifest) if manifest is not None else None
        self._prompt = bytes(prompt)
        self._seed = bytes(seed)
        self._layout = layout            # where each token's retained rows live on the device
        self._n_tokens = n_tokens
        self._token_src = token_ids     # host sequence or device tensor, read on demand
        self._n_prompt_tokens = n_prompt_tokens
        self._digests = digests          # device [4 + ..., 32]: trace root, io root, prompt hash, seed commitment
        self._trees = trees              # TreeSet: tree 0 trace, tree 1 io
        self._kv_roots = kv_roots        # device [n_layers, 32] or None
        self._kv_trees = kv_trees
        self._n_kv_layers = n_kv_layers
        self._kv_view = None
        self._witnessed = None           # set_witnessed_scores: carried into the receipts
        # accepted for the reference's interface (verilm-py/src/lib.rs:592-600): deep prefix openings
        # need the bridge (RMSNorm) weights and shell openings, which this library does not build,
        # so the receipts are those the reference gives without bridge weights (prefix_retained /
        # prefix_shell_openings None)
        self.deep_prefix = False
        self._kv_host = None             # (K rows, V rows) per layer in host memory, after retain_kv("cpu")
        self._kvt = None                 # transcript inputs when the KV rows were recomputed and never stored
        self._host = None

    @property
    def _token_ids(self) -> List[int]:
        if not isinstance(self._token_src, list):
            t = self._token_src
            if isinstance(t, torch.Tensor):
                self._ctx.sync()
                t = t.cpu().numpy().view(np.uint32)
            self._token_src = [int(x) for x in t]
        return self._token_src

    def _h(self):
        if self._host is None:
            self._ctx.sync()
            d = self._digests.cpu().numpy()
            kv = self._kv_roots.cpu().numpy() if self._kv_roots is not None else np.zeros((0, 32), np.uint8)
            self._host = {"merkle_root": bytes(d[0]), "io_root": bytes(d[1]), "prompt_hash": bytes(d[2]),
                          "seed_commitment": bytes(d[3]), "kv_roots": [bytes(r) for r in kv]}
        return self._host

    # --- reference handle API (verilm-py/src/lib.rs:651-674) ---
    def _batch_commitment(self) -> dict:
        """``BatchCommitment`` (types.rs:1710-1759) with [u8; 32] fields as bytes."""
        h = self._h()
        sp = self._spec or {}
        return {
            "merkle_root": h["merkle_root"], "io_root": h["io_root"], "n_tokens": self._n_tokens,
            "manifest_hash": sp.get("manifest_hash"), "input_spec_hash": sp.get("input_spec_hash"),
            "model_spec_hash": sp.get("model_spec_hash"), "decode_spec_hash": sp.get("decode_spec_hash"),
            "output_spec_hash": sp.get("output_spec_hash"), "version": "V4",
            "prompt_hash": h["prompt_hash"], "seed_commitment": h["seed_commitment"],
            "n_prompt_tokens": self._n_prompt_tokens, "kv_roots": list(h["kv_roots"]),
        }

    def commitment(self) -> dict:
        """The serde_json value of ``BatchCommitment``: digests as lists of byte values."""
        c = self._batch_commitment()
        return {k: (list(v) if isinstance(v, bytes) else ([list(x) for x in v] if k == "kv_roots" else v))
                for k, v in c.items()}

    def commitment_json(self) -> str:
        """serde_json form of ``BatchCommitment`` (types.rs:1710-1759)."""
        return json.dumps(self.commitment(), separators=(",", ":"))

    def merkle_root_hex(self) -> str:
        return self._h()["merkle_root"].hex()

    def io_root_hex(self) -> str:
        return self._h()["io_root"].hex()

    def manifest_hash_hex(self):
        return self._spec["manifest_hash"].hex() if self._spec else None

    def n_tokens(self) -> int:
        return self._n_tokens

    def kv_roots_hex(self) -> List[str]:
        return [r.hex() for r in self._h()["kv_roots"]]

    # --- openings (merkle::prove over the committed trees) ---
    def _proof(self, trees: C.TreeSet, tree: int, index: int):
        sib, depth = trees.prove([tree], [index])
        self._ctx.sync()
        s = sib[0, :depth[0]].cpu().numpy()
        return {"leaf_index": int(index), "siblings": [bytes(x).hex() for x in s]}

    def retained_proof(self, token_index: int) -> dict:
        """MerkleProof of the token's retained leaf against merkle_root."""
        if not 0 <= token_index < self._n_tokens:
            raise ValueError(f"token_index {token_index} out of range (n_tokens={self._n_tokens})")
        return self._proof(self._trees, 0, token_index)

    def io_proof(self, token_index: int) -> dict:
        """MerkleProof of the token's IO chain value against io_root."""
        if not 0 <= token_index < self._n_tokens:
            raise ValueError(f"token_index {token_index} out of range (n_tokens={self._n_tokens})")
        return self._proof(self._trees, 1, token_index)

    def kv_proof(self, layer: int, position: int) -> dict:
        """MerkleProof of KV leaf (layer, position) against kv_roots[layer]."""
        if self._kv_trees is None:
            raise ValueError("no KV transcript was committed")
        if not 0 <= layer < self._n_kv_layers:
            raise ValueError(f"layer {layer} out of range")
        return self._proof(self._kv_trees, layer, position)

    # --- KV openings of open_v4 (prover/src/lib.rs:1564-1588) ---
    def set_witnessed_scores(self, scores, n_q_heads: int) -> None:
        """Attach witnessed attention scores, one flat row-major f32 array per
        layer (``scores[qh * seq_len + t]``), carried into every receipt with
        its KV openings (verilm-py/src/lib.rs:623-648; types.rs:1327-1334)."""
        n_q_heads = int(n_q_heads)
        if n_q_heads < 1:
            raise ValueError("n_q_heads must be positive")
        ws = []
        for i, arr in enumerate(scores):
            if isinstance(arr, torch.Tensor):
                arr = arr.detach().float().cpu().numpy()
            a = np.ascontiguousarray(np.asarray(arr, dtype=np.float32).ravel())
            if a.size % n_q_heads:
                raise ValueError(f"layer {i} score array length {a.size} not divisible by n_q_heads {n_q_heads}")
            ws.append({"scores": a, "n_q_heads": n_q_heads, "seq_len": a.size // n_q_heads})
        self._witnessed = ws

    def retain_kv(self, device="cuda") -> None:
        """Copy this request's K/V rows out of the cache the commit read, so
        that later KV openings no longer depend on the engine keeping those
        pages (the reference copies every ``KvEntry`` into its handle at
        commit, prover/src/lib.rs:449-482).  The rows keep their dtype (bf16: a
        quarter of the reference's f64 entries): on ``device`` (default the
        commit's GPU, a contiguous ``[n_positions, n_kv_heads, head_dim]``
        tensor per layer that openings read in place) or ``"cpu"`` (host
        memory; openings widen the opened rows there).  Call it before the
        engine reuses the request's pages.  A commitment whose K/V were
        recomputed from x_attn holds its own inputs and needs none of this."""
        view = self._kv_view
        if view is None:
            if self._kv_host is not None or self._kvt is not None:
                return
            raise ValueError("this commitment read no KV cache")
        n = int(view.seq_lens[0])
        dev = f"cuda:{self._ctx.device}"
        ks, vs = [], []
        with torch.cuda.stream(self._ctx.stream):
            if view.block_tables is not None:
                bs = int(view.k_layers[0].shape[1])
                pos = torch.arange(n, device=dev)
                page = view.block_tables[0].to(torch.long).index_select(0, pos // bs)
                slot = pos % bs
                for kl, vl in zip(view.k_layers, view.v_layers):
                    ks.append(kl[page, slot].contiguous())
                    vs.append(vl[page, slot].contiguous())
            else:
                off = int(view.seq_row_offset[0]) if view.seq_row_offset is not None else 0
                for kl, vl in zip(view.k_layers, view.v_layers):
                    # a copy even when the slice is already contiguous (.contiguous() would alias it)
                    ks.append(kl[off:off + n].clone(memory_format=torch.contiguous_format))
                    vs.append(vl[off:off + n].clone(memory_format=torch.contiguous_format))
        if str(device) == "cpu":
            self._ctx.sync()
            self._kv_host = ([k.cpu() for k in ks], [v.cpu() for v in vs])
            self._kv_view = None
        else:
            self._kv_view = C.KvCacheView(k_layers=ks, v_layers=vs, seq_lens=[n], layer_base=view.layer_base)

    def kv_openings(self, token_index: int, layer_indices: Optional[Sequence[int]] = None):
        """``(layers, entries f64 [n_sel, t+1, 2, kv_dim], siblings uint8 [n_sel, t+1, depth, 32])`` on the host.

        Entry [i][p] is the ``KvEntry`` of layer ``layers[i]`` at position p
        (``k_roped`` = [..., 0, :], ``v_deq`` = [..., 1, :]); the proof
        verifies ``hash_kv_entry(layer, p, k, v)`` against ``kv_roots[layer]``.
        Rows the commit hashed without storing (the weight-provider path) are
        recomputed here for the opened positions only.
        """
        if self._kv_trees is None:
            raise ValueError("no KV transcript was committed")
        if self._kv_host is not None:
            n_pos = int(self._kv_host[0][0].shape[0])
        elif self._kv_view is not None:
            n_pos = self._kv_view.seq_lens[0]
        else:
            n_pos = self._n_kv_positions()
        if not 0 <= token_index < n_pos:
            raise ValueError(f"token_index {token_index} out of range")
        layers = list(range(self._n_kv_layers)) if layer_indices is None else [int(l) for l in layer_indices]
        layers = [l for l in layers if 0 <= l < self._n_kv_layers]   # open_v4 skips unknown layers
        if self._kv_host is not None:
            # rows retained in host memory: widen to f64 here (exact), proofs from the device trees
            n = token_index + 1
            if not layers:
                return layers, np.zeros((0, n, 2, 0)), np.zeros((0, n, 0, 32), np.uint8)
            ent = np.stack([np.stack([_widen(self._kv_host[0][l][:n]), _widen(self._kv_host[1][l][:n])], axis=1)
                            for l in layers])
            sib, depth = self._kv_trees.prove([l for l in layers for _ in range(n)], list(range(n)) * len(layers))
            self._ctx.sync()
            return layers, ent, sib.cpu().numpy()[:, : depth[0]].reshape(len(layers), n, depth[0], 32)
        if self._kvt is None:
            ent, sib, _ = C.kv_open(self._ctx, self._kv_view, self._kv_trees, 0, layers, token_index + 1)
            self._ctx.sync()
            return layers, ent.cpu().numpy(), sib.cpu().numpy()
        if not layers:
            return layers, np.zeros((0, token_index + 1, 2, 0)), np.zeros((0, token_index + 1, 0, 32), np.uint8)
        with torch.cuda.stream(self._ctx.stream):
            sub = _transcript_subset(self._kvt, layers, token_index + 1)
        k, v = C.kv_transcript(self._ctx, sub)
        n = token_index + 1
        sib, depth = self._kv_trees.prove([l for l in layers for _ in range(n)], list(range(n)) * len(layers))
        self._ctx.sync()
        ent = np.stack([k.cpu().numpy(), v.cpu().numpy()], axis=2)          # [n_sel, n, 2, kv]
        return layers, ent, sib.cpu().numpy()[:, : depth[0]].reshape(len(layers), n, depth[0], 32)

    def _n_kv_positions(self) -> int:
        x = self._kvt.x_attn
        return int((x[0] if not isinstance(x, torch.Tensor) else x[0]).shape[0])

    def audit_kv_json(self, token_index: int, layer_indices: Optional[Sequence[int]] = None) -> str:
        """The ``kv_entries`` / ``kv_proofs`` fields of ``V4AuditResponse`` in serde_json form
        (f64 as little-endian hex, ``f64_hex_vec`` in types.rs:1253-1317)."""
        _layers, ent, sib = self.kv_openings(token_index, layer_indices)
        entries = [[{"k_roped": [x.tobytes().hex() for x in e[0].astype("<f8")],
                     "v_deq": [x.tobytes().hex() for x in e[1].astype("<f8")]} for e in layer] for layer in ent]
        proofs = [[{"leaf_index": p, "siblings": [list(map(int, s)) for s in layer[p]]}
                   for p in range(layer.shape[0])] for layer in sib]
        return json.dumps({"kv_entries": entries, "kv_proofs": proofs}, separators=(",", ":"))

    def audit_kv_bincode(self, token_index: int, layer_indices: Optional[Sequence[int]] = None) -> bytes:
        """bincode v1 of ``Some(kv_entries)`` then ``Some(kv_proofs)``, the bytes these two
        ``V4AuditResponse`` fields take inside a VV4A receipt (serialize.rs:43-50)."""
        _layers, ent, sib = self.kv_openings(token_index, layer_indices)
        out = bytearray(b"\x01") + struct.pack("<Q", ent.shape[0])
        kv = ent.shape[-1]
        for layer in ent:
            out += struct.pack("<Q", layer.shape[0])
            for e in layer:
                out += struct.pack("<Q", kv) + e[0].astype("<f8").tobytes()
                out += struct.pack("<Q", kv) + e[1].astype("<f8").tobytes()
        out += b"\x01" + struct.pack("<Q", sib.shape[0])
        for layer in sib:
            out += struct.pack("<Q", layer.shape[0])
            for p in range(layer.shape[0]):
                out += struct.pack("<IQ", p, layer.shape[1]) + layer[p].tobytes()
        return bytes(out)

    # --- audit receipts (verilm-py/src/lib.rs:681-786) ---
    def _retained(self, t: int) -> dict:
        """``RetainedTokenState`` of token t (types.rs:1201-1229), read back from the
        capture rows its leaf hashed; x_attn is None, as build_retained_from_captures
        leaves it (prover/src/lib.rs:162-167)."""
        lay = self._layout
        f, row = int(lay.tok_fwd[t]), int(lay.tok_row[t])
        dev = f"cuda:{self._ctx.device}"
        layers = []
        for l in range(lay.n_layers):
            a = torch.as_tensor(C._DevView(int(lay.a_rows[f][l]) + row * lay.hidden, lay.hidden, self), device=dev)
            sc = torch.as_tensor(C._DevView(int(lay.scale_a[f][l]) + 4 * row * lay.scale_stride, 4, self), device=dev)
            layers.append({"a": bytes(a.cpu().numpy()), "scale_a": struct.unpack("<f", bytes(sc.cpu().numpy()))[0],
                           "x_attn_i8": None, "scale_x_attn": None})
        return {"layers": layers}

    def _proofs(self, trees: C.TreeSet, tree: int, leaves: Sequence[int]) -> list:
        if not leaves:
            return []
        sib, depth = trees.prove([tree] * len(leaves), list(leaves))
        self._ctx.sync()
        s = sib.cpu().numpy()
        return [{"leaf_index": int(j), "siblings": [bytes(x) for x in s[k, :depth[k]]]} for k, j in enumerate(leaves)]

    def v4_audit_response(self, token_index: int, layer_indices=None, output_text=None,
                          include_kv: bool = True) -> dict:
        """The ``V4AuditResponse`` (types.rs:1475-1567) of one challenged token as
        open_v4_structural builds it (prover/src/lib.rs:1596-1687), plus the KV
        entries and proofs of open_v4 (1564-1588) for ``layer_indices`` (all
        committed layers when None).  ``shell_opening`` is None: the shell replay
        is verifier-side math this library does not build."""
        i = int(token_index)
        if not 0 <= i < self._n_tokens:
            raise ValueError(f"token_index {token_index} out of range (n_tokens={self._n_tokens})")
        if self._layout is None:
            raise ValueError("this handle keeps no capture layout to open")
        self._ctx.sync()
        leaves = self._trees.nodes(0)[: self._n_tokens].cpu().numpy()
        ios = self._trees.nodes(1)[: self._n_tokens].cpu().numpy()
        if i == 0:
            ph = self._ctx.to_device(np.frombuffer(self._h()["prompt_hash"], np.uint8).reshape(1, 32))
            g = self._ctx.empty(1, 32)
            check(lib().vc_io_genesis(self._ctx.handle, 1, ctypes.c_void_p(ph.data_ptr()),
                                      ctypes.c_void_p(g.data_ptr())))
            prev = bytes(g.cpu().numpy()[0])
        else:
            prev = bytes(ios[i - 1])
        resp = {
            "token_index": i, "retained": self._retained(i),
            "merkle_proof": self._proofs(self._trees, 0, [i])[0], "io_proof": self._proofs(self._trees, 1, [i])[0],
            "token_id": int(self._token_ids[i]) & 0xFFFFFFFF, "prev_io_hash": prev,
            "prefix_leaf_hashes": [bytes(x) for x in leaves[:i]],
            "prefix_merkle_proofs": self._proofs(self._trees, 0, list(range(i))),
            "prefix_token_ids": np.asarray([int(x) & 0xFFFFFFFF for x in self._token_ids[:i]], dtype="<u4"),
            "commitment": self._batch_commitment(), "revealed_seed": self._seed, "shell_opening": None,
            "manifest": self._manifest, "prompt": self._prompt, "n_prompt_tokens": self._n_prompt_tokens,
            "output_text": output_text, "prefix_embedding_rows": None, "prefix_embedding_proofs": None,
            "prefix_retained": None, "prefix_shell_openings": None, "kv_entries": None, "kv_proofs": None,
            "witnessed_scores": self._witnessed if include_kv else None,
        }
        if include_kv and self._kv_trees is not None:
            layers, ent, sib = self.kv_openings(i, layer_indices)
            resp["kv_entries"] = [[{"k_roped": e[0].astype("<f8"), "v_deq": e[1].astype("<f8")} for e in lay]
                                  for lay in ent]
            resp["kv_proofs"] = [[{"leaf_index": p, "siblings": [bytes(x) for x in lay[p]]}
                                  for p in range(lay.shape[0])] for lay in sib]
        return resp

    def audit_v4(self, token_index: int, layer_indices=None, output_text=None, include_kv: bool = True) -> str:
        """serde_json of the token's ``V4AuditResponse`` (verilm-py/src/lib.rs:683-695)."""
        return _receipt.v4_audit_json(self.v4_audit_response(token_index, layer_indices, output_text, include_kv))

    def audit_v4_binary(self, token_index: int, layer_indices=None, output_text=None,
                        include_kv: bool = True) -> bytes:
        """``"VV4A" || zstd(bincode)`` of the token's ``V4AuditResponse``
        (verilm-py/src/lib.rs:699-712, serialize.rs:43-50)."""
        return _receipt.serialize_v4_audit(self.v4_audit_response(token_index, layer_indices, output_text,
                                                                   include_kv))

    def leaf_hashes(self) -> torch.Tensor:
        """The retained leaves (tree 0's level 0), a device view ``[n_tokens, 32]``."""
        return self._trees.nodes(0)[: self._n_tokens]

    def io_hashes(self) -> torch.Tensor:
        return self._trees.nodes(1)[: self._n_tokens]


class MinimalBatchStateHandle(_Committed):
    """Counterpart of ``MinimalBatchStateHandle`` (verilm-py/src/lib.rs:576-787)."""

    def __init__(self, *a, x_attn=None, **k):
        super().__init__(*a, **k)
        self._x_attn = x_attn
        # accepted for the reference's interface (lib.rs:603-611): it selects the x_attn of the
        # shell opening, which this library does not build
        self.use_captured_x_attn = False

    def has_captured_x_attn(self) -> bool:
        return self._x_attn is not None

    def clear_captured_x_attn(self) -> None:
        self._x_attn = None


class PackedBatchStateHandle(_Committed):
    """Counterpart of ``PackedBatchStateHandle`` (verilm-py/src/lib.rs:993-1168)."""


def _check_common(token_ids, sampling_seed, manifest):
    """Argument checks of the boundary (verilm-py/src/lib.rs:843-897); returns
    the seed and the parsed manifest (extract_manifest, lib.rs:173-490) or None."""
    seed = bytes(sampling_seed)
    if len(seed) != 32:
        raise ValueError("sampling_seed must be exactly 32 bytes")
    for t in token_ids:
        if not 0 <= int(t) <= 0xFFFFFFFF:
            raise ValueError(f"token id {t} does not fit u32")
    return seed, (_manifest.from_dict(manifest) if manifest is not None else None)


def _finish(ctx, layout: C.TraceLayout, token_ids, prompt, seed, n_prompt_tokens, kv_cache, handle_cls,
            manifest=None, kvt: Optional[C.KvTranscriptInputs] = None, **extra):
    n = len(layout.tok_fwd)
    n_ids = token_ids.numel() if isinstance(token_ids, torch.Tensor) else len(token_ids)
    if n != n_ids:
        raise ValueError("retained state count must match token_ids")
    if n == 0:
        raise ValueError("need at least one leaf")
    kv_roots = kv_trees = None
    n_kv_layers = 0
    side = None
    if kv_cache is not None and len(kv_cache.seq_lens) != 1:
        raise ValueError("kv_cache must describe exactly the request's one sequence")
    # The KV trees run on a second stream, beside the trace leaves and the IO
    # chain: for one request those are a few thousand serial SHA chains on one
    # SM each.  The side stream waits only for the work queued before the fork.
    if kv_cache is not None or kvt is not None:
        side = ctx.fork()
    if kvt is not None:
        # the one-pass transcript kernel holds whole SMs (one persistent CTA each):
        # it goes first, and the trace leaves start on the SMs it leaves
        kv_roots, kv_trees = C.kv_transcript_commit(side, kvt, keep_trees=True)
        kv_trees.ctx = ctx               # later openings run on the main stream, after the join below
        n_kv_layers = len(kvt.wk)
    # leaves and io values in one buffer so both trees build in one launch
    both = ctx.empty(2 * n, 32)
    C.trace_leaves(ctx, layout, out=both[:n])
    if kv_cache is not None:
        # launched after the trace leaves, so that their latency-bound CTAs are
        # placed one per SM before the KV kernel's CTAs fill the GPU (placed after
        # them, several trace CTAs shared SMs and the request took 36 instead of
        # 18 ms of trace leaves)
        r, kv_trees = C.kv_commit(side, kv_cache, keep_trees=True)
        kv_trees.ctx = ctx
        kv_roots = r[0]
        n_kv_layers = len(kv_cache.k_layers)
    if isinstance(token_ids, torch.Tensor) and token_ids.is_cuda:
        if token_ids.dtype not in (torch.int32, torch.uint32) or token_ids.numel() != n:
            raise ValueError("token_ids on the device must be a 32-bit tensor of n_tokens entries")
        tok = token_ids.reshape(-1).contiguous()
    else:
        tok = ctx.to_device(np.asarray([int(t) for t in token_ids], dtype=np.uint32).view(np.int32))
    digests = ctx.empty(4, 32)
    ph = C.prompt_hashes(ctx, [bytes(prompt)])
    C.io_chain(ctx, both[:n], tok, ph, [0, n], out=both[n:])
    roots, trees = C.build_trees(ctx, both, [0, n, 2 * n], keep_trees=True, roots_out=digests[:2])
    seeds = ctx.to_device(np.frombuffer(seed, dtype=np.uint8).reshape(1, 32))
    sc = C.seed_commitments(ctx, seeds)
    with torch.cuda.stream(ctx.stream):
        digests[2].copy_(ph[0])
        digests[3:4].copy_(sc)
    if side is not None:
        ctx.join(side)
    h = handle_cls(ctx, n, token_ids, n_prompt_tokens, digests, trees, kv_roots, kv_trees, n_kv_layers,
                   manifest=manifest, prompt=prompt, seed=seed, layout=layout, **extra)
    h._kv_view = kv_cache
    h._kvt = kvt
    return h


def _wrap_rows(n_tokens, rows, n_prompt_tokens, which):
    """Row index per token for an optional per-token list (prover/src/lib.rs:367-390)."""
    if which == "logits":
        gen_start = max(0, n_prompt_tokens - 1) if n_prompt_tokens is not None else 0
        return [t - gen_start if (t >= gen_start and t - gen_start < rows) else -1 for t in range(n_tokens)]
    return [t if t < rows else -1 for t in range(n_tokens)]


class CaptureHook:
    """The capture wrapper's bookkeeping (verilm-py/src/lib.rs:1842-1960): call
    counting, per-call scale references and their drain, for a hook written
    against ``verilm_rs.CaptureHook``.  ``drain_scales`` returns host numpy as
    the reference does; ``drain_scales_device`` keeps the concatenated scales
    on the device (``commit_minimal_from_captures`` reads CUDA scales in place).
    :class:`commitllm_b200.capture.DeviceCaptureBuffer` is the whole device-side
    hook."""

    def __init__(self, calls_per_fwd: int, projs_per_layer: int, o_proj_idx: int = 1):
        if calls_per_fwd < 1 or projs_per_layer < 1:
            raise ValueError("calls_per_fwd and projs_per_layer must be positive")
        self._calls_per_fwd, self._projs = int(calls_per_fwd), int(projs_per_layer)
        self._counter = 0
        self._minimal = 0
        self._total = 0
        self._scales: list = []

    def record(self, scale_a) -> int:
        """Keep the scale; return the call's projection index in its layer
        (0 qkv, 1 o_proj, 2 gate_up, 3 down)."""
        idx = self._counter % self._calls_per_fwd
        self._counter += 1
        self._scales.append(scale_a)
        self._minimal += 1
        self._total += 1
        return idx % self._projs

    def _cat(self):
        try:
            return torch.cat(self._scales)
        except RuntimeError:                        # prefill [bs, 1] beside decode [1]: flatten each
            return torch.cat([t.flatten() for t in self._scales])

    def drain_scales(self):
        """``(float32 numpy array, call count)`` of the scales recorded since the last drain."""
        count, self._minimal = self._minimal, 0
        if not self._scales:
            return np.array([], dtype=np.float32), 0
        cat = self._cat()
        self._scales = []
        return cat.detach().float().cpu().numpy().reshape(-1), count

    def drain_scales_device(self):
        """As :meth:`drain_scales`, the scales left on their device (no host copy)."""
        count, self._minimal = self._minimal, 0
        if not self._scales:
            return torch.empty(0, dtype=torch.float32), 0
        cat = self._cat()
        self._scales = []
        return cat.detach().to(torch.float32).reshape(-1), count

    def reset_counter(self) -> None:
        self._counter = 0

    @property
    def call_counter(self) -> int:
        return self._counter

    @property
    def total_captured(self) -> int:
        return self._total

    @property
    def minimal_call_count(self) -> int:
        return self._minimal


def commit_minimal_from_captures(o_proj_inputs, scales, n_layers, fwd_batch_sizes, token_ids, prompt,
                                 sampling_seed, manifest=None, weight_provider=None, final_residuals=None,
                                 n_prompt_tokens=None, x_attn_inputs=None, lp_hidden_bf16=None,
                                 captured_logits_f32=None, *, kv_cache: Optional[C.KvCacheView] = None,
                                 ctx: Optional[C.Context] = None) -> MinimalBatchStateHandle:
    """V4 commitment from minimal captures (verilm-py/src/lib.rs:800-985)."""
    ctx = ctx or C.Context()
    seed, man = _check_common(token_ids, sampling_seed, manifest)
    fwd_batch_sizes = [int(b) for b in fwd_batch_sizes]
    n_layers = int(n_layers)
    scales_h = scales if (isinstance(scales, torch.Tensor) and scales.is_cuda) else _f32_host(scales)
    expected = sum(bs * 4 * n_layers for bs in fwd_batch_sizes)
    n_scales = scales_h.numel() if isinstance(scales_h, torch.Tensor) else scales_h.size
    if n_scales != expected:
        raise ValueError(f"expected {expected} scales (4 × batch_size per layer entry), got {n_scales}")
    if len(o_proj_inputs) < len(fwd_batch_sizes) * n_layers:
        raise ValueError("o_proj_inputs must hold one entry per (forward pass, layer)")
    scales_d = ctx.to_device(scales_h, dtype=torch.float32)
    a_dev = []
    for x in o_proj_inputs[: len(fwd_batch_sizes) * n_layers]:
        if isinstance(x, torch.Tensor) and x.is_cuda:
            a_dev.append(x.contiguous())
        else:
            a_dev.append(ctx.to_device(_u8_host(x)))
    hidden = None
    a_rows, s_rows = [], []
    cursor = 0
    e = 0
    for bs in fwd_batch_sizes:
        ar, sr = [], []
        for _l in range(n_layers):
            t = a_dev[e]
            dim = (t.numel() * t.element_size()) // bs if bs else 0
            if hidden is None:
                hidden = dim
            elif dim != hidden:
                raise ValueError("every o_proj input row must have the same length")
            ar.append(t.data_ptr())
            sr.append(scales_d.data_ptr() + 4 * (cursor + bs))   # the o_proj block of this entry
            cursor += 4 * bs
            e += 1
        a_rows.append(ar)
        s_rows.append(sr)
    tok_fwd, tok_row = [], []
    for f, bs in enumerate(fwd_batch_sizes):
        tok_fwd += [f] * bs
        tok_row += list(range(bs))
    n_tok = len(tok_fwd)
    lay = C.TraceLayout(n_layers=n_layers, hidden=hidden or 0, fwd_rows=fwd_batch_sizes, tok_fwd=tok_fwd,
                        tok_row=tok_row, a_rows=a_rows, scale_a=s_rows, scale_stride=1)
    keep = [a_dev, scales_d]
    if final_residuals is not None:
        t, rows = _rows_tensor(ctx, final_residuals, np.float32, torch.float32, "final_residuals")
        if t is not None:
            lay.final_residual, lay.tok_fr_row = t, _wrap_rows(n_tok, rows, n_prompt_tokens, "fr")
            keep.append(t)
    if lp_hidden_bf16 is not None:
        t, rows = _rows_tensor(ctx, lp_hidden_bf16, np.uint16, torch.int16, "lp_hidden_bf16")
        if t is not None:
            lay.lp_hidden, lay.tok_lp_row = t, _wrap_rows(n_tok, rows, n_prompt_tokens, "lp")
            keep.append(t)
    if captured_logits_f32 is not None:
        t, rows = _rows_tensor(ctx, captured_logits_f32, np.float32, torch.float32, "captured_logits_f32")
        if t is not None:
            lay.logits, lay.tok_logits_row = t, _wrap_rows(n_tok, rows, n_prompt_tokens, "logits")
            keep.append(t)
    kvt = None
    if x_attn_inputs is not None and weight_provider is not None:
        # the reference's path: K/V recomputed from x_attn + weights and committed (one pass)
        if kv_cache is not None:
            raise ValueError("pass either kv_cache or x_attn_inputs with weight_provider, not both")
        kvt, held = _kv_transcript_from_captures(ctx, weight_provider, x_attn_inputs, scales_d, fwd_batch_sizes,
                                                 n_layers)
        keep += held
    h = _finish(ctx, lay, token_ids, prompt, seed, n_prompt_tokens, kv_cache, MinimalBatchStateHandle,
                manifest=man, kvt=kvt, x_attn=x_attn_inputs)
    h._inputs = keep
    return h


def commit_minimal_packed(packed_a, packed_scales, n_layers, hidden_dim, fwd_batch_sizes, token_ids, prompt,
                          sampling_seed, manifest=None, weight_provider=None, packed_final_res=None,
                          final_res_dim=0, n_prompt_tokens=None, *, kv_cache: Optional[C.KvCacheView] = None,
                          ctx: Optional[C.Context] = None) -> PackedBatchStateHandle:
    """V4 commitment from packed buffers (verilm-py/src/lib.rs:1189-1310)."""
    ctx = ctx or C.Context()
    seed, man = _check_common(token_ids, sampling_seed, manifest)
    fwd_batch_sizes = [int(b) for b in fwd_batch_sizes]
    n_layers, hidden_dim = int(n_layers), int(hidden_dim)
    n_tok = sum(fwd_batch_sizes)
    if n_tok != len(token_ids):
        raise ValueError("token count must match token_ids")
    a = packed_a if (isinstance(packed_a, torch.Tensor) and packed_a.is_cuda) else ctx.to_device(_u8_host(packed_a))
    if a.numel() * a.element_size() != n_tok * n_layers * hidden_dim:
        raise ValueError(f"packed_a length ({a.numel() * a.element_size()}) != expected "
                         f"({n_tok} tokens × {n_layers} layers × {hidden_dim} dim)")
    s = packed_scales if (isinstance(packed_scales, torch.Tensor) and packed_scales.is_cuda) else _f32_host(packed_scales)
    n_s = s.numel() if isinstance(s, torch.Tensor) else s.size
    if n_s != n_tok * n_layers * 4:
        raise ValueError("scale rearrangement consumed wrong number of values")
    s = ctx.to_device(s, dtype=torch.float32)
    a_rows, s_rows = [], []
    cum = 0
    cursor = 0
    for bs in fwd_batch_sizes:
        ar, sr = [], []
        for l in range(n_layers):
            ar.append(a.data_ptr() + (cum * n_layers + l * bs) * hidden_dim)
            sr.append(s.data_ptr() + 4 * (cursor + bs))   # drain order: [qkv | o_proj | gate | down] x bs
            cursor += 4 * bs
        a_rows.append(ar)
        s_rows.append(sr)
        cum += bs
    tok_fwd, tok_row = [], []
    for f, bs in enumerate(fwd_batch_sizes):
        tok_fwd += [f] * bs
        tok_row += list(range(bs))
    lay = C.TraceLayout(n_layers=n_layers, hidden=hidden_dim, fwd_rows=fwd_batch_sizes, tok_fwd=tok_fwd,
                        tok_row=tok_row, a_rows=a_rows, scale_a=s_rows, scale_stride=1)
    keep = [a, s]
    if packed_final_res is not None:
        fr = packed_final_res if (isinstance(packed_final_res, torch.Tensor) and packed_final_res.is_cuda) \
            else ctx.to_device(_u8_host(packed_final_res))
        fr = fr.contiguous().view(torch.uint8)
        if fr.numel() != n_tok * int(final_res_dim) * 4:
            raise ValueError(f"packed_final_res length ({fr.numel()}) != expected "
                             f"({n_tok} tokens × {final_res_dim} dim × 4)")
        lay.final_residual = fr.view(torch.float32).view(n_tok, int(final_res_dim))
        lay.tok_fr_row = list(range(n_tok))
        keep.append(fr)
    h = _finish(ctx, lay, token_ids, prompt, seed, n_prompt_tokens, kv_cache, PackedBatchStateHandle, manifest=man)
    h._inputs = keep
    return h


def commit_request(a: torch.Tensor, scales_a: torch.Tensor, token_ids, prompt, sampling_seed, *,
                   n_prompt_tokens: Optional[int] = None, captured_logits_f32: Optional[torch.Tensor] = None,
                   kv_cache: Optional[C.KvCacheView] = None, manifest=None,
                   x_attn: Optional[torch.Tensor] = None, scale_x_attn: Optional[torch.Tensor] = None,
                   weight_provider: Optional[WeightProvider] = None,
                   ctx: Optional[C.Context] = None) -> MinimalBatchStateHandle:
    """One request's whole commitment, from captures already in device memory.

    An entry of this library with no PyO3 counterpart: it makes the commitment
    ``commit_minimal_from_captures`` makes (``commit_minimal``,
    prover/src/lib.rs:336-544: trace leaves, IO chain, trace and IO trees,
    manifest hashes, KV trees), but takes the captures as whole tensors, so a
    long request costs a handful of launches and no per-entry host work; the
    KV trees run on a second stream beside the trace leaves and the serial IO
    chain.

    a: int8 ``[n_tokens, n_layers, hidden]`` (the o_proj input row of each
    committed token and layer, token order); scales_a: float32
    ``[n_tokens, n_layers]``; token_ids: ``n_tokens`` ids (``all_ids[1:]``, a
    host sequence or a 32-bit CUDA tensor); captured_logits_f32: float32
    ``[rows, vocab]``, row j bound to token ``gen_start + j`` with
    ``gen_start = n_prompt_tokens - 1`` (prover/src/lib.rs:367-390);
    kv_cache: the request's K/V rows (one sequence).  Or, as the reference
    commits them, K/V recomputed from x_attn: int8 ``[n_tokens, layers,
    hidden]`` (the qkv_proj input rows), scale_x_attn float32 ``[n_tokens,
    layers]`` and a weight_provider (one pass, ``vc_kv_transcript_commit``).
    """
    ctx = ctx or C.Context()
    C._require_cuda(a, "a")
    C._require_cuda(scales_a, "scales_a")
    if a.dtype not in (torch.int8, torch.uint8) or a.dim() != 3 or not a.is_contiguous():
        raise ValueError("a must be a contiguous int8 [n_tokens, n_layers, hidden] CUDA tensor")
    n, L, H = (int(x) for x in a.shape)
    if scales_a.dtype != torch.float32 or tuple(scales_a.shape) != (n, L) or not scales_a.is_contiguous():
        raise ValueError(f"scales_a must be a contiguous float32 [{n}, {L}] CUDA tensor")
    ids = token_ids if isinstance(token_ids, torch.Tensor) else list(token_ids)
    if isinstance(ids, list):
        seed, man = _check_common(ids, sampling_seed, manifest)
    else:
        seed, man = _check_common([], sampling_seed, manifest)
    # every token its own one-row pass: row pointers of token t, layer l
    tl = np.arange(n, dtype=np.uint64)[:, None] * np.uint64(L) + np.arange(L, dtype=np.uint64)[None, :]
    lay = C.TraceLayout(n_layers=L, hidden=H, fwd_rows=np.ones(n, np.int32), tok_fwd=np.arange(n, dtype=np.int32),
                        tok_row=np.zeros(n, np.int32), a_rows=np.uint64(a.data_ptr()) + tl * np.uint64(H),
                        scale_a=np.uint64(scales_a.data_ptr()) + tl * np.uint64(4), scale_stride=1)
    keep = [a, scales_a]
    if captured_logits_f32 is not None:
        C._require_cuda(captured_logits_f32, "captured_logits_f32")
        lg = captured_logits_f32
        if lg.dtype != torch.float32 or lg.dim() != 2 or lg.stride(1) != 1:
            raise ValueError("captured_logits_f32 must be a float32 [rows, vocab] CUDA tensor with unit column stride")
        gen_start = max(0, n_prompt_tokens - 1) if n_prompt_tokens is not None else 0
        t = np.arange(n, dtype=np.int64) - gen_start
        lay.logits = lg
        lay.tok_logits_row = np.where((t >= 0) & (t < lg.shape[0]), t, -1).astype(np.int32)
        keep.append(lg)
    kvt = None
    if (x_attn is None) != (weight_provider is None) or (x_attn is None) != (scale_x_attn is None):
        raise ValueError("x_attn, scale_x_attn and weight_provider go together")
    if x_attn is not None:
        if kv_cache is not None:
            raise ValueError("pass either kv_cache or x_attn with weight_provider, not both")
        C._require_cuda(x_attn, "x_attn")
        C._require_cuda(scale_x_attn, "scale_x_attn")
        if x_attn.dtype != torch.int8 or x_attn.dim() != 3 or int(x_attn.shape[0]) != n:
            raise ValueError(f"x_attn must be an int8 [{n}, layers, hidden] CUDA tensor")
        if scale_x_attn.dtype != torch.float32 or tuple(scale_x_attn.shape) != tuple(x_attn.shape[:2]):
            raise ValueError(f"scale_x_attn must be a float32 [{n}, {int(x_attn.shape[1])}] CUDA tensor")
        kvt = _kvt_token_major(ctx, weight_provider, x_attn, scale_x_attn.contiguous())
        keep += [x_attn, scale_x_attn]
    h = _finish(ctx, lay, ids, prompt, seed, n_prompt_tokens, kv_cache, MinimalBatchStateHandle, manifest=man,
                kvt=kvt, x_attn=x_attn)
    h._inputs = keep
    return h
