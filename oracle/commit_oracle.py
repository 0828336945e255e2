"""The oracle: a CPU restatement of CommitLLM's trace-commitment encodings.

TEST INFRASTRUCTURE ONLY.  Nothing in the product path (``commitllm_b200``)
imports this module; only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` leg of ``bench.py`` use it, as the checker.

Every function restates one function of the reference (lambdaclass/CommitLLM)
and cites the file:line it follows.  The hash is FIPS 180-4 SHA-256, the
algorithm of the ``sha2`` crate v0.10.9 that ``verilm-core`` pins
(``crates/verilm-core/Cargo.toml:7``, ``Cargo.lock:783-784``); Python's
``hashlib.sha256`` computes the same function.  All integers are encoded
little-endian, as the reference's ``to_le_bytes`` calls do.

Pinned against the reference's golden vectors in ``tests/golden/`` (see
``tests/test_oracle_golden.py``): the ``golden_e2e_verify`` merkle_root /
io_root pins and the two frozen ``v4_audit_*.bin`` receipts.
"""
from __future__ import annotations

import hashlib
import struct
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np

ZERO32 = bytes(32)


def sha256(*parts: bytes) -> bytes:
    h = hashlib.sha256()
    for p in parts:
        h.update(p)
    return h.digest()


# ---------------------------------------------------------------------------
# Merkle tree: crates/verilm-core/src/merkle.rs:11-123
# ---------------------------------------------------------------------------

def hash_pair(left: bytes, right: bytes) -> bytes:
    """``hash_pair`` (merkle.rs:118-123): SHA256(left || right), no tag."""
    return sha256(left, right)


def hash_leaf(data: bytes) -> bytes:
    """``hash_leaf`` (merkle.rs:126-130)."""
    return sha256(data)


def next_pow2(n: int) -> int:
    p = 1
    while p < n:
        p <<= 1
    return p


@dataclass
class MerkleTree:
    """``MerkleTree`` (merkle.rs:295-301): nodes level-concatenated bottom-up."""
    nodes: List[bytes]
    n_leaves: int
    padded_size: int
    root: bytes


@dataclass
class MerkleProof:
    """``MerkleProof`` (merkle.rs:303-307): siblings bottom-up."""
    leaf_index: int
    siblings: List[bytes] = field(default_factory=list)


def build_tree(leaves: Sequence[bytes]) -> MerkleTree:
    """``build_tree`` (merkle.rs:11-48).

    Pads level 0 to the next power of two with all-zero leaves (padding
    happens at level 0 only), then hashes pairs level by level.
    """
    if len(leaves) == 0:
        raise ValueError("need at least one leaf")
    n = next_pow2(len(leaves))
    nodes = list(leaves) + [ZERO32] * (n - len(leaves))
    start, size = 0, n
    while size > 1:
        for i in range(0, size, 2):
            nodes.append(hash_pair(nodes[start + i], nodes[start + i + 1]))
        start += size
        size //= 2
    return MerkleTree(nodes=nodes, n_leaves=len(leaves), padded_size=n, root=nodes[-1])


def compute_root(leaves: Sequence[bytes]) -> bytes:
    """``compute_root`` (merkle.rs:55-76): same root as ``build_tree``."""
    if len(leaves) == 0:
        raise ValueError("need at least one leaf")
    level = list(leaves) + [ZERO32] * (next_pow2(len(leaves)) - len(leaves))
    while len(level) > 1:
        level = [hash_pair(level[i], level[i + 1]) for i in range(0, len(level), 2)]
    return level[0]


def prove(tree: MerkleTree, index: int) -> MerkleProof:
    """``prove`` (merkle.rs:79-99)."""
    if not (0 <= index < tree.n_leaves):
        raise IndexError("leaf index out of range")
    sib = []
    idx, start, size = index, 0, tree.padded_size
    while size > 1:
        s = idx + 1 if idx % 2 == 0 else idx - 1
        sib.append(tree.nodes[start + s])
        start += size
        size //= 2
        idx //= 2
    return MerkleProof(leaf_index=index, siblings=sib)


def verify(root: bytes, leaf: bytes, proof: MerkleProof) -> bool:
    """``verify`` (merkle.rs:102-116)."""
    cur, idx = leaf, proof.leaf_index
    for s in proof.siblings:
        cur = hash_pair(cur, s) if idx % 2 == 0 else hash_pair(s, cur)
        idx //= 2
    return cur == root


def zero_subtree_roots(max_height: int) -> List[bytes]:
    """Z_0 = 0^32, Z_{k+1} = H(Z_k || Z_k): the root of an all-padding subtree.

    Not a reference function; it is what ``build_tree`` computes for a
    subtree whose leaves are all zero padding (merkle.rs:22-39).
    """
    z = [ZERO32]
    for _ in range(max_height):
        z.append(hash_pair(z[-1], z[-1]))
    return z


# ---------------------------------------------------------------------------
# Leaf encodings: crates/verilm-core/src/merkle.rs:144-293
# ---------------------------------------------------------------------------

def bf16_to_f64(bits: np.ndarray) -> np.ndarray:
    """Widen raw bf16 bit patterns to f64, exactly.

    bf16 -> f32 is a 16-bit left shift; f32 -> f64 is numpy's (IEEE) widening,
    which is exact for every finite value including subnormals.  NaNs keep their
    payload with the quiet bit set.  This is the value set a KV entry holds when
    the K/V cache row is bf16 (``KvEntry`` is ``Vec<f64>``, types.rs:1244-1251).
    """
    b = np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16
    f32 = b.view(np.float32)
    with np.errstate(invalid="ignore"):
        out = f32.astype(np.float64)
    # numpy's cast of a signalling NaN is platform defined: force the quiet bit
    # explicitly so the encoding is pinned (sign | 0x7FF | quiet | payload<<29).
    nan = np.isnan(f32)
    if nan.any():
        u = b[nan].astype(np.uint64)
        sign = (u >> 31) << 63
        payload = (u & 0x7FFFFF) << 29
        quiet = np.uint64(1) << np.uint64(51)
        out_bits = out.view(np.uint64).copy()
        out_bits[nan] = sign | (np.uint64(0x7FF) << np.uint64(52)) | quiet | payload
        out = out_bits.view(np.float64)
    return out


def f32_to_f64(vals: np.ndarray) -> np.ndarray:
    """Widen f32 to f64 with the same NaN rule as :func:`bf16_to_f64`."""
    b = np.ascontiguousarray(vals, dtype=np.float32).view(np.uint32)
    f32 = b.view(np.float32)
    with np.errstate(invalid="ignore"):
        out = f32.astype(np.float64)
    nan = np.isnan(f32)
    if nan.any():
        u = b[nan].astype(np.uint64)
        sign = (u >> 31) << 63
        payload = (u & 0x7FFFFF) << 29
        quiet = np.uint64(1) << np.uint64(51)
        out_bits = out.view(np.uint64).copy()
        out_bits[nan] = sign | (np.uint64(0x7FF) << np.uint64(52)) | quiet | payload
        out = out_bits.view(np.float64)
    return out


def hash_kv_entry(layer: int, position: int, k_roped: np.ndarray, v_deq: np.ndarray) -> bytes:
    """``hash_kv_entry`` (merkle.rs:285-293) with ``hash_f64_into`` (274-278).

    SHA256("vi-kv-v1" || u32le(layer) || u32le(pos) || f64le[k] || f64le[v]).
    """
    k = np.ascontiguousarray(k_roped, dtype="<f8")
    v = np.ascontiguousarray(v_deq, dtype="<f8")
    return sha256(b"vi-kv-v1", struct.pack("<II", layer & 0xFFFFFFFF, position & 0xFFFFFFFF),
                  k.tobytes(), v.tobytes())


@dataclass
class RetainedLayerState:
    """``RetainedLayerState`` (types.rs:1201-1219)."""
    a: bytes                       # i8 bytes
    scale_a: float                 # f32
    x_attn_i8: Optional[bytes] = None
    scale_x_attn: Optional[float] = None


def _f32le(x: float) -> bytes:
    return struct.pack("<f", x)


def hash_retained_state_direct(layers: Sequence[RetainedLayerState]) -> bytes:
    """``hash_retained_state_direct`` (merkle.rs:144-161).

    SHA256("vi-retained-v3" || for each layer: a || f32le(scale_a) ||
    (0x01 || x_attn_i8 || f32le(scale_x_attn) when both are Some, else 0x00)).
    """
    h = hashlib.sha256(b"vi-retained-v3")
    for ls in layers:
        h.update(bytes(ls.a))
        h.update(_f32le(ls.scale_a))
        if ls.x_attn_i8 is not None and ls.scale_x_attn is not None:
            h.update(b"\x01")
            h.update(bytes(ls.x_attn_i8))
            h.update(_f32le(ls.scale_x_attn))
        else:
            h.update(b"\x00")
    return h.digest()


def _f32_bytes(arr) -> bytes:
    return np.ascontiguousarray(arr, dtype="<f4").tobytes()


def hash_retained_with_residual(layers, final_residual=None) -> bytes:
    """``hash_retained_with_residual`` (merkle.rs:170-185)."""
    base = hash_retained_state_direct(layers)
    if final_residual is None:
        return base
    return sha256(b"vi-retained-fr-v1", base, _f32_bytes(final_residual))


def hash_retained_with_lp_hidden(layers, final_residual=None, lp_hidden_bf16=None) -> bytes:
    """``hash_retained_with_lp_hidden`` (merkle.rs:195-215): u16le bf16 bits."""
    base = hash_retained_with_residual(layers, final_residual)
    if lp_hidden_bf16 is None:
        return base
    lp = np.ascontiguousarray(lp_hidden_bf16, dtype="<u2").tobytes()
    return sha256(b"vi-retained-lp-v1", base, lp)


def hash_retained_with_captured_logits(layers, final_residual=None, lp_hidden_bf16=None,
                                       captured_logits_f32=None) -> bytes:
    """``hash_retained_with_captured_logits`` (merkle.rs:224-241)."""
    base = hash_retained_with_lp_hidden(layers, final_residual, lp_hidden_bf16)
    if captured_logits_f32 is None:
        return base
    return sha256(b"vi-retained-logits-v1", base, _f32_bytes(captured_logits_f32))


# ---------------------------------------------------------------------------
# IO chain and bindings: merkle.rs:250-257, 553-577
# ---------------------------------------------------------------------------

def io_hash_v4(leaf_hash: bytes, token_id: int, prev_io_hash: bytes) -> bytes:
    """``io_hash_v4`` (merkle.rs:250-257)."""
    return sha256(b"vi-io-v4", leaf_hash, struct.pack("<I", token_id & 0xFFFFFFFF), prev_io_hash)


def hash_seed(seed: bytes) -> bytes:
    """``hash_seed`` (merkle.rs:553-558)."""
    return sha256(b"vi-seed-v1", seed)


def hash_prompt(prompt: bytes) -> bytes:
    """``hash_prompt`` (merkle.rs:561-566)."""
    return sha256(b"vi-prompt-v1", prompt)


def io_genesis_v4(prompt_hash: bytes) -> bytes:
    """``io_genesis_v4`` (merkle.rs:572-577)."""
    return sha256(b"vi-io-genesis-v4", prompt_hash)


def io_chain(trace_leaves: Sequence[bytes], token_ids: Sequence[int], prompt: bytes) -> List[bytes]:
    """The IO chain loop of ``commit_minimal`` (verilm-prover/src/lib.rs:403-410)."""
    prev = io_genesis_v4(hash_prompt(prompt))
    out = []
    for leaf, tok in zip(trace_leaves, token_ids):
        prev = io_hash_v4(leaf, tok, prev)
        out.append(prev)
    return out


# ---------------------------------------------------------------------------
# Four-spec manifest hashing: merkle.rs:324-457, specs from the flat manifest
# by DeploymentManifest::split (types.rs:512-520, From impls 574-775).
# A manifest here is a dict of the Rust field names; [u8; 32] as bytes,
# Option as None, Vec<(u32, f32)> as a list of pairs.
# ---------------------------------------------------------------------------

def _opt32(h, v):
    """hash_optional_32 (merkle.rs:459-467)."""
    if v is None:
        h.update(b"\x00")
    else:
        h.update(b"\x01")
        h.update(v)


def _opt_u32(h, v):
    """hash_optional_u32 (merkle.rs:469-477)."""
    if v is None:
        h.update(b"\x00")
    else:
        h.update(b"\x01")
        h.update(struct.pack("<I", v))


def _opt_f64(h, v):
    """hash_optional_f64 (merkle.rs:479-487)."""
    if v is None:
        h.update(b"\x00")
    else:
        h.update(b"\x01")
        h.update(struct.pack("<d", v))


def _opt_str(h, v):
    """hash_optional_string (merkle.rs:489-498)."""
    if v is None:
        h.update(b"\x00")
    else:
        b = v.encode()
        h.update(b"\x01")
        h.update(struct.pack("<I", len(b)))
        h.update(b)


def hash_input_spec(m) -> bytes:
    """``hash_input_spec`` (merkle.rs:324-335)."""
    h = hashlib.sha256(b"vi-input-v1")
    h.update(m["tokenizer_hash"])
    _opt32(h, m["system_prompt_hash"])
    _opt32(h, m["chat_template_hash"])
    _opt_str(h, m["bos_eos_policy"])
    _opt_str(h, m["truncation_policy"])
    _opt_str(h, m["special_token_policy"])
    _opt_str(h, m["padding_policy"])
    return h.digest()


def hash_model_spec(m) -> bytes:
    """``hash_model_spec`` (merkle.rs:338-367)."""
    h = hashlib.sha256(b"vi-model-v1")
    _opt32(h, m["weight_hash"])
    _opt32(h, m["quant_hash"])
    _opt32(h, m["rope_config_hash"])
    if m["rmsnorm_eps"] is not None:
        h.update(b"\x01")
        h.update(struct.pack("<d", m["rmsnorm_eps"]))
    else:
        h.update(b"\x00")
    _opt32(h, m["adapter_hash"])
    _opt_u32(h, m["n_layers"])
    _opt_u32(h, m["hidden_dim"])
    _opt_u32(h, m["vocab_size"])
    _opt32(h, m["embedding_merkle_root"])
    _opt_str(h, m["quant_family"])
    _opt_str(h, m["scale_derivation"])
    _opt_u32(h, m["quant_block_size"])
    _opt_u32(h, m["kv_dim"])
    _opt_u32(h, m["ffn_dim"])
    _opt_u32(h, m["d_head"])
    _opt_u32(h, m["n_q_heads"])
    _opt_u32(h, m["n_kv_heads"])
    _opt_f64(h, m["rope_theta"])
    return h.digest()


def hash_decode_spec(m) -> bytes:
    """``hash_decode_spec`` (merkle.rs:370-401)."""
    h = hashlib.sha256(b"vi-decode-v1")
    h.update(struct.pack("<f", m["temperature"]))
    h.update(struct.pack("<I", m["top_k"]))
    h.update(struct.pack("<f", m["top_p"]))
    h.update(struct.pack("<f", m["repetition_penalty"]))
    h.update(struct.pack("<f", m["frequency_penalty"]))
    h.update(struct.pack("<f", m["presence_penalty"]))
    h.update(struct.pack("<I", len(m["logit_bias"])))
    for tok, bias in m["logit_bias"]:
        h.update(struct.pack("<I", tok))
        h.update(struct.pack("<f", bias))
    h.update(struct.pack("<I", len(m["bad_word_ids"])))
    for tok in m["bad_word_ids"]:
        h.update(struct.pack("<I", tok))
    g = m["guided_decoding"].encode()
    h.update(struct.pack("<I", len(g)))
    h.update(g)
    if m["sampler_version"] is not None:
        sv = m["sampler_version"].encode()
        h.update(b"\x01")
        h.update(struct.pack("<I", len(sv)))
        h.update(sv)
    else:
        h.update(b"\x00")
    _opt_str(h, m["decode_mode"])
    return h.digest()


def hash_output_spec(m) -> bytes:
    """``hash_output_spec`` (merkle.rs:404-427)."""
    h = hashlib.sha256(b"vi-output-v1")
    h.update(m["eos_policy"].encode())
    h.update(struct.pack("<I", len(m["stop_sequences"])))
    for st in m["stop_sequences"]:
        b = st.encode()
        h.update(struct.pack("<I", len(b)))
        h.update(b)
    h.update(struct.pack("<I", m["max_tokens"]))
    h.update(struct.pack("<I", m["min_tokens"]))
    h.update(bytes([1 if m["ignore_eos"] else 0]))
    _opt_str(h, m["detokenization_policy"])
    if m["eos_token_id"] is not None:
        h.update(bytes([1]))
        h.update(struct.pack("<I", m["eos_token_id"]))
    else:
        h.update(bytes([0]))
    return h.digest()


def hash_manifest_composed(h_input: bytes, h_model: bytes, h_decode: bytes, h_output: bytes) -> bytes:
    """``hash_manifest_composed`` (merkle.rs:432-446)."""
    return sha256(b"vi-manifest-v4", h_input, h_model, h_decode, h_output)


def hash_manifest(m) -> bytes:
    """``hash_manifest`` (merkle.rs:452-457)."""
    return hash_manifest_composed(hash_input_spec(m), hash_model_spec(m), hash_decode_spec(m), hash_output_spec(m))


# ---------------------------------------------------------------------------
# commit_minimal: crates/verilm-prover/src/lib.rs:336-499 (hashing parts)
# ---------------------------------------------------------------------------

@dataclass
class Commitment:
    """The hashed fields of ``BatchCommitment`` (types.rs:1710-1759)."""
    merkle_root: bytes
    io_root: bytes
    n_tokens: int
    prompt_hash: bytes
    seed_commitment: bytes
    n_prompt_tokens: Optional[int]
    kv_roots: List[bytes]
    trace_leaves: List[bytes]
    io_hashes: List[bytes]
    trace_tree: MerkleTree
    io_tree: MerkleTree
    kv_trees: List[MerkleTree]


def trace_leaves_of(all_retained, final_residuals=None, lp_hidden_bf16=None,
                    captured_logits_f32=None, n_prompt_tokens=None) -> List[bytes]:
    """Hot loop A of ``commit_minimal`` (prover/src/lib.rs:367-393).

    ``captured_logits_f32[j]`` binds to token ``gen_start + j`` with
    ``gen_start = n_prompt_tokens - 1`` (saturating); the optional lists bind
    only to indices they have (``.get(i)``).
    """
    gen_start = max(0, (n_prompt_tokens or 0) - 1) if n_prompt_tokens is not None else 0
    leaves = []
    for i, layers in enumerate(all_retained):
        fr = final_residuals[i] if final_residuals is not None and i < len(final_residuals) else None
        lp = lp_hidden_bf16[i] if lp_hidden_bf16 is not None and i < len(lp_hidden_bf16) else None
        cl = None
        if i >= gen_start and captured_logits_f32 is not None and (i - gen_start) < len(captured_logits_f32):
            cl = captured_logits_f32[i - gen_start]
        leaves.append(hash_retained_with_captured_logits(layers, fr, lp, cl))
    return leaves


def kv_tree_for_layer(layer_idx: int, k_rows: np.ndarray, v_rows: np.ndarray) -> MerkleTree:
    """Hot loop C of ``commit_minimal`` (prover/src/lib.rs:449-482) for one layer.

    ``k_rows``/``v_rows`` are f64 ``[n_pos, kv_dim]``; leaf ``pos`` is
    ``hash_kv_entry(layer_idx, pos, k[pos], v[pos])``.
    """
    leaves = [hash_kv_entry(layer_idx, p, k_rows[p], v_rows[p]) for p in range(k_rows.shape[0])]
    return build_tree(leaves)


def commit_minimal(all_retained, token_ids, prompt: bytes, sampling_seed: bytes,
                   final_residuals=None, kv_transcripts=None, lp_hidden_bf16=None,
                   captured_logits_f32=None, n_prompt_tokens=None) -> Commitment:
    """``commit_minimal`` (prover/src/lib.rs:336-499) minus the manifest.

    ``kv_transcripts`` is ``[layer] -> (k f64 [n_pos, kv_dim], v f64 [n_pos, kv_dim])``.
    """
    if len(all_retained) != len(token_ids):
        raise ValueError("retained state count must match token_ids")
    leaves = trace_leaves_of(all_retained, final_residuals, lp_hidden_bf16,
                             captured_logits_f32, n_prompt_tokens)
    ios = io_chain(leaves, token_ids, prompt)
    trace_tree = build_tree(leaves)
    io_tree = build_tree(ios)
    kv_trees = []
    if kv_transcripts is not None:
        for l, (k, v) in enumerate(kv_transcripts):
            kv_trees.append(kv_tree_for_layer(l, k, v))
    return Commitment(
        merkle_root=trace_tree.root, io_root=io_tree.root, n_tokens=len(all_retained),
        prompt_hash=hash_prompt(prompt), seed_commitment=hash_seed(sampling_seed),
        n_prompt_tokens=n_prompt_tokens, kv_roots=[t.root for t in kv_trees],
        trace_leaves=leaves, io_hashes=ios, trace_tree=trace_tree, io_tree=io_tree,
        kv_trees=kv_trees)


def build_retained_from_captures(o_proj_inputs: Sequence[bytes], scales: Sequence[float],
                                 n_layers: int, fwd_batch_sizes: Sequence[int]):
    """``commit_minimal_from_captures``' scale split (verilm-py/src/lib.rs:843-885)
    followed by ``build_retained_from_captures`` (prover/src/lib.rs:128-186).

    ``scales`` holds, per (fwd pass, layer), ``[B qkv | B o_proj | B gate | B down]``;
    ``scale_a`` is the o_proj block.  ``x_attn_i8`` is never placed in the
    retained state (prover/src/lib.rs:162-167).
    """
    out = []
    cursor = 0
    entry = 0
    per_fwd = []
    for bs in fwd_batch_sizes:
        layer_rows = []
        for _l in range(n_layers):
            a = bytes(o_proj_inputs[entry])
            s_o = scales[cursor + bs: cursor + 2 * bs]
            cursor += 4 * bs
            layer_rows.append((a, s_o))
            entry += 1
        per_fwd.append((bs, layer_rows))
    for bs, layer_rows in per_fwd:
        for b in range(bs):
            layers = []
            for a, s_o in layer_rows:
                dim = len(a) // bs
                layers.append(RetainedLayerState(a=a[b * dim:(b + 1) * dim], scale_a=float(np.float32(s_o[b]))))
            out.append(layers)
    return out


def packed_token_layers(packed_a: bytes, packed_scales: np.ndarray, n_layers: int, hidden_dim: int,
                        fwd_batch_sizes: Sequence[int]):
    """``PackedBatchState::hash_token``'s addressing (prover/src/lib.rs:639-681).

    a(f, l, b) at ``cum[f]*L*H + l*bs_f*H + b*H``; scale_a at
    ``packed_scales[(t*L + l)*4 + 1]``.
    """
    scales = np.asarray(packed_scales, dtype=np.float32)
    out = []
    cum = 0
    t = 0
    for bs in fwd_batch_sizes:
        for b in range(bs):
            layers = []
            for l in range(n_layers):
                off = cum * n_layers * hidden_dim + l * bs * hidden_dim + b * hidden_dim
                layers.append(RetainedLayerState(a=bytes(packed_a[off:off + hidden_dim]),
                                                 scale_a=float(scales[(t * n_layers + l) * 4 + 1])))
            out.append(layers)
            t += 1
        cum += bs
    return out


def sha256_blocks(msg_len: int) -> int:
    """FIPS 180-4 block count for a message of ``msg_len`` bytes."""
    return (msg_len + 9 + 63) // 64


# ---------------------------------------------------------------------------
# KV transcript from captured x_attn and the Wk/Wv weights:
# crates/verilm-prover/src/lib.rs:207-329 (compute_kv_transcript)
# ---------------------------------------------------------------------------

@dataclass
class RopeScaling:
    """``RopeScaling`` (crates/verilm-core/src/constants.rs:126-137)."""
    rope_type: str = "llama3"
    factor: float = 8.0
    low_freq_factor: float = 1.0
    high_freq_factor: float = 4.0
    original_max_position_embeddings: int = 8192


def scaled_inv_freq(d_head: int, rope_theta: float, scaling: Optional[RopeScaling] = None) -> List[float]:
    """``ModelConfig::scaled_inv_freq`` (constants.rs:253-297), f64 throughout.

    ``math.pow`` is the C library's ``pow``, the function Rust's ``f64::powf``
    calls on Linux, so the frequencies are the reference's bit for bit.
    """
    import math
    half = d_head // 2
    base = [1.0 / math.pow(rope_theta, float(2 * k) / float(d_head)) for k in range(half)]
    if scaling is None:
        return base
    if scaling.rope_type == "llama3":
        old_ctx = float(scaling.original_max_position_embeddings)
        low_wl = old_ctx / scaling.low_freq_factor
        high_wl = old_ctx / scaling.high_freq_factor
        out = []
        for f in base:
            wl = 2.0 * math.pi / f
            if wl < high_wl:
                out.append(f)
            elif wl > low_wl:
                out.append(f / scaling.factor)
            else:
                smooth = (old_ctx / wl - scaling.low_freq_factor) / (scaling.high_freq_factor - scaling.low_freq_factor)
                out.append(f * ((1.0 - smooth) / scaling.factor + smooth))
        return out
    if scaling.rope_type == "linear":
        return [f / scaling.factor for f in base]
    return base


def rope_cos_sin(n_positions: int, inv_freq: Sequence[float]):
    """cos/sin of ``position as f64 * inv_freq[i]`` (rope.rs:48-52), with the
    C library's ``cos``/``sin`` (what Rust's ``f64::cos``/``sin`` call)."""
    import math
    half = len(inv_freq)
    c = np.empty((n_positions, half), np.float64)
    s = np.empty((n_positions, half), np.float64)
    for p in range(n_positions):
        for i, f in enumerate(inv_freq):
            a = float(p) * f
            c[p, i] = math.cos(a)
            s[p, i] = math.sin(a)
    return c, s


def matmul_i32(w: np.ndarray, x: np.ndarray) -> np.ndarray:
    """``matmul_i32`` (crates/verilm-core/src/matmul.rs:12-22) for a batch of
    vectors: ``x [n][cols] i8`` times ``w [rows][cols] i8`` -> ``[n][rows] i32``.

    Computed as an f64 matrix product: every product and every partial sum is
    an integer below 2^53 in magnitude, so the f64 result is exact whatever the
    summation order, and equals the i32 sum while that does not overflow.
    """
    acc = np.asarray(x, np.float64) @ np.asarray(w, np.float64).T
    return acc.astype(np.int64).astype(np.int32)


def compute_kv_transcript(x_attn: np.ndarray, wk: Sequence[np.ndarray], wv: Sequence[np.ndarray],
                          scale_x: np.ndarray, n_kv_heads: int, d_head: int,
                          per_tensor=None, per_channel=None, biases=None,
                          rope_theta: float = 10000.0, rope_scaling: Optional[RopeScaling] = None):
    """``compute_kv_transcript`` (prover/src/lib.rs:207-329).

    x_attn: ``[n_tokens][n_layers][hidden]`` i8 (captured ``x_attn``, token
    order = position); wk/wv: per layer ``[kv_dim][hidden]`` i8; scale_x:
    ``[n_tokens][n_layers]`` f32 (``scale_x_attn``).  per_tensor: per layer
    ``(sw_k, sw_v)`` f32 or None; per_channel: per layer ``(cw_k, cw_v)``
    ``[kv_dim]`` f32 arrays (either may be None: that layer uses its per-tensor
    scale, 0.0 when absent, lib.rs:244-279); biases: per layer ``(b_k, b_v)``
    ``[kv_dim]`` f32 or None (lib.rs:283-302).  With neither scale list the
    toy path applies: clamp to i8, as f64 (lib.rs:307-316).

    Returns ``k_roped, v_deq`` as ``[n_layers][n_tokens][kv_dim]`` f64.
    Arithmetic order follows rope.rs exactly: per-tensor ``acc * (sw*sx)``
    (rope.rs:107-112), per-channel ``(acc*sw[c])*sx`` (rope.rs:124-138), then
    ``+ bias``, then RoPE per head ``h[i]c - h[i+half]s``, ``h[i+half]c + h[i]s``
    (rope.rs:38-60, 88-100); numpy elementwise f64 ops round each step, like
    Rust's (no fused multiply-add).
    """
    x_attn = np.asarray(x_attn, np.int8)
    n_tok, n_layers, hidden = x_attn.shape
    kv_dim = n_kv_heads * d_head
    use_rope = bool(per_tensor) or bool(per_channel)
    scale_x = np.asarray(scale_x, np.float32)
    k_out = np.empty((n_layers, n_tok, kv_dim), np.float64)
    v_out = np.empty((n_layers, n_tok, kv_dim), np.float64)
    if use_rope:
        inv = scaled_inv_freq(d_head, rope_theta, rope_scaling)
        cos, sin = rope_cos_sin(n_tok, inv)
    half = d_head // 2
    for l in range(n_layers):
        x = x_attn[:, l, :]
        k_acc = matmul_i32(wk[l], x)
        v_acc = matmul_i32(wv[l], x)
        if not use_rope:
            k_out[l] = np.clip(k_acc, -128, 127).astype(np.float64)
            v_out[l] = np.clip(v_acc, -128, 127).astype(np.float64)
            continue
        sx = scale_x[:, l].astype(np.float64)[:, None]
        vals = []
        for m, acc in ((0, k_acc), (1, v_acc)):
            ch = None
            if per_channel and l < len(per_channel) and per_channel[l] is not None \
                    and per_channel[l][m] is not None and len(per_channel[l][m]) > 0:
                ch = np.asarray(per_channel[l][m], np.float32).astype(np.float64)
            if ch is not None:
                f = (acc.astype(np.float64) * ch[None, :]) * sx
            else:
                sw = 0.0
                if per_tensor and l < len(per_tensor) and per_tensor[l] is not None:
                    sw = float(np.float32(per_tensor[l][m]))
                f = acc.astype(np.float64) * (sw * sx)
            if biases and l < len(biases) and biases[l] is not None and biases[l][m] is not None \
                    and len(biases[l][m]) > 0:
                f = f + np.asarray(biases[l][m], np.float32).astype(np.float64)[None, :]
            vals.append(f)
        k, v = vals
        kr = np.empty_like(k)
        for h in range(n_kv_heads):
            lo = k[:, h * d_head:h * d_head + half]
            hi = k[:, h * d_head + half:(h + 1) * d_head]
            kr[:, h * d_head:h * d_head + half] = lo * cos - hi * sin
            kr[:, h * d_head + half:(h + 1) * d_head] = hi * cos + lo * sin
        k_out[l] = kr
        v_out[l] = v
    return k_out, v_out
