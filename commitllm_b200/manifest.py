"""Deployment manifest and its four-spec commitment hashes.

The reference binds each commitment to the deployment configuration:
``commit_minimal`` splits the ``DeploymentManifest`` into InputSpec,
ModelSpec, DecodeSpec and OutputSpec, hashes each and composes them into
``manifest_hash`` (crates/verilm-prover/src/lib.rs:422-440;
crates/verilm-core/src/merkle.rs:324-457; types in
crates/verilm-core/src/types.rs:335-775).  These are once-per-request host
hashes of a few hundred bytes, so they run here on the host with SHA-256
(``hashlib``), beside the GPU commit of the request.

:func:`from_dict` mirrors the PyO3 boundary's ``extract_manifest``
(crates/verilm-py/src/lib.rs:173-490): the same keys, defaults, hex decoding
and errors (``ValueError`` for bad hex or a missing ``tokenizer_hash``,
``TypeError`` for a value of the wrong type), and the same normalisation
(``logit_bias`` sorted by token id, ``bad_word_ids`` sorted and deduplicated).
"""
from __future__ import annotations

import hashlib
import struct
from typing import Dict, List, Optional, Tuple

# DeploymentManifest fields in declaration order (types.rs:335-505) with
# their Rust types; the order is also the bincode field order.
FIELDS: List[Tuple[str, str]] = [
    ("tokenizer_hash", "b32"), ("temperature", "f32"), ("top_k", "u32"), ("top_p", "f32"),
    ("eos_policy", "str"), ("weight_hash", "opt_b32"), ("quant_hash", "opt_b32"),
    ("system_prompt_hash", "opt_b32"), ("repetition_penalty", "f32"), ("frequency_penalty", "f32"),
    ("presence_penalty", "f32"), ("logit_bias", "logit_bias"), ("bad_word_ids", "vec_u32"),
    ("guided_decoding", "str"), ("stop_sequences", "vec_str"), ("max_tokens", "u32"),
    ("chat_template_hash", "opt_b32"), ("rope_config_hash", "opt_b32"), ("rmsnorm_eps", "opt_f64"),
    ("sampler_version", "opt_str"), ("decode_mode", "opt_str"), ("bos_eos_policy", "opt_str"),
    ("truncation_policy", "opt_str"), ("special_token_policy", "opt_str"), ("padding_policy", "opt_str"),
    ("adapter_hash", "opt_b32"), ("n_layers", "opt_u32"), ("hidden_dim", "opt_u32"), ("vocab_size", "opt_u32"),
    ("embedding_merkle_root", "opt_b32"), ("quant_family", "opt_str"), ("scale_derivation", "opt_str"),
    ("quant_block_size", "opt_u32"), ("attn_backend", "opt_str"), ("attn_dtype", "opt_str"),
    ("kv_dim", "opt_u32"), ("ffn_dim", "opt_u32"), ("d_head", "opt_u32"), ("n_q_heads", "opt_u32"),
    ("n_kv_heads", "opt_u32"), ("rope_theta", "opt_f64"), ("min_tokens", "u32"), ("ignore_eos", "bool"),
    ("detokenization_policy", "opt_str"), ("eos_token_id", "opt_u32"),
]
KIND = dict(FIELDS)

# Defaults of extract_manifest for absent keys (lib.rs:189-330); Option fields default to None.
_DEFAULTS = {"temperature": 0.0, "top_k": 0, "top_p": 1.0, "eos_policy": "stop", "repetition_penalty": 1.0,
             "frequency_penalty": 0.0, "presence_penalty": 0.0, "logit_bias": [], "bad_word_ids": [],
             "guided_decoding": "", "stop_sequences": [], "max_tokens": 0, "min_tokens": 0, "ignore_eos": False}
# Keys whose Python None the boundary rejects instead of reading as absent
# (their get_item is not filtered for None, lib.rs:189-280).
_NONE_REJECTED = {"temperature", "top_k", "top_p", "eos_policy", "weight_hash", "quant_hash", "system_prompt_hash",
                  "repetition_penalty", "frequency_penalty", "presence_penalty", "logit_bias", "bad_word_ids",
                  "guided_decoding", "stop_sequences", "max_tokens"}


def _hex32(v, name: str) -> bytes:
    if not isinstance(v, str):
        raise TypeError(f"{name}: expected a hex string, got {type(v).__name__}")
    try:
        b = bytes.fromhex(v)
    except ValueError as e:
        raise ValueError(f"invalid {name} hex: {e}") from None
    if len(b) != 32:
        raise ValueError(f"{name} must be 32 bytes (64 hex chars), got {len(b)}")
    return b


def _u32(v, name: str) -> int:
    if isinstance(v, bool) or not isinstance(v, int):
        raise TypeError(f"{name}: expected an int")
    if not 0 <= v <= 0xFFFFFFFF:
        raise OverflowError(f"{name}: {v} does not fit u32")
    return int(v)


def _f32(v, name: str) -> float:
    if isinstance(v, bool) or not isinstance(v, (int, float)):
        raise TypeError(f"{name}: expected a float")
    return struct.unpack("<f", struct.pack("<f", float(v)))[0]


def _f64(v, name: str) -> float:
    if isinstance(v, bool) or not isinstance(v, (int, float)):
        raise TypeError(f"{name}: expected a float")
    return float(v)


def _str(v, name: str) -> str:
    if not isinstance(v, str):
        raise TypeError(f"{name}: expected a str")
    return v


def from_dict(d: Dict) -> Dict:
    """A ``DeploymentManifest`` (field name -> value: bytes for hashes, int,
    float, str, list) from the dict the serving layer builds
    (sidecar/verilm/server.py:951-999), as ``extract_manifest`` reads it."""
    if not isinstance(d, dict):
        raise TypeError("manifest must be a dict")
    if "tokenizer_hash" not in d or d["tokenizer_hash"] is None:
        raise ValueError("manifest missing tokenizer_hash")
    m: Dict = {}
    for name, kind in FIELDS:
        present = name in d and not (d[name] is None and name not in _NONE_REJECTED)
        if not present:
            m[name] = _DEFAULTS.get(name)
            continue
        v = d[name]
        if v is None:
            raise TypeError(f"{name}: None is not accepted")
        base = kind[4:] if kind.startswith("opt_") else kind
        if base == "b32":
            m[name] = _hex32(v, name)
        elif base == "u32":
            m[name] = _u32(v, name)
        elif base == "f32":
            m[name] = _f32(v, name)
        elif base == "f64":
            m[name] = _f64(v, name)
        elif base == "str":
            m[name] = _str(v, name)
        elif base == "bool":
            if not isinstance(v, bool):
                raise TypeError(f"{name}: expected a bool")
            m[name] = v
        elif base == "logit_bias":
            pairs = [(_u32(p[0], name), _f32(p[1], name)) for p in v]
            m[name] = sorted(pairs, key=lambda p: p[0])          # stable, by token id
        elif base == "vec_u32":
            m[name] = sorted(set(_u32(x, name) for x in v))
        elif base == "vec_str":
            m[name] = [_str(x, name) for x in v]
        else:  # pragma: no cover - FIELDS is closed
            raise AssertionError(kind)
    return m


# ---------------------------------------------------------------------------
# Spec encodings (merkle.rs:324-457).  Each spec is one SHA-256 over a tag and
# its fields in a fixed order: optional values as 0x00 | 0x01 || value,
# strings and lists length-prefixed with a u32le count, numbers little-endian.
# ---------------------------------------------------------------------------

class _Msg:
    def __init__(self, tag: bytes):
        self.h = hashlib.sha256(tag)

    def raw(self, b: bytes) -> "_Msg":
        self.h.update(b)
        return self

    def u32(self, v: int) -> "_Msg":
        return self.raw(struct.pack("<I", v))

    def f32(self, v: float) -> "_Msg":
        return self.raw(struct.pack("<f", v))

    def text(self, s: str) -> "_Msg":
        b = s.encode()
        return self.u32(len(b)).raw(b)

    def opt(self, v, put) -> "_Msg":
        if v is None:
            return self.raw(b"\x00")
        self.raw(b"\x01")
        put(v)
        return self

    def opt32(self, v: Optional[bytes]) -> "_Msg":
        return self.opt(v, self.raw)

    def opt_u32(self, v: Optional[int]) -> "_Msg":
        return self.opt(v, self.u32)

    def opt_f64(self, v: Optional[float]) -> "_Msg":
        return self.opt(v, lambda x: self.raw(struct.pack("<d", x)))

    def opt_text(self, v: Optional[str]) -> "_Msg":
        return self.opt(v, self.text)

    def digest(self) -> bytes:
        return self.h.digest()


def input_spec_hash(m: Dict) -> bytes:
    """hash_input_spec (merkle.rs:324-335) of the manifest's InputSpec (types.rs:560-572)."""
    return (_Msg(b"vi-input-v1").raw(m["tokenizer_hash"]).opt32(m["system_prompt_hash"])
            .opt32(m["chat_template_hash"]).opt_text(m["bos_eos_policy"]).opt_text(m["truncation_policy"])
            .opt_text(m["special_token_policy"]).opt_text(m["padding_policy"]).digest())


def model_spec_hash(m: Dict) -> bytes:
    """hash_model_spec (merkle.rs:338-367) of the ModelSpec (types.rs:653-677).
    attn_backend and attn_dtype are carried by the spec but not hashed."""
    h = _Msg(b"vi-model-v1").opt32(m["weight_hash"]).opt32(m["quant_hash"]).opt32(m["rope_config_hash"])
    h.opt_f64(m["rmsnorm_eps"]).opt32(m["adapter_hash"])
    for k in ("n_layers", "hidden_dim", "vocab_size"):
        h.opt_u32(m[k])
    h.opt32(m["embedding_merkle_root"]).opt_text(m["quant_family"]).opt_text(m["scale_derivation"])
    h.opt_u32(m["quant_block_size"])
    for k in ("kv_dim", "ffn_dim", "d_head", "n_q_heads", "n_kv_heads"):
        h.opt_u32(m[k])
    return h.opt_f64(m["rope_theta"]).digest()


def decode_spec_hash(m: Dict) -> bytes:
    """hash_decode_spec (merkle.rs:370-401) of the DecodeSpec (types.rs:719-733)."""
    h = _Msg(b"vi-decode-v1").f32(m["temperature"]).u32(m["top_k"]).f32(m["top_p"])
    h.f32(m["repetition_penalty"]).f32(m["frequency_penalty"]).f32(m["presence_penalty"])
    h.u32(len(m["logit_bias"]))
    for tok, bias in m["logit_bias"]:
        h.u32(tok).f32(bias)
    h.u32(len(m["bad_word_ids"]))
    for tok in m["bad_word_ids"]:
        h.u32(tok)
    h.text(m["guided_decoding"]).opt_text(m["sampler_version"])
    return h.opt_text(m["decode_mode"]).digest()


def output_spec_hash(m: Dict) -> bytes:
    """hash_output_spec (merkle.rs:404-427) of the OutputSpec (types.rs:762-774).
    eos_policy is hashed without a length prefix, as the reference does."""
    h = _Msg(b"vi-output-v1").raw(m["eos_policy"].encode()).u32(len(m["stop_sequences"]))
    for s in m["stop_sequences"]:
        h.text(s)
    h.u32(m["max_tokens"]).u32(m["min_tokens"]).raw(bytes([1 if m["ignore_eos"] else 0]))
    return h.opt_text(m["detokenization_policy"]).opt_u32(m["eos_token_id"]).digest()


def compose(h_input: bytes, h_model: bytes, h_decode: bytes, h_output: bytes) -> bytes:
    """hash_manifest_composed (merkle.rs:432-446): M = H("vi-manifest-v4" || the four spec hashes)."""
    return _Msg(b"vi-manifest-v4").raw(h_input).raw(h_model).raw(h_decode).raw(h_output).digest()


def spec_hashes(m: Dict) -> Dict[str, bytes]:
    """The five BatchCommitment fields of commit_minimal (prover/src/lib.rs:422-440)."""
    hi, hm, hd, ho = input_spec_hash(m), model_spec_hash(m), decode_spec_hash(m), output_spec_hash(m)
    return {"manifest_hash": compose(hi, hm, hd, ho), "input_spec_hash": hi, "model_spec_hash": hm,
            "decode_spec_hash": hd, "output_spec_hash": ho}


def to_dict(m: Dict) -> Dict:
    """The inverse of :func:`from_dict`: hashes as hex, for logging and JSON."""
    out = {}
    for name, kind in FIELDS:
        v = m[name]
        out[name] = v.hex() if isinstance(v, (bytes, bytearray)) else (list(map(list, v)) if kind == "logit_bias" else v)
    return out
