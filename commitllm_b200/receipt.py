"""Audit receipts: ``V4AuditResponse`` in the reference's wire formats.

Binary: ``"VV4A" || zstd(bincode v1 of V4AuditResponse)`` at zstd level 3
(crates/verilm-core/src/serialize.rs:17-59), the bytes ``audit_v4_binary``
returns (crates/verilm-py/src/lib.rs:699-712).  JSON: serde_json of the same
struct, the string ``audit_v4`` returns (lib.rs:683-695).

bincode v1 with default options writes a struct as its fields in declaration
order with no framing: integers fixed-width little-endian, ``usize`` and
every length as u64, ``bool`` as one byte, ``Option`` as a 0/1 tag byte then
the value, a unit enum variant as its u32 index, ``[u8; 32]`` as 32 raw bytes.
The schemas below follow the field order of crates/verilm-core/src/types.rs.

Values are plain Python: a struct is a dict keyed by the Rust field names,
``[u8; 32]`` and ``Vec<u8>`` / ``Vec<i8>`` are ``bytes``, numeric vectors are
numpy arrays, ``Option::None`` is ``None``.  zstd is the system
``libzstd.so.1``.
"""
from __future__ import annotations

import ctypes
import json
import struct
from typing import Any, Dict, List, Tuple

import numpy as np

from . import manifest as _manifest

MAGIC = b"VV4A"
ZSTD_LEVEL = 3


# ---------------------------------------------------------------------------
# Schema vocabulary
# ---------------------------------------------------------------------------

class T:
    """A bincode type: ``kind`` plus its parameters."""

    def __init__(self, kind: str, *args):
        self.kind, self.args = kind, args


U8, U32, U64, F32, F64, BOOL, STR, B32, BYTES = (T(k) for k in ("u8", "u32", "u64", "f32", "f64", "bool", "str",
                                                                 "b32", "bytes"))
USIZE = U64


def VEC(t: T) -> T:
    return T("vec", t)


def OPT(t: T) -> T:
    return T("opt", t)


def ARR(dtype: str) -> T:
    """A numeric Vec (u64 length + packed little-endian elements), as a numpy array."""
    return T("arr", np.dtype(dtype))


def TUP(*ts: T) -> T:
    return T("tup", *ts)


def STRUCT(name: str, fields: List[Tuple[str, T]]) -> T:
    return T("struct", name, fields)


def ENUM(name: str, variants: List[str]) -> T:
    """A unit-variant enum, valued by variant name."""
    return T("enum", name, variants)


MERKLE_PROOF = STRUCT("MerkleProof", [("leaf_index", U32), ("siblings", VEC(B32))])          # merkle.rs:303-307
RETAINED_LAYER = STRUCT("RetainedLayerState", [                                               # types.rs:1201-1219
    ("a", BYTES), ("scale_a", F32), ("x_attn_i8", OPT(BYTES)), ("scale_x_attn", OPT(F32))])
RETAINED_TOKEN = STRUCT("RetainedTokenState", [("layers", VEC(RETAINED_LAYER))])               # types.rs:1227-1229
KV_ENTRY = STRUCT("KvEntry", [("k_roped", ARR("<f8")), ("v_deq", ARR("<f8"))])                # types.rs:1244-1251
WITNESSED_SCORES = STRUCT("WitnessedScores", [                                                # types.rs:1327-1331
    ("scores", ARR("<f4")), ("n_q_heads", USIZE), ("seq_len", USIZE)])
SHELL_LAYER = STRUCT("ShellLayerOpening", [                                                   # types.rs:1345-1364
    ("attn_out", ARR("<i4")), ("g", ARR("<i4")), ("u", ARR("<i4")), ("ffn_out", ARR("<i4")),
    ("q", OPT(ARR("<i4"))), ("k", OPT(ARR("<i4"))), ("v", OPT(ARR("<i4"))),
    ("scale_x_attn", F32), ("scale_x_ffn", F32), ("scale_h", F32)])
SHELL_TOKEN = STRUCT("ShellTokenOpening", [                                                   # types.rs:1378-1397
    ("layers", VEC(SHELL_LAYER)), ("layer_indices", OPT(ARR("<u8"))), ("initial_residual", OPT(ARR("<f4"))),
    ("embedding_proof", OPT(MERKLE_PROOF)), ("final_residual", OPT(ARR("<f4"))),
    ("logits_i32", OPT(ARR("<i4"))), ("lp_hidden_bf16", OPT(ARR("<u2"))), ("captured_logits_f32", OPT(ARR("<f4")))])

_MANIFEST_T = {"b32": B32, "f32": F32, "u32": U32, "str": STR, "f64": F64, "bool": BOOL,
               "logit_bias": VEC(TUP(U32, F32)), "vec_u32": VEC(U32), "vec_str": VEC(STR)}
DEPLOYMENT_MANIFEST = STRUCT("DeploymentManifest", [                                          # types.rs:335-505
    (name, OPT(_MANIFEST_T[kind[4:]]) if kind.startswith("opt_") else _MANIFEST_T[kind])
    for name, kind in _manifest.FIELDS])
COMMITMENT_VERSION = ENUM("CommitmentVersion", ["V4"])                                         # types.rs:1692-1694
BATCH_COMMITMENT = STRUCT("BatchCommitment", [                                                # types.rs:1710-1759
    ("merkle_root", B32), ("io_root", B32), ("n_tokens", U32), ("manifest_hash", OPT(B32)),
    ("input_spec_hash", OPT(B32)), ("model_spec_hash", OPT(B32)), ("decode_spec_hash", OPT(B32)),
    ("output_spec_hash", OPT(B32)), ("version", COMMITMENT_VERSION), ("prompt_hash", OPT(B32)),
    ("seed_commitment", OPT(B32)), ("n_prompt_tokens", OPT(U32)), ("kv_roots", VEC(B32))])
V4_AUDIT_RESPONSE = STRUCT("V4AuditResponse", [                                               # types.rs:1475-1567
    ("token_index", U32), ("retained", RETAINED_TOKEN), ("merkle_proof", MERKLE_PROOF), ("io_proof", MERKLE_PROOF),
    ("token_id", U32), ("prev_io_hash", B32), ("prefix_leaf_hashes", VEC(B32)),
    ("prefix_merkle_proofs", VEC(MERKLE_PROOF)), ("prefix_token_ids", ARR("<u4")), ("commitment", BATCH_COMMITMENT),
    ("revealed_seed", B32), ("shell_opening", OPT(SHELL_TOKEN)), ("manifest", OPT(DEPLOYMENT_MANIFEST)),
    ("prompt", OPT(BYTES)), ("n_prompt_tokens", OPT(U32)), ("output_text", OPT(STR)),
    ("prefix_embedding_rows", OPT(VEC(ARR("<f4")))), ("prefix_embedding_proofs", OPT(VEC(MERKLE_PROOF))),
    ("prefix_retained", OPT(VEC(RETAINED_TOKEN))), ("prefix_shell_openings", OPT(VEC(SHELL_TOKEN))),
    ("kv_entries", OPT(VEC(VEC(KV_ENTRY)))), ("kv_proofs", OPT(VEC(VEC(MERKLE_PROOF)))),
    ("witnessed_scores", OPT(VEC(WITNESSED_SCORES)))])


# ---------------------------------------------------------------------------
# bincode v1
# ---------------------------------------------------------------------------

_FIXED = {"u8": "<B", "u32": "<I", "u64": "<Q", "f32": "<f", "f64": "<d"}


def _enc(t: T, v: Any, out: bytearray) -> None:
    k = t.kind
    if k in _FIXED:
        out += struct.pack(_FIXED[k], v)
    elif k == "bool":
        out.append(1 if v else 0)
    elif k == "b32":
        b = bytes(v)
        if len(b) != 32:
            raise ValueError(f"[u8; 32] value of {len(b)} bytes")
        out += b
    elif k == "bytes":
        b = bytes(v)
        out += struct.pack("<Q", len(b)) + b
    elif k == "str":
        b = v.encode()
        out += struct.pack("<Q", len(b)) + b
    elif k == "arr":
        a = np.ascontiguousarray(np.asarray(v, dtype=t.args[0]))
        out += struct.pack("<Q", a.size) + a.tobytes()
    elif k == "vec":
        out += struct.pack("<Q", len(v))
        for x in v:
            _enc(t.args[0], x, out)
    elif k == "opt":
        if v is None:
            out.append(0)
        else:
            out.append(1)
            _enc(t.args[0], v, out)
    elif k == "tup":
        for tt, x in zip(t.args, v):
            _enc(tt, x, out)
    elif k == "struct":
        for name, ft in t.args[1]:
            if name not in v:
                raise KeyError(f"{t.args[0]}.{name} missing")
            _enc(ft, v[name], out)
    elif k == "enum":
        out += struct.pack("<I", t.args[1].index(v))
    else:  # pragma: no cover - the vocabulary is closed
        raise AssertionError(k)


class _Reader:
    def __init__(self, buf: bytes):
        self.b, self.o = memoryview(buf), 0

    def take(self, n: int) -> bytes:
        if n < 0 or self.o + n > len(self.b):
            raise ValueError("bincode: truncated input")
        v = bytes(self.b[self.o:self.o + n])
        self.o += n
        return v

    def fixed(self, fmt: str):
        return struct.unpack(fmt, self.take(struct.calcsize(fmt)))[0]

    def length(self) -> int:
        n = self.fixed("<Q")
        if n > len(self.b) - self.o:
            raise ValueError("bincode: length past the end of the input")
        return n


def _dec(t: T, r: _Reader) -> Any:
    k = t.kind
    if k in _FIXED:
        return r.fixed(_FIXED[k])
    if k == "bool":
        b = r.take(1)[0]
        if b > 1:
            raise ValueError("bincode: bad bool")
        return bool(b)
    if k == "b32":
        return r.take(32)
    if k == "bytes":
        return r.take(r.length())
    if k == "str":
        return r.take(r.length()).decode()
    if k == "arr":
        dt = t.args[0]
        n = r.length()
        return np.frombuffer(r.take(n * dt.itemsize), dtype=dt).copy()
    if k == "vec":
        return [_dec(t.args[0], r) for _ in range(r.length())]
    if k == "opt":
        tag = r.take(1)[0]
        if tag > 1:
            raise ValueError("bincode: bad Option tag")
        return _dec(t.args[0], r) if tag else None
    if k == "tup":
        return tuple(_dec(tt, r) for tt in t.args)
    if k == "struct":
        return {name: _dec(ft, r) for name, ft in t.args[1]}
    if k == "enum":
        i = r.fixed("<I")
        if i >= len(t.args[1]):
            raise ValueError(f"bincode: bad {t.args[0]} variant {i}")
        return t.args[1][i]
    raise AssertionError(k)  # pragma: no cover


def bincode_encode(t: T, value: Any) -> bytes:
    out = bytearray()
    _enc(t, value, out)
    return bytes(out)


def bincode_decode(t: T, data: bytes) -> Any:
    r = _Reader(data)
    v = _dec(t, r)
    if r.o != len(r.b):
        raise ValueError(f"bincode: {len(r.b) - r.o} trailing bytes")
    return v


# ---------------------------------------------------------------------------
# zstd framing (serialize.rs:43-59)
# ---------------------------------------------------------------------------

_zstd = None


def _libzstd():
    global _zstd
    if _zstd is None:
        lib = ctypes.CDLL("libzstd.so.1")
        lib.ZSTD_compressBound.restype = ctypes.c_size_t
        lib.ZSTD_compressBound.argtypes = [ctypes.c_size_t]
        lib.ZSTD_compress.restype = ctypes.c_size_t
        lib.ZSTD_compress.argtypes = [ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_int]
        lib.ZSTD_decompress.restype = ctypes.c_size_t
        lib.ZSTD_decompress.argtypes = [ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_size_t]
        lib.ZSTD_getFrameContentSize.restype = ctypes.c_ulonglong
        lib.ZSTD_getFrameContentSize.argtypes = [ctypes.c_char_p, ctypes.c_size_t]
        lib.ZSTD_isError.restype = ctypes.c_uint
        lib.ZSTD_isError.argtypes = [ctypes.c_size_t]
        _zstd = lib
    return _zstd


def zstd_compress(data: bytes, level: int = ZSTD_LEVEL) -> bytes:
    lib = _libzstd()
    cap = lib.ZSTD_compressBound(len(data))
    out = ctypes.create_string_buffer(cap)
    n = lib.ZSTD_compress(out, cap, data, len(data), level)
    if lib.ZSTD_isError(n):
        raise RuntimeError("zstd compression failed")
    return out.raw[:n]


def zstd_decompress(data: bytes, max_size: int = 1 << 34) -> bytes:
    lib = _libzstd()
    size = lib.ZSTD_getFrameContentSize(data, len(data))
    if size >= (1 << 63):
        raise ValueError("zstd frame without a content size")
    if size > max_size:
        raise ValueError(f"zstd frame of {size} bytes exceeds the {max_size}-byte limit")
    out = ctypes.create_string_buffer(max(int(size), 1))
    n = lib.ZSTD_decompress(out, size, data, len(data))
    if lib.ZSTD_isError(n):
        raise ValueError("zstd decompression failed")
    return out.raw[:n]


def serialize_v4_audit(resp: Dict) -> bytes:
    """``serialize_v4_audit`` (serialize.rs:43-50)."""
    return MAGIC + zstd_compress(bincode_encode(V4_AUDIT_RESPONSE, resp))


def deserialize_v4_audit(data: bytes) -> Dict:
    """``deserialize_v4_audit`` (serialize.rs:52-59): ValueError on a bad magic or body."""
    if len(data) < 4 or bytes(data[:4]) != MAGIC:
        raise ValueError("invalid V4 audit magic")
    return bincode_decode(V4_AUDIT_RESPONSE, zstd_decompress(bytes(data[4:])))


# ---------------------------------------------------------------------------
# serde_json form
# ---------------------------------------------------------------------------

def _json_f32(x: float):
    x = np.float32(x)
    if not np.isfinite(x):
        return None                       # serde_json writes non-finite floats as null
    return float(str(x))                  # the shortest decimal that reads back as this f32


def _to_json(t: T, v: Any):
    k = t.kind
    if v is None:
        return None
    if k in ("u8", "u32", "u64"):
        return int(v)
    if k == "f32":
        return _json_f32(v)
    if k == "f64":
        return float(v) if np.isfinite(v) else None
    if k == "bool":
        return bool(v)
    if k == "str":
        return v
    if k == "b32":
        return list(bytes(v))
    if k == "bytes":
        return list(bytes(v))
    if k == "arr":
        dt = t.args[0]
        if dt.kind == "f":
            if dt.itemsize == 8:
                return [float(x) if np.isfinite(x) else None for x in np.asarray(v)]
            return [_json_f32(x) for x in np.asarray(v)]
        return [int(x) for x in np.asarray(v)]
    if k == "vec":
        return [_to_json(t.args[0], x) for x in v]
    if k == "opt":
        return _to_json(t.args[0], v)
    if k == "tup":
        return [_to_json(tt, x) for tt, x in zip(t.args, v)]
    if k == "enum":
        return v
    if k == "struct":
        name = t.args[0]
        out = {}
        for fname, ft in t.args[1]:
            if name == "KvEntry":
                # f64_hex_vec (types.rs:1253-1317): each f64 as the hex of its LE bytes
                out[fname] = [x.tobytes().hex() for x in np.asarray(v[fname], dtype="<f8")]
            elif name == "RetainedLayerState" and fname in ("a", "x_attn_i8"):
                out[fname] = None if v[fname] is None else np.frombuffer(bytes(v[fname]), np.int8).tolist()
            else:
                out[fname] = _to_json(ft, v[fname])
        return out
    raise AssertionError(k)  # pragma: no cover


def v4_audit_json(resp: Dict) -> str:
    """serde_json of ``V4AuditResponse`` (what ``audit_v4`` returns)."""
    return json.dumps(_to_json(V4_AUDIT_RESPONSE, resp), separators=(",", ":"))
