"""Regenerate ``reference_pins.json`` from the reference's own test data.

Run in a container that has the reference checked out (read-only); its
root is a required argument::

    python tests/golden/make_golden.py <path of the reference checkout>

What it extracts (all read as data, nothing of the reference is executed):

* ``crates/verilm-verify/tests/fixtures/v4_audit_canonical.bin`` and
  ``v4_audit_fullbridge.bin``: frozen ``V4AuditResponse`` receipts written by
  ``tests/gen_fixtures.rs:295-420``.  Wire format ``"VV4A" || zstd(bincode v1)``
  (``crates/verilm-core/src/serialize.rs:43-59``).  Decoded here with the
  system ``libzstd.so.1`` and a bincode-v1 reader for the leading fields of
  ``V4AuditResponse`` (types.rs:1475-1502) and ``BatchCommitment``
  (types.rs:1710-1759).  Their file SHA-256 is pinned by
  ``crates/verilm-verify/tests/cross_version.rs:431-442``.
  The whole receipt is decoded (through ``witnessed_scores``, the last field,
  to the end of the buffer); the decompressed bincode is kept as hex so that
  a bincode writer can be checked byte for byte, and the fullbridge receipt's
  ``manifest`` pins the four-spec hashes its commitment carries.
* The golden hex pins of ``golden_e2e_verify``
  (``crates/verilm-test-vectors/tests/golden_conformance.rs:206-261``): the
  same toy model (seed 12345, input 0..16) as the canonical fixture, prompt
  ``b"golden test"``, token 42.
* ``golden_manifest`` and its pinned ``hash_manifest`` / ``hash_model_spec``
  hex (``golden_conformance.rs:132-201``), read from the Rust struct literal.

The prompts and token ids are the inputs written in those two test files.
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import os
import re
import struct
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def zstd_decompress(data: bytes) -> bytes:
    lib = ctypes.CDLL("libzstd.so.1")
    lib.ZSTD_getFrameContentSize.restype = ctypes.c_ulonglong
    lib.ZSTD_getFrameContentSize.argtypes = [ctypes.c_char_p, ctypes.c_size_t]
    lib.ZSTD_decompress.restype = ctypes.c_size_t
    lib.ZSTD_decompress.argtypes = [ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_size_t]
    lib.ZSTD_isError.restype = ctypes.c_uint
    lib.ZSTD_isError.argtypes = [ctypes.c_size_t]
    size = lib.ZSTD_getFrameContentSize(data, len(data))
    if size >= (1 << 63):
        # encode_all streams without a content size: bound the output instead.
        size = 64 << 20
    out = ctypes.create_string_buffer(size)
    n = lib.ZSTD_decompress(out, size, data, len(data))
    if lib.ZSTD_isError(n):
        raise ValueError("zstd: decompression failed")
    return out.raw[:n]


class Bincode:
    """bincode v1 default options: fixed-width little-endian ints, u64 lengths."""

    def __init__(self, buf: bytes):
        self.b, self.o = buf, 0

    def take(self, n):
        v = self.b[self.o:self.o + n]
        if len(v) != n:
            raise ValueError("truncated")
        self.o += n
        return v

    def u8(self):
        return self.take(1)[0]

    def u32(self):
        return struct.unpack("<I", self.take(4))[0]

    def u64(self):
        return struct.unpack("<Q", self.take(8))[0]

    def f32_bits(self):
        return struct.unpack("<I", self.take(4))[0]

    def arr32(self):
        return self.take(32)

    def option(self, f):
        tag = self.u8()
        if tag == 0:
            return None
        if tag != 1:
            raise ValueError("bad option tag")
        return f()

    def vec(self, f):
        return [f() for _ in range(self.u64())]

    def bytes_vec(self):
        return self.take(self.u64())

    def bytes_vec_f64(self):
        n = self.u64()
        return self.take(8 * n).hex()


def read_proof(r: Bincode):
    return {"leaf_index": r.u32(), "siblings": [s.hex() for s in r.vec(r.arr32)]}


def _prefix_len(blob: bytes) -> int:
    """Bytes of the decompressed receipt that read_v4_audit_prefix consumes."""
    holder = {}
    read_v4_audit_prefix(blob, holder)
    return holder["end"]


def read_v4_audit_prefix(blob: bytes, _end=None):
    if blob[:4] != b"VV4A":
        raise ValueError("not a VV4A receipt")
    r = Bincode(zstd_decompress(blob[4:]))
    out = {"token_index": r.u32()}
    layers = []
    for _ in range(r.u64()):
        a = r.bytes_vec()
        scale_a = r.f32_bits()
        xa = r.option(r.bytes_vec)
        sx = r.option(r.f32_bits)
        layers.append({"a": a.hex(), "scale_a_bits": scale_a,
                       "x_attn_i8": None if xa is None else xa.hex(),
                       "scale_x_attn_bits": sx})
    out["retained_layers"] = layers
    out["merkle_proof"] = read_proof(r)
    out["io_proof"] = read_proof(r)
    out["token_id"] = r.u32()
    out["prev_io_hash"] = r.arr32().hex()
    out["prefix_leaf_hashes"] = [h.hex() for h in r.vec(r.arr32)]
    out["prefix_merkle_proofs"] = r.vec(lambda: read_proof(r))
    out["prefix_token_ids"] = r.vec(r.u32)
    c = {}
    c["merkle_root"] = r.arr32().hex()
    c["io_root"] = r.arr32().hex()
    c["n_tokens"] = r.u32()
    for k in ("manifest_hash", "input_spec_hash", "model_spec_hash", "decode_spec_hash",
              "output_spec_hash"):
        v = r.option(r.arr32)
        c[k] = None if v is None else v.hex()
    c["version"] = r.u32()
    v = r.option(r.arr32)
    c["prompt_hash"] = None if v is None else v.hex()
    v = r.option(r.arr32)
    c["seed_commitment"] = None if v is None else v.hex()
    c["n_prompt_tokens"] = r.option(r.u32)
    c["kv_roots"] = [x.hex() for x in r.vec(r.arr32)]
    out["commitment"] = c
    out["revealed_seed"] = r.arr32().hex()
    if _end is not None:
        _end["end"] = r.o
    return out


def _b32(r):
    return r.arr32().hex()


def read_manifest(r: Bincode):
    """DeploymentManifest (types.rs:335-505), fields in declaration order."""
    f32 = lambda: struct.unpack("<f", r.take(4))[0]
    f64 = lambda: struct.unpack("<d", r.take(8))[0]
    text = lambda: r.bytes_vec().decode()
    m = {}
    m["tokenizer_hash"] = _b32(r)
    m["temperature"] = f32()
    m["top_k"] = r.u32()
    m["top_p"] = f32()
    m["eos_policy"] = text()
    for k in ("weight_hash", "quant_hash", "system_prompt_hash"):
        m[k] = r.option(lambda: _b32(r))
    for k in ("repetition_penalty", "frequency_penalty", "presence_penalty"):
        m[k] = f32()
    m["logit_bias"] = r.vec(lambda: [r.u32(), f32()])
    m["bad_word_ids"] = r.vec(r.u32)
    m["guided_decoding"] = text()
    m["stop_sequences"] = r.vec(text)
    m["max_tokens"] = r.u32()
    m["chat_template_hash"] = r.option(lambda: _b32(r))
    m["rope_config_hash"] = r.option(lambda: _b32(r))
    m["rmsnorm_eps"] = r.option(f64)
    for k in ("sampler_version", "decode_mode", "bos_eos_policy", "truncation_policy", "special_token_policy",
              "padding_policy"):
        m[k] = r.option(text)
    m["adapter_hash"] = r.option(lambda: _b32(r))
    for k in ("n_layers", "hidden_dim", "vocab_size"):
        m[k] = r.option(r.u32)
    m["embedding_merkle_root"] = r.option(lambda: _b32(r))
    m["quant_family"] = r.option(text)
    m["scale_derivation"] = r.option(text)
    m["quant_block_size"] = r.option(r.u32)
    m["attn_backend"] = r.option(text)
    m["attn_dtype"] = r.option(text)
    for k in ("kv_dim", "ffn_dim", "d_head", "n_q_heads", "n_kv_heads"):
        m[k] = r.option(r.u32)
    m["rope_theta"] = r.option(f64)
    m["min_tokens"] = r.u32()
    m["ignore_eos"] = bool(r.u8())
    m["detokenization_policy"] = r.option(text)
    m["eos_token_id"] = r.option(r.u32)
    return m


def _i32_vec(r):
    n = r.u64()
    return list(struct.unpack(f"<{n}i", r.take(4 * n)))


def _f32_vec(r):
    n = r.u64()
    return list(struct.unpack(f"<{n}f", r.take(4 * n)))


def read_shell_opening(r: Bincode):
    """ShellTokenOpening (types.rs:1378-1397) with its ShellLayerOpenings (1345-1364)."""
    def layer():
        d = {k: _i32_vec(r) for k in ("attn_out", "g", "u", "ffn_out")}
        for k in ("q", "k", "v"):
            d[k] = r.option(lambda: _i32_vec(r))
        for k in ("scale_x_attn", "scale_x_ffn", "scale_h"):
            d[k] = struct.unpack("<f", r.take(4))[0]
        return d
    o = {"layers": r.vec(layer)}
    o["layer_indices"] = r.option(lambda: r.vec(r.u64))
    o["initial_residual"] = r.option(lambda: _f32_vec(r))
    o["embedding_proof"] = r.option(lambda: read_proof(r))
    o["final_residual"] = r.option(lambda: _f32_vec(r))
    o["logits_i32"] = r.option(lambda: _i32_vec(r))
    o["lp_hidden_bf16"] = r.option(lambda: r.vec(lambda: struct.unpack("<H", r.take(2))[0]))
    o["captured_logits_f32"] = r.option(lambda: _f32_vec(r))
    return o


def read_v4_audit_rest(r: Bincode, out: dict) -> None:
    """The fields of V4AuditResponse after revealed_seed (types.rs:1502-1567)."""
    out["shell_opening"] = r.option(lambda: read_shell_opening(r))
    out["manifest"] = r.option(lambda: read_manifest(r))
    out["prompt_field"] = r.option(lambda: r.bytes_vec().hex())
    out["n_prompt_tokens"] = r.option(r.u32)
    out["output_text"] = r.option(lambda: r.bytes_vec().decode())
    out["prefix_embedding_rows"] = r.option(lambda: r.vec(lambda: _f32_vec(r)))
    out["prefix_embedding_proofs"] = r.option(lambda: r.vec(lambda: read_proof(r)))
    if r.u8() != 0:
        raise ValueError("prefix_retained present: not decoded here")
    if r.u8() != 0:
        raise ValueError("prefix_shell_openings present: not decoded here")
    out["prefix_retained"] = out["prefix_shell_openings"] = None
    out["kv_entries"] = r.option(lambda: r.vec(lambda: r.vec(lambda: {"k_roped": r.bytes_vec_f64(),
                                                                     "v_deq": r.bytes_vec_f64()})))
    out["kv_proofs"] = r.option(lambda: r.vec(lambda: r.vec(lambda: read_proof(r))))
    out["witnessed_scores"] = r.option(lambda: r.vec(lambda: {"scores": _f32_vec(r), "n_q_heads": r.u64(),
                                                              "seq_len": r.u64()}))
    if r.o != len(r.b):
        raise ValueError(f"{len(r.b) - r.o} bytes left after witnessed_scores")


def _rust_value(text: str):
    """A value of golden_manifest()'s struct literal as the Python value the
    manifest dicts use: [u8; 32] as hex, Option as None, strings, numbers."""
    t = text.strip()
    if t == "None":
        return None
    if t.startswith("Some(") and t.endswith(")"):
        return _rust_value(t[5:-1])
    m = re.fullmatch(r"\[(0x[0-9a-fA-F]+|\d+)u?8?; 32\]", t)
    if m:
        return bytes([int(m.group(1), 0)] * 32).hex()
    if t in ("vec![]",):
        return []
    if t == "String::new()":
        return ""
    m = re.fullmatch(r'"(.*)"\.into\(\)', t)
    if m:
        return m.group(1)
    if t in ("true", "false"):
        return t == "true"
    if re.fullmatch(r"-?\d+", t):
        return int(t)
    return float(t)


def golden_manifest(ref_root: str):
    src = open(os.path.join(ref_root, "crates/verilm-test-vectors/tests/golden_conformance.rs")).read()
    body = re.search(r"fn golden_manifest\(\) -> DeploymentManifest \{\s*DeploymentManifest \{(.*?)\n    \}\n\}",
                     src, flags=re.S).group(1)
    m = {}
    for line in body.splitlines():
        line = line.strip().rstrip(",")
        if not line or line.startswith("//"):
            continue
        k, v = line.split(":", 1)
        m[k.strip()] = _rust_value(v)
    pins = {}
    for test, key in (("golden_manifest_hash", "manifest_hash"), ("golden_model_spec_hash", "model_spec_hash")):
        blk = re.search(r"fn " + test + r"\(\) \{(.*?)\n\}", src, flags=re.S).group(1)
        pins[key] = re.search(r'"([0-9a-f]{64})"', blk).group(1)
    return {"manifest": m, **pins, "source": "golden_conformance.rs:132-201"}


def main(ref_root: str) -> None:
    fx = os.path.join(ref_root, "crates/verilm-verify/tests/fixtures")
    pins = {"source": "lambdaclass/CommitLLM test data, decoded by tests/golden/make_golden.py"}
    for name, prompt, pin in (
        ("v4_audit_canonical.bin", "frozen fixture prompt",
         "2fd03cda21b6185ab455afd37f1d32d2aa773fb901b1ea5bd2ef9598cfa012ae"),
        ("v4_audit_fullbridge.bin", "canonical frozen fixture", None),
    ):
        blob = open(os.path.join(fx, name), "rb").read()
        file_sha = hashlib.sha256(blob).hexdigest()
        if pin is not None and file_sha != pin:
            raise SystemExit(f"{name}: file checksum {file_sha} != cross_version.rs pin {pin}")
        rec = read_v4_audit_prefix(blob)
        r = Bincode(zstd_decompress(blob[4:]))
        full = read_v4_audit_prefix(blob)
        r.o = _prefix_len(blob)
        read_v4_audit_rest(r, full)
        for k in ("shell_opening", "manifest", "prompt_field", "n_prompt_tokens", "output_text",
                  "prefix_embedding_rows", "prefix_embedding_proofs", "prefix_retained", "prefix_shell_openings",
                  "kv_entries", "kv_proofs", "witnessed_scores"):
            rec[k] = full[k]
        rec["bincode_hex"] = r.b.hex()
        rec["file_sha256"] = file_sha
        rec["prompt"] = prompt          # gen_fixtures.rs:313, 389
        rec["sampling_seed"] = "07" * 32  # gen_fixtures.rs:314, 390
        pins[name] = rec
    # golden_conformance.rs:206-261: same toy model and input as the canonical
    # fixture (gen_fixtures.rs:303-308), different prompt.
    pins["golden_e2e_verify"] = {
        "retained_from": "v4_audit_canonical.bin",
        "prompt": "golden test",
        "token_ids": [42],
        "n_prompt_tokens": 1,
        "merkle_root": "de54562ec98e6ec3dc1cb484758553713dc93caffee16d167cd2064dd512a880",
        "io_root": "62240adf4325d2c15b3d81be456351851d4796d6ba202fd7e24fc4c5729cf5f7",
    }
    pins["golden_manifest"] = golden_manifest(ref_root)
    with open(os.path.join(HERE, "reference_pins.json"), "w") as f:
        json.dump(pins, f, indent=1, sort_keys=True)
    print("wrote", os.path.join(HERE, "reference_pins.json"))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <path of the reference checkout>")
    main(sys.argv[1])
