"""Regenerate ``reference_pins.json`` from the reference's own test data.

Run in a container that has the reference checked out (read-only) at
``/root/reference``::

    python tests/golden/make_golden.py [/root/reference]

What it extracts (all read as data, nothing of the reference is executed):

* ``crates/verilm-verify/tests/fixtures/v4_audit_canonical.bin`` and
  ``v4_audit_fullbridge.bin``: frozen ``V4AuditResponse`` receipts written by
  ``tests/gen_fixtures.rs:295-420``.  Wire format ``"VV4A" || zstd(bincode v1)``
  (``crates/verilm-core/src/serialize.rs:43-59``).  Decoded here with the
  system ``libzstd.so.1`` and a bincode-v1 reader for the leading fields of
  ``V4AuditResponse`` (types.rs:1475-1502) and ``BatchCommitment``
  (types.rs:1710-1759).  Their file SHA-256 is pinned by
  ``crates/verilm-verify/tests/cross_version.rs:431-442``.
* The golden hex pins of ``golden_e2e_verify``
  (``crates/verilm-test-vectors/tests/golden_conformance.rs:206-261``): the
  same toy model (seed 12345, input 0..16) as the canonical fixture, prompt
  ``b"golden test"``, token 42.

The prompts and token ids are the inputs written in those two test files.
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import os
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


def read_proof(r: Bincode):
    return {"leaf_index": r.u32(), "siblings": [s.hex() for s in r.vec(r.arr32)]}


def read_v4_audit_prefix(blob: bytes):
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
    return out


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
    with open(os.path.join(HERE, "reference_pins.json"), "w") as f:
        json.dump(pins, f, indent=1, sort_keys=True)
    print("wrote", os.path.join(HERE, "reference_pins.json"))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
