"""Manifest hashes and the VV4A receipt codec against the reference's own pins (CPU).

Pins (tests/golden/reference_pins.json, made by tests/golden/make_golden.py):
* golden_conformance.rs:132-201: hash_manifest and hash_model_spec of the
  golden manifest;
* the frozen fullbridge receipt (crates/verilm-verify/tests/fixtures): the
  five manifest/spec hashes of its commitment against the manifest it carries;
* both frozen receipts: their decompressed bincode, decoded and re-encoded
  byte for byte by commitllm_b200.receipt.
"""
import json
import os

import numpy as np
import pytest

from commitllm_b200 import manifest as M
from commitllm_b200 import receipt as R
from oracle import commit_oracle as O

PINS = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_pins.json")))
SPEC_KEYS = ("manifest_hash", "input_spec_hash", "model_spec_hash", "decode_spec_hash", "output_spec_hash")


def _oracle_manifest(d):
    """The pins' JSON manifest (hashes as hex) as the oracle's dict (hashes as bytes)."""
    return {k: (bytes.fromhex(v) if v is not None and M.KIND[k].endswith("b32") else v) for k, v in d.items()}


def _server_dict(d):
    """The dict a server passes: absent optional values left out."""
    return {k: v for k, v in d.items() if v is not None}


def test_oracle_manifest_hash_golden_pins():
    g = PINS["golden_manifest"]
    m = _oracle_manifest(g["manifest"])
    assert O.hash_manifest(m).hex() == g["manifest_hash"]
    assert O.hash_model_spec(m).hex() == g["model_spec_hash"]


def test_manifest_hashes_golden_pins():
    g = PINS["golden_manifest"]
    h = M.spec_hashes(M.from_dict(_server_dict(g["manifest"])))
    assert h["manifest_hash"].hex() == g["manifest_hash"]
    assert h["model_spec_hash"].hex() == g["model_spec_hash"]


def test_manifest_hashes_of_the_frozen_fullbridge_receipt():
    r = PINS["v4_audit_fullbridge.bin"]
    c = r["commitment"]
    h = M.spec_hashes(M.from_dict(_server_dict(r["manifest"])))
    m = _oracle_manifest(r["manifest"])
    want = {"manifest_hash": O.hash_manifest(m), "input_spec_hash": O.hash_input_spec(m),
            "model_spec_hash": O.hash_model_spec(m), "decode_spec_hash": O.hash_decode_spec(m),
            "output_spec_hash": O.hash_output_spec(m)}
    for k in SPEC_KEYS:
        assert h[k].hex() == c[k] == want[k].hex(), k


def _full_manifest(**over):
    d = {"tokenizer_hash": "ab" * 32, "temperature": 0.8, "top_k": 40, "top_p": 0.95, "eos_policy": "sample",
         "weight_hash": "01" * 32, "quant_hash": "02" * 32, "system_prompt_hash": "03" * 32,
         "repetition_penalty": 1.1, "frequency_penalty": 0.2, "presence_penalty": 0.3,
         "logit_bias": [[50, -1.5], [7, 2.0], [50, 0.5]], "bad_word_ids": [9, 3, 9, 1], "guided_decoding": "json",
         "stop_sequences": ["\n\n", "END"], "max_tokens": 512, "chat_template_hash": "04" * 32,
         "rope_config_hash": "05" * 32, "rmsnorm_eps": 1e-6, "sampler_version": "chacha20-vi-sample-v1",
         "decode_mode": "sampled", "bos_eos_policy": "add_bos", "truncation_policy": "left",
         "special_token_policy": "encode", "padding_policy": "none", "adapter_hash": "06" * 32, "n_layers": 80,
         "hidden_dim": 8192, "vocab_size": 128256, "embedding_merkle_root": "07" * 32, "quant_family": "W8A8",
         "scale_derivation": "absmax", "quant_block_size": 32, "attn_backend": "sdpa", "attn_dtype": "bfloat16",
         "kv_dim": 1024, "ffn_dim": 28672, "d_head": 128, "n_q_heads": 64, "n_kv_heads": 8, "rope_theta": 500000.0,
         "min_tokens": 2, "ignore_eos": True, "detokenization_policy": "strip_special", "eos_token_id": 128009,
         "attn_mode": "stock"}
    d.update(over)
    return d


def test_every_manifest_field_matches_the_oracle():
    d = _full_manifest()
    m = M.from_dict(d)
    assert m["logit_bias"] == [(7, 2.0), (50, -1.5), (50, 0.5)]       # stable sort by token id
    assert m["bad_word_ids"] == [1, 3, 9]                             # sorted, deduplicated
    om = dict(m)
    h = M.spec_hashes(m)
    assert h["input_spec_hash"] == O.hash_input_spec(om)
    assert h["model_spec_hash"] == O.hash_model_spec(om)
    assert h["decode_spec_hash"] == O.hash_decode_spec(om)
    assert h["output_spec_hash"] == O.hash_output_spec(om)
    assert h["manifest_hash"] == O.hash_manifest(om)


@pytest.mark.parametrize("field", [k for k, _ in M.FIELDS if k != "attn_backend" and k != "attn_dtype"])
def test_each_hashed_field_changes_its_spec_hash(field):
    """Sensitivity (merkle.rs spec-hash tests): every hashed field moves the manifest hash."""
    base = M.from_dict(_full_manifest())
    kind = M.KIND[field]
    m = dict(base)
    v = m[field]
    if kind.endswith("b32"):
        m[field] = None if (v is not None and kind.startswith("opt_")) else bytes(32)
    elif kind.endswith("str") and kind != "vec_str":
        m[field] = None if kind.startswith("opt_") else v + "x"
    elif kind.endswith("u32") and kind != "vec_u32":
        m[field] = None if kind.startswith("opt_") else v + 1
    elif kind.endswith("f32") or kind.endswith("f64"):
        m[field] = None if kind.startswith("opt_") else v + 0.5
    elif kind == "bool":
        m[field] = not v
    else:
        m[field] = list(v)[:-1]
    assert M.spec_hashes(m)["manifest_hash"] != M.spec_hashes(base)["manifest_hash"]


def test_attention_runtime_fields_are_not_hashed():
    """hash_model_spec (merkle.rs:338-367) carries but does not hash attn_backend / attn_dtype."""
    a = M.spec_hashes(M.from_dict(_full_manifest()))
    b = M.spec_hashes(M.from_dict(_full_manifest(attn_backend="eager", attn_dtype="float16")))
    assert a == b


def test_manifest_errors_mirror_the_boundary():
    with pytest.raises(ValueError, match="missing tokenizer_hash"):
        M.from_dict({"temperature": 0.0})
    with pytest.raises(ValueError, match="must be 32 bytes"):
        M.from_dict({"tokenizer_hash": "ab"})
    with pytest.raises(ValueError, match="invalid tokenizer_hash hex"):
        M.from_dict({"tokenizer_hash": "zz" * 32})
    with pytest.raises(TypeError):
        M.from_dict({"tokenizer_hash": "00" * 32, "top_k": 1.5})
    with pytest.raises(TypeError):
        M.from_dict({"tokenizer_hash": "00" * 32, "weight_hash": None})   # not filtered for None (lib.rs:211-217)
    m = M.from_dict({"tokenizer_hash": "00" * 32, "chat_template_hash": None, "min_tokens": None})
    assert m["chat_template_hash"] is None and m["min_tokens"] == 0      # these read None as absent
    assert m["top_p"] == 1.0 and m["eos_policy"] == "stop" and m["repetition_penalty"] == 1.0


@pytest.mark.parametrize("name", ["v4_audit_canonical.bin", "v4_audit_fullbridge.bin"])
def test_receipt_bincode_round_trips_the_frozen_fixtures(name):
    raw = bytes.fromhex(PINS[name]["bincode_hex"])
    resp = R.bincode_decode(R.V4_AUDIT_RESPONSE, raw)
    assert R.bincode_encode(R.V4_AUDIT_RESPONSE, resp) == raw
    r = PINS[name]
    c = resp["commitment"]
    assert c["merkle_root"].hex() == r["commitment"]["merkle_root"]
    assert c["io_root"].hex() == r["commitment"]["io_root"]
    assert c["version"] == "V4"
    assert resp["token_id"] == r["token_id"] and resp["prev_io_hash"].hex() == r["prev_io_hash"]
    assert [l["a"].hex() for l in resp["retained"]["layers"]] == [l["a"] for l in r["retained_layers"]]
    if name == "v4_audit_fullbridge.bin":
        assert resp["shell_opening"] is not None and resp["manifest"] is not None
        h = M.spec_hashes(resp["manifest"])
        for k in SPEC_KEYS:
            assert h[k] == c[k], k


def test_vv4a_framing_round_trip():
    raw = bytes.fromhex(PINS["v4_audit_fullbridge.bin"]["bincode_hex"])
    resp = R.bincode_decode(R.V4_AUDIT_RESPONSE, raw)
    blob = R.serialize_v4_audit(resp)
    assert blob[:4] == b"VV4A"
    assert R.zstd_decompress(blob[4:]) == raw
    back = R.deserialize_v4_audit(blob)
    assert R.bincode_encode(R.V4_AUDIT_RESPONSE, back) == raw
    with pytest.raises(ValueError, match="magic"):
        R.deserialize_v4_audit(b"VKEY" + blob[4:])
    with pytest.raises(ValueError):
        R.bincode_decode(R.V4_AUDIT_RESPONSE, raw[:-3])
    with pytest.raises(ValueError, match="trailing"):
        R.bincode_decode(R.V4_AUDIT_RESPONSE, raw + b"\0")


def test_receipt_json_shapes():
    raw = bytes.fromhex(PINS["v4_audit_fullbridge.bin"]["bincode_hex"])
    resp = R.bincode_decode(R.V4_AUDIT_RESPONSE, raw)
    resp["kv_entries"] = [[{"k_roped": np.array([1.5, -0.0]), "v_deq": np.array([2.0, np.inf])}]]
    d = json.loads(R.v4_audit_json(resp))
    assert d["commitment"]["version"] == "V4"
    assert len(d["commitment"]["merkle_root"]) == 32 and all(0 <= x < 256 for x in d["commitment"]["merkle_root"])
    assert d["kv_entries"][0][0]["k_roped"] == [np.float64(1.5).tobytes().hex(), np.float64(-0.0).tobytes().hex()]
    assert d["kv_entries"][0][0]["v_deq"][1] == np.float64(np.inf).tobytes().hex()
    assert all(-128 <= x < 128 for x in d["retained"]["layers"][0]["a"])
    assert d["manifest"]["tokenizer_hash"] == [0] * 32
