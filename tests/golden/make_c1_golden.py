"""Freeze the oracle's outputs for the CPU-runnable reference case (C1).

    python tests/golden/make_c1_golden.py

C1: a tiny Llama-shaped transcript -- 2 layers, 4 KV heads, head_dim 64, one
sequence of 128 tokens, K/V bf16 ~ N(0, 1); 128 token ids ~ U[0, 32000);
Merkle openings of 8 random positions in every layer.  The IO chain runs over
retained-state leaves of a synthetic retained state (2 layers, a_i8 rows of
512 bytes, f32 scale_a), the encoding of merkle.rs:144-161.

The inputs are regenerated from the seeds in ``tests/synth.py``; only the
expected digests are stored (``c1_golden.json``), computed by the Python
oracle (never by the GPU path).
"""
from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import commit_oracle as O  # noqa: E402
from tests import synth  # noqa: E402

C1 = dict(n_layers=2, n_heads=4, head_dim=64, n_tokens=128, vocab=32000, hidden=512,
          seed_kv=1, seed_tok=2, seed_pos=3, seed_a=4, seed_scale=5, n_open=8,
          prompt="C1 synthetic prompt", sampling_seed="11" * 32, n_prompt_tokens=1)


def c1_inputs(cfg=C1):
    k, v = synth.kv_rows_bf16(cfg["seed_kv"], cfg["n_layers"], cfg["n_tokens"], cfg["n_heads"], cfg["head_dim"])
    tok = synth.token_ids(cfg["seed_tok"], cfg["n_tokens"], cfg["vocab"])
    pos = synth.positions(cfg["seed_pos"], cfg["n_tokens"], cfg["n_open"])
    a = synth.activations_i8(cfg["seed_a"], (cfg["n_tokens"], cfg["n_layers"], cfg["hidden"]))
    sc = synth.scales_f32(cfg["seed_scale"], cfg["n_tokens"] * cfg["n_layers"]).reshape(cfg["n_tokens"], cfg["n_layers"])
    return k, v, tok, pos, a, sc


def main():
    cfg = C1
    k, v, tok, pos, a, sc = c1_inputs(cfg)
    kv = []
    for l in range(cfg["n_layers"]):
        kf = O.bf16_to_f64(k[l].reshape(cfg["n_tokens"], -1))
        vf = O.bf16_to_f64(v[l].reshape(cfg["n_tokens"], -1))
        kv.append((kf, vf))
    retained = [[O.RetainedLayerState(a=a[t, l].tobytes(), scale_a=float(sc[t, l])) for l in range(cfg["n_layers"])]
                for t in range(cfg["n_tokens"])]
    com = O.commit_minimal(retained, [int(x) for x in tok], cfg["prompt"].encode(),
                           bytes.fromhex(cfg["sampling_seed"]), kv_transcripts=kv,
                           n_prompt_tokens=cfg["n_prompt_tokens"])
    openings = []
    for l in range(cfg["n_layers"]):
        for p in pos:
            pr = O.prove(com.kv_trees[l], int(p))
            leaf = com.kv_trees[l].nodes[int(p)]
            assert O.verify(com.kv_roots[l], leaf, pr)
            openings.append({"layer": l, "pos": int(p), "leaf": leaf.hex(), "siblings": [s.hex() for s in pr.siblings]})
    out = {
        "config": cfg,
        "kv_roots": [r.hex() for r in com.kv_roots],
        "kv_openings": openings,
        "merkle_root": com.merkle_root.hex(),
        "io_root": com.io_root.hex(),
        "prompt_hash": com.prompt_hash.hex(),
        "seed_commitment": com.seed_commitment.hex(),
        "trace_leaves_head": [x.hex() for x in com.trace_leaves[:4]],
        "io_hashes_head": [x.hex() for x in com.io_hashes[:4]],
        "io_hashes_last": com.io_hashes[-1].hex(),
    }
    with open(os.path.join(HERE, "c1_golden.json"), "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", os.path.join(HERE, "c1_golden.json"))


if __name__ == "__main__":
    main()
