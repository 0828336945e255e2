"""The oracle's two restatements of compute_kv_transcript agree, and agree with
a plain scalar loop written straight from crates/verilm-prover/src/lib.rs:207-329
and crates/verilm-core/src/rope.rs (no GPU)."""
import math

import numpy as np
import pytest

from oracle import commit_oracle as O
from oracle import vco


def scalar_reference(x, wk, wv, sx, nh, hd, sw, inv):
    """One position and layer at a time, one f64 operation per Python expression."""
    n_tok, L, H = x.shape
    kv = nh * hd
    k = np.empty((L, n_tok, kv))
    v = np.empty((L, n_tok, kv))
    for t in range(n_tok):
        for l in range(L):
            xr = [int(c) for c in x[t, l]]
            acc_k = [sum(int(a) * b for a, b in zip(wk[l][r], xr)) for r in range(kv)]
            acc_v = [sum(int(a) * b for a, b in zip(wv[l][r], xr)) for r in range(kv)]
            sk = float(np.float32(sw[l][0])) * float(sx[t, l])
            sv = float(np.float32(sw[l][1])) * float(sx[t, l])
            kf = [a * sk for a in acc_k]
            v[l, t] = [a * sv for a in acc_v]
            for h in range(nh):
                for i in range(hd // 2):
                    ang = float(t) * inv[i]
                    c, s = math.cos(ang), math.sin(ang)
                    lo, hi = kf[h * hd + i], kf[h * hd + hd // 2 + i]
                    k[l, t, h * hd + i] = lo * c - hi * s
                    k[l, t, h * hd + hd // 2 + i] = hi * c + lo * s
    return k, v


@pytest.mark.parametrize("scaling", [None, O.RopeScaling(), O.RopeScaling(rope_type="linear", factor=2.0)])
def test_transcript_restatements_agree(scaling):
    rng = np.random.default_rng(5)
    n_tok, L, H, nh, hd = 6, 2, 40, 2, 16
    x = rng.integers(-128, 128, (n_tok, L, H), dtype=np.int8)
    wk = [rng.integers(-128, 128, (nh * hd, H), dtype=np.int8) for _ in range(L)]
    wv = [rng.integers(-128, 128, (nh * hd, H), dtype=np.int8) for _ in range(L)]
    sx = rng.random((n_tok, L), dtype=np.float32)
    sw = [(np.float32(0.0123), np.float32(0.0071)), (np.float32(0.002), np.float32(0.3))]
    inv = O.scaled_inv_freq(hd, 500000.0, scaling)
    k_np, v_np = O.compute_kv_transcript(x, wk, wv, sx, nh, hd, per_tensor=sw, rope_theta=500000.0,
                                         rope_scaling=scaling)
    k_c, v_c = vco.kv_transcript(x, wk, wv, sx, nh, hd, sw=np.array(sw, np.float32), inv_freq=np.array(inv))
    k_s, v_s = scalar_reference(x, wk, wv, sx, nh, hd, sw, inv)
    for a, b in ((k_np, k_c), (k_np, k_s), (v_np, v_c), (v_np, v_s)):
        assert np.array_equal(a.view(np.uint64), b.view(np.uint64))


def test_transcript_toy_path_clamps():
    rng = np.random.default_rng(6)
    x = rng.integers(-128, 128, (3, 2, 16), dtype=np.int8)
    wk = [rng.integers(-128, 128, (4, 16), dtype=np.int8) for _ in range(2)]
    wv = [rng.integers(-128, 128, (4, 16), dtype=np.int8) for _ in range(2)]
    k, v = O.compute_kv_transcript(x, wk, wv, np.ones((3, 2), np.float32), 2, 2)
    k_c, v_c = vco.kv_transcript(x, wk, wv, np.ones((3, 2), np.float32), 2, 2)
    assert np.array_equal(k, k_c) and np.array_equal(v, v_c)
    assert k.min() >= -128 and k.max() <= 127
    acc = x[:, 0].astype(np.int64) @ wk[0].T.astype(np.int64)
    assert np.array_equal(k[0], np.clip(acc, -128, 127).astype(np.float64))


def test_scaled_inv_freq_llama3_bands():
    """constants.rs:253-297: high frequencies unchanged, low ones divided by the factor."""
    base = O.scaled_inv_freq(128, 500000.0, None)
    sc = O.scaled_inv_freq(128, 500000.0, O.RopeScaling())
    assert sc[0] == base[0]
    assert sc[-1] == base[-1] / 8.0
    assert any(base[i] / 8.0 < sc[i] < base[i] for i in range(64))
