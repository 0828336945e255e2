"""ctypes wrapper of the oracle's C restatement (``oracle/_build/libvco.so``).

Test infrastructure only.  Descriptors are the ``vc_kv_desc`` /
``vc_trace_desc`` structs of include/vcommit.h, with HOST pointers.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import build_oracle

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = build_oracle.LIB
        if not os.path.exists(path):
            path = build_oracle.build()
        l = ctypes.CDLL(path)
        P = ctypes.c_void_p
        l.vco_kv_commit.restype = ctypes.c_int
        l.vco_kv_commit.argtypes = [P, P, P, P, ctypes.c_int]
        l.vco_kv_leaf.restype = None
        l.vco_kv_leaf.argtypes = [P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int64, P]
        l.vco_build_tree.restype = None
        l.vco_build_tree.argtypes = [P, ctypes.c_int64, P]
        l.vco_compute_root.restype = None
        l.vco_compute_root.argtypes = [P, ctypes.c_int64, P]
        l.vco_trace_leaves.restype = ctypes.c_int
        l.vco_trace_leaves.argtypes = [P, P, ctypes.c_int]
        l.vco_io_chain.restype = None
        l.vco_io_chain.argtypes = [P, P, ctypes.c_int64, P, ctypes.c_int64, P]
        l.vco_sha_probe.restype = None
        l.vco_sha_probe.argtypes = [P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int]
        l.vco_kv_transcript.restype = None
        l.vco_kv_transcript.argtypes = [ctypes.c_int32] * 5 + [P] * 8
        _lib = l
    return _lib


def _ptr(a: np.ndarray) -> ctypes.c_void_p:
    return ctypes.c_void_p(a.ctypes.data)


def build_tree(leaves: np.ndarray) -> np.ndarray:
    """merkle::build_tree nodes ``[2*pad-1, 32]`` of ``leaves [n, 32]`` uint8."""
    leaves = np.ascontiguousarray(leaves, dtype=np.uint8)
    n = leaves.shape[0]
    pad = 1 << (n - 1).bit_length() if n > 1 else 1
    nodes = np.zeros((2 * pad - 1, 32), np.uint8)
    lib().vco_build_tree(_ptr(leaves), n, _ptr(nodes))
    return nodes


def compute_root(leaves: np.ndarray) -> bytes:
    leaves = np.ascontiguousarray(leaves, dtype=np.uint8)
    out = np.zeros(32, np.uint8)
    lib().vco_compute_root(_ptr(leaves), leaves.shape[0], _ptr(out))
    return out.tobytes()


def io_chain(leaves: np.ndarray, token_ids, prompt: bytes) -> np.ndarray:
    leaves = np.ascontiguousarray(leaves, dtype=np.uint8)
    tok = np.ascontiguousarray(np.asarray(token_ids, dtype=np.uint32))
    pr = np.frombuffer(prompt, dtype=np.uint8) if prompt else np.zeros(1, np.uint8)
    out = np.zeros_like(leaves)
    lib().vco_io_chain(_ptr(leaves), _ptr(tok), leaves.shape[0], _ptr(pr), len(prompt), _ptr(out))
    return out


def kv_transcript(x: np.ndarray, wk, wv, scale_x: np.ndarray, n_heads: int, head_dim: int, sw=None,
                  inv_freq=None):
    """compute_kv_transcript in C, one thread (per-tensor scales ``sw`` [n_layers][2] or the toy path).
    x: int8 [n_tok][n_layers][hidden]; returns (k, v) f64 [n_layers][n_tok][kv]."""
    x = np.ascontiguousarray(x, np.int8)
    n_tok, n_layers, hidden = x.shape
    kv = n_heads * head_dim
    wk = [np.ascontiguousarray(w, np.int8) for w in wk]
    wv = [np.ascontiguousarray(w, np.int8) for w in wv]
    pk = (ctypes.c_void_p * n_layers)(*[w.ctypes.data for w in wk])
    pv = (ctypes.c_void_p * n_layers)(*[w.ctypes.data for w in wv])
    sx = np.ascontiguousarray(scale_x, np.float32)
    swa = None if sw is None else np.ascontiguousarray(sw, np.float32)
    inv = np.ascontiguousarray(inv_freq if inv_freq is not None else np.zeros(max(1, head_dim // 2)), np.float64)
    k = np.empty((n_layers, n_tok, kv), np.float64)
    v = np.empty((n_layers, n_tok, kv), np.float64)
    lib().vco_kv_transcript(n_tok, n_layers, hidden, n_heads, head_dim, _ptr(x), pk, pv, _ptr(sx),
                            None if swa is None else _ptr(swa), _ptr(inv), _ptr(k), _ptr(v))
    return k, v
