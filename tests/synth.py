"""Seeded synthetic inputs shared by the tests, the fixtures and the bench.

Every generator is numpy PCG64 (``default_rng(seed)``), which gives the same
bytes on every platform.  Values follow the benchmark shapes: K/V ~ N(0, 1)
rounded to bf16, activations ~ U[-128, 127], logits ~ N(0, 3^2).
"""
from __future__ import annotations

import numpy as np


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def kv_rows_bf16(seed: int, n_layers: int, n_rows: int, n_heads: int, head_dim: int):
    """K and V of every layer as bf16 bits, ``[n_layers, n_rows, n_heads, head_dim]``."""
    rng = np.random.default_rng(seed)
    k = f32_to_bf16_bits(rng.standard_normal((n_layers, n_rows, n_heads, head_dim), dtype=np.float32))
    v = f32_to_bf16_bits(rng.standard_normal((n_layers, n_rows, n_heads, head_dim), dtype=np.float32))
    return k, v


def token_ids(seed: int, n: int, vocab: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, vocab, size=n, dtype=np.uint32)


def activations_i8(seed: int, shape) -> np.ndarray:
    return np.random.default_rng(seed).integers(-128, 128, size=shape, dtype=np.int16).astype(np.int8)


def scales_f32(seed: int, n: int) -> np.ndarray:
    return (np.random.default_rng(seed).random(n, dtype=np.float32) * 0.05 + 1e-3).astype(np.float32)


def logits_f32(seed: int, shape) -> np.ndarray:
    return (np.random.default_rng(seed).standard_normal(shape, dtype=np.float32) * 3.0).astype(np.float32)


def positions(seed: int, n: int, k: int) -> np.ndarray:
    return np.sort(np.random.default_rng(seed).choice(n, size=k, replace=False))
