"""Seeded synthetic inputs shared by tests, fixtures and the bench.

Values are ~N(0,1) FP32 from numpy's PCG64 generator: ``standard_normal``
with the given seed, drawn in the order q, K, V (the reference workloads are
model shapes, not datasets; these tensors stand in for them).
"""
from __future__ import annotations

import numpy as np


def normal(seed: int, *shape, dtype=np.float32):
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.standard_normal(shape, dtype=np.float32).astype(dtype, copy=False)


def decode_case(seed, n_heads, n_kv_heads, head_dim, n_rows, kv_stride=None):
    """q [n_heads*hd], K/V [n_rows][kv_stride] (padding columns stay random)."""
    if kv_stride is None:
        kv_stride = n_kv_heads * head_dim
    rng = np.random.Generator(np.random.PCG64(seed))
    q = rng.standard_normal(n_heads * head_dim, dtype=np.float32)
    k = rng.standard_normal((n_rows, kv_stride), dtype=np.float32)
    v = rng.standard_normal((n_rows, kv_stride), dtype=np.float32)
    return q, k, v


def to_f16_bits(x: np.ndarray) -> np.ndarray:
    """Round to binary16 (round-to-nearest-even) and return the uint16 bit patterns."""
    return np.ascontiguousarray(x.astype(np.float16)).view(np.uint16)
