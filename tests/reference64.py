"""float64 restatement of the attention math (independent of the C oracle).

Used to self-check the oracle and to build shard records in the host tests.
"""
from __future__ import annotations

import numpy as np


def decode64(q, k, v, n_heads, n_kv_heads, head_dim, n_pos, kv_stride=None, scale=None):
    if kv_stride is None:
        kv_stride = n_kv_heads * head_dim
    if scale is None:
        scale = 1.0 / np.sqrt(head_dim)
    q = np.asarray(q, dtype=np.float64).reshape(n_heads, head_dim)
    k = np.asarray(k, dtype=np.float64).reshape(-1, kv_stride)[:n_pos, : n_kv_heads * head_dim]
    v = np.asarray(v, dtype=np.float64).reshape(-1, kv_stride)[:n_pos, : n_kv_heads * head_dim]
    k = k.reshape(n_pos, n_kv_heads, head_dim)
    v = v.reshape(n_pos, n_kv_heads, head_dim)
    kv_mul = n_heads // n_kv_heads
    out = np.zeros((n_heads, head_dim))
    for h in range(n_heads):
        g = h // kv_mul
        s = k[:, g, :] @ q[h] * scale
        p = np.exp(s - s.max())
        out[h] = (p / p.sum()) @ v[:, g, :]
    return out.reshape(-1)


def records64(q, k, v, n_heads, n_kv_heads, head_dim, rows, scale=None):
    """Shard record set [n_heads][head_dim+2] = (o/l, m, l) over the given rows."""
    if scale is None:
        scale = 1.0 / np.sqrt(head_dim)
    kv = n_kv_heads * head_dim
    q = np.asarray(q, dtype=np.float64).reshape(n_heads, head_dim)
    K = np.asarray(k, dtype=np.float64).reshape(-1, kv)[rows].reshape(-1, n_kv_heads, head_dim)
    V = np.asarray(v, dtype=np.float64).reshape(-1, kv)[rows].reshape(-1, n_kv_heads, head_dim)
    kv_mul = n_heads // n_kv_heads
    rec = np.zeros((n_heads, head_dim + 2))
    if K.shape[0] == 0:
        rec[:, head_dim] = -np.inf
        return rec
    for h in range(n_heads):
        g = h // kv_mul
        s = K[:, g, :] @ q[h] * scale
        m = s.max()
        p = np.exp(s - m)
        l = p.sum()
        rec[h, :head_dim] = (p @ V[:, g, :]) / l
        rec[h, head_dim] = m
        rec[h, head_dim + 1] = l
    return rec


def lse_combine64(recs, head_dim):
    """Merges record sets [S][n_heads][head_dim+2] (same rule as gla_lse_combine)."""
    recs = np.asarray(recs, dtype=np.float64)
    m = recs[:, :, head_dim]
    l = recs[:, :, head_dim + 1]
    live = l > 0
    M = np.where(live, m, -np.inf).max(axis=0)
    w = np.where(live, l * np.exp(np.where(live, m, 0) - M[None, :]), 0.0)
    o = (w[:, :, None] * recs[:, :, :head_dim]).sum(axis=0) / w.sum(axis=0)[:, None]
    return o.reshape(-1)
