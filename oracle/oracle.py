"""ctypes loader for the CPU oracle (oracle/attention_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()``
and by the ``cpu_baseline`` / ``--impl reference`` legs of bench.py, always as
the checker or the timed CPU baseline, never as the product path.

PARITY UNPINNED: the reference (GPULlama3.java) has no attention tests or
golden vectors and its Java cannot run in this environment; the C file
restates ``InferenceCore.java:105-144`` and ``FloatTensor.java:86-227``
statement by statement.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u16p = ctypes.POINTER(ctypes.c_uint16)


def build(force: bool = False) -> str:
    """Compiles liboracle.so with the committed Makefile (gcc)."""
    if force or not os.path.exists(_LIB_PATH):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.oracle_decode_f32.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.oracle_decode_f32_div.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_float, ctypes.c_int]
        L.oracle_decode_f16.argtypes = [_f32p, _u16p, _u16p, _f32p, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.oracle_prefill_causal_f32.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_int,
                                                ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                ctypes.c_int]
        L.oracle_rope_freqs.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_double, ctypes.c_int,
                                        ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                        ctypes.c_float, _f32p, _f32p]
        L.oracle_rope_interleaved.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_int, ctypes.c_int, _f32p, _f32p]
        L.oracle_rope_neox.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_int, _f32p, _f32p]
        L.oracle_half_to_float.argtypes = [_u16p, _f32p, ctypes.c_int64]
        L.oracle_wo_residual_f16.argtypes = [_f32p, _f32p, _u16p, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_int]
        _i8p = ctypes.POINTER(ctypes.c_int8)
        L.oracle_float_to_half.argtypes = [_f32p, _u16p, ctypes.c_int64]
        L.oracle_quantize_q8.argtypes = [_f32p, _f32p, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_int, _i8p, _i8p, ctypes.c_int64, _u16p]
        L.oracle_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a: np.ndarray, t=_f32p):
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data_as(t)


def max_threads() -> int:
    return int(lib().oracle_max_threads())


def decode_f32(q, k, v, n_heads, n_kv_heads, head_dim, n_pos, kv_stride=None, n_threads=0,
               divisor=None):
    """Decode attention of one token over rows 0..n_pos-1 (InferenceCore.java:105-144).

    q [n_heads*head_dim] f32; k, v [>= n_pos][kv_stride] f32. Returns xb f32.
    """
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    if kv_stride is None:
        kv_stride = n_kv_heads * head_dim
    assert n_pos >= 1 and k.size >= (n_pos - 1) * kv_stride + n_kv_heads * head_dim
    xb = np.zeros(n_heads * head_dim, dtype=np.float32)
    kv_mul = n_heads // n_kv_heads
    if divisor is None:
        lib().oracle_decode_f32(_p(q), _p(k), _p(v), _p(xb), n_heads, head_dim, kv_stride, kv_mul,
                                n_pos - 1, n_threads)
    else:
        lib().oracle_decode_f32_div(_p(q), _p(k), _p(v), _p(xb), n_heads, head_dim, kv_stride,
                                    kv_mul, n_pos - 1, float(divisor), n_threads)
    return xb


def decode_f16(q, k16, v16, n_heads, n_kv_heads, head_dim, n_pos, kv_stride=None, n_threads=0):
    """FP32 reference semantics applied to the decoded FP16 cache (uint16 bit patterns)."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k16 = np.ascontiguousarray(k16).view(np.uint16)
    v16 = np.ascontiguousarray(v16).view(np.uint16)
    if kv_stride is None:
        kv_stride = n_kv_heads * head_dim
    xb = np.zeros(n_heads * head_dim, dtype=np.float32)
    lib().oracle_decode_f16(_p(q), _p(k16, _u16p), _p(v16, _u16p), _p(xb), n_heads, head_dim,
                            kv_stride, n_heads // n_kv_heads, n_pos - 1, n_threads)
    return xb


def prefill_causal_f32(q, k, v, L, n_heads, n_kv_heads, head_dim, n_threads=0):
    """Causal attention as the reference ingests a prompt: decode at p = 0..L-1."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    out = np.zeros((L, n_heads * head_dim), dtype=np.float32)
    lib().oracle_prefill_causal_f32(_p(q), _p(k), _p(v), _p(out), L, n_heads, n_kv_heads,
                                    head_dim, n_threads)
    return out


def rope_freqs(context_length, head_dim, theta, scaling=None):
    """RoPE.precomputeFreqsCis -> (cr, ci), each [context_length*head_dim/2] f32."""
    n = context_length * (head_dim // 2)
    cr = np.zeros(n, dtype=np.float32)
    ci = np.zeros(n, dtype=np.float32)
    if scaling is None:
        lib().oracle_rope_freqs(context_length, head_dim, float(theta), 0, 1.0, 1.0, 1.0, 1.0,
                                _p(cr), _p(ci))
    else:
        sf, lo, hi, old = scaling
        lib().oracle_rope_freqs(context_length, head_dim, float(theta), 1, sf, lo, hi, old,
                                _p(cr), _p(ci))
    return cr, ci


def rope_interleaved(q, k, head_dim, position, cr, ci):
    """In-place Llama rotation of q [dim] and k [kv_dim] (InferenceCore.java:82-94)."""
    lib().oracle_rope_interleaved(_p(q), _p(k), q.size, k.size, head_dim, position, _p(cr), _p(ci))


def rope_neox(q, k, n_heads, n_kv_heads, head_dim, position, cr, ci):
    """In-place NeoX rotation (InferenceCore.java:210-225)."""
    lib().oracle_rope_neox(_p(q), _p(k), n_heads, n_kv_heads, head_dim, position, _p(cr), _p(ci))


def half_to_float(h):
    h = np.ascontiguousarray(h).view(np.uint16)
    out = np.zeros(h.shape, dtype=np.float32)
    lib().oracle_half_to_float(_p(h, _u16p), _p(out), h.size)
    return out


def wo_residual_f16(x, hb, w16, n, d, local_size=32):
    """x_res[i] += w[i]·xb as the GPU task matrixVectorGenericWithResidual does
    it (TransformerComputeKernelsLayered.java:715-733): returns the new hb."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.array(hb, dtype=np.float32, copy=True)
    w16 = np.ascontiguousarray(w16).view(np.uint16)
    lib().oracle_wo_residual_f16(_p(x), _p(out), _p(w16, _u16p), n, d, local_size)
    return out


def float_to_half(x):
    """IEEE float32 -> float16 bits, round to nearest even."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.shape, dtype=np.uint16)
    lib().oracle_float_to_half(_p(x), _p(out, _u16p), x.size)
    return out


def quantize_q8(k, v, n_kv, hd):
    """Q8 KV cache rows of FP32 k/v [rows][n_kv*hd] (GGML Q8_0 quantiser):
    returns (kq int8, vq int8, scales uint16 [rows][n_kv][8])."""
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    rows = k.shape[0]
    kq = np.zeros((rows, n_kv * hd), dtype=np.int8)
    vq = np.zeros_like(kq)
    sc = np.zeros((rows, n_kv, 8), dtype=np.uint16)
    i8 = ctypes.POINTER(ctypes.c_int8)
    lib().oracle_quantize_q8(_p(k), _p(v), n_kv * hd, rows, n_kv, hd, _p(kq, i8), _p(vq, i8),
                             n_kv * hd, _p(sc, _u16p))
    return kq, vq, sc


def dequantize_q8(kq, vq, sc, n_kv, hd):
    """FP32 values q * scale of a Q8 cache (exact in FP32)."""
    rows = kq.shape[0]
    nb = hd // 32
    s = half_to_float(sc).reshape(rows, n_kv, 8)
    ks = np.repeat(s[:, :, :nb], 32, axis=2).reshape(rows, n_kv * hd)
    vs = np.repeat(s[:, :, 4:4 + nb], 32, axis=2).reshape(rows, n_kv * hd)
    return (kq.astype(np.float32) * ks).astype(np.float32), \
        (vq.astype(np.float32) * vs).astype(np.float32)
