"""ctypes binding of libgpullama_attn (the C ABI in include/gpullama_attn.h).

This is the Python counterpart of the Java 21 FFM binding a GPULlama3.java
maintainer adds: every call goes through the exported C symbols with raw
device pointers.  Tensors may be passed as torch CUDA tensors (their
``data_ptr()`` is used) or as integer device addresses.

There is no fallback: importing this module fails loudly when the shared
library has not been built (``python gpullama3.java_b200/build_lib.py``).
"""
from __future__ import annotations

import ctypes
import math
import os

__all__ = ["GlaError", "Context", "lib", "LIB_PATH", "DTYPE_F32", "DTYPE_F16",
           "ROPE_INTERLEAVED", "ROPE_NEOX", "EXPORTED_SYMBOLS", "debug_partition", "device_view"]

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libgpullama_attn.so")

GLA_OK = 0
DTYPE_F32 = 0
DTYPE_F16 = 1
DTYPE_Q8 = 2
ROPE_INTERLEAVED = 0
ROPE_NEOX = 1
OPT_EARLY_KV_PREFETCH = 1  # values: 0 off, 1 host n_pos, 2 (default) also device positions
OPT_SHARD_EXCHANGE = 2     # 1 (default): peer exchange when available, 0: NCCL all-gather
OPT_COMM_TIMEOUT_MS = 3    # host deadline of every step that waits for other ranks
OPT_TRACE = 4              # 1: decode calls record per-CTA phase stamps (debug_trace)

STATUS_NAMES = {
    0: "GLA_OK", -1: "GLA_ERR_INVALID_ARG", -2: "GLA_ERR_CUDA", -3: "GLA_ERR_NOT_SUPPORTED",
    -4: "GLA_ERR_ALIGNMENT", -5: "GLA_ERR_TIMEOUT", -6: "GLA_ERR_COMM", -7: "GLA_ERR_NO_DEVICE",
    -8: "GLA_ERR_OUT_OF_MEMORY",
}

_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_F = ctypes.c_float

# name -> (restype, argtypes); the list mirrors include/gpullama_attn.h
_SIGS = {
    "gla_version": (_I32, []),
    "gla_status_string": (ctypes.c_char_p, [_I32]),
    "gla_create": (_I32, [_I32, _P, ctypes.POINTER(_P)]),
    "gla_destroy": (_I32, [_P]),
    "gla_set_stream": (_I32, [_P, _P]),
    "gla_last_error": (ctypes.c_char_p, [_P]),
    "gla_device_status": (_I32, [_P, ctypes.POINTER(_I32)]),
    "gla_reserve": (_I32, [_P, _I32, _I32, _I32, _I32]),
    "gla_num_sms": (_I32, [_P]),
    "gla_set_option": (_I32, [_P, _I32, _I32]),
    "gla_kv_cache_alloc": (_I32, [_P, _I32, _I32, _I32, _I32, ctypes.POINTER(_P),
                                  ctypes.POINTER(_P)]),
    "gla_kv_cache_free": (_I32, [_P, _P, _P]),
    "gla_process_heads_flash_attention": (_I32, [_P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _P,
                                                 _I32, _I32]),
    "gla_process_heads_flash_attention_f16kv": (_I32, [_P, _P, _P, _P, _P, _I32, _I32, _I32, _I32,
                                                       _P, _I32, _I32]),
    "gla_decode_f32kv": (_I32, [_P, _P, _P, _P, _P, _I32, _I32, _I32, _I64, _I32, _F]),
    "gla_decode_f16kv": (_I32, [_P, _P, _P, _P, _P, _I32, _I32, _I32, _I64, _I32, _F]),
    "gla_decode_batched_f32kv": (_I32, [_P, _P, _P, _P, _P, _I32, _P, _I32, _I32, _I32, _I32,
                                        _I64, _F]),
    "gla_decode_batched_f16kv": (_I32, [_P, _P, _P, _P, _P, _I32, _P, _I32, _I32, _I32, _I32,
                                        _I64, _F]),
    "gla_decode_partial_f32kv": (_I32, [_P, _P, _P, _P, _P, _I32, _I32, _I32, _I64, _I32, _F]),
    "gla_decode_partial_f16kv": (_I32, [_P, _P, _P, _P, _P, _I32, _I32, _I32, _I64, _I32, _F]),
    "gla_lse_combine": (_I32, [_P, _P, _I32, _I32, _I32, _P]),
    "gla_comm_unique_id_size": (_I32, []),
    "gla_comm_get_unique_id": (_I32, [_P]),
    "gla_comm_init": (_I32, [_P, _I32, _I32, _P]),
    "gla_decode_sharded_f16kv": (_I32, [_P, _P, _P, _P, _P, _I32, _I32, _I32, _I64, _I32, _F]),
    "gla_decode_sharded_f32kv": (_I32, [_P, _P, _P, _P, _P, _I32, _I32, _I32, _I64, _I32, _F]),
    "gla_prefill_causal_f16": (_I32, [_P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _F]),
    "gla_rope_append_f32": (_I32, [_P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _P, _F, _I32]),
    "gla_debug_trace": (_I64, [_P, _P, _I64]),
    "gla_debug_advance_position": (_I32, [_P, _P, _I32, _I32]),
    "gla_debug_xch_loopback": (_I32, [_P, _I32]),
    "gla_debug_partition": (_I64, [_P, _I32, _I32, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P,
                                   _P, _P, _I64]),
    "gla_comm_peer_exchange": (_I32, [_P]),
    "gla_comm_wait": (_I32, [_P]),
    "gla_comm_resync": (_I32, [_P]),
    "gla_rope_append_attention_f32": (_I32, [_P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32,
                                             _P, _I32, _I32, _F, _I32]),
    "gla_decode_f32kv_noalloc": (_I32, [_P, _P, _P, _P, _I32, _I32, _I32, _I64, _I32, _F, _P]),
    "gla_wo_residual_f16": (_I32, [_P, _P, _P, _P, _I32, _I32]),
    "gla_decode_q8kv": (_I32, [_P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I64, _I32, _F]),
    "gla_kv_quantize_q8": (_I32, [_P, _P, _P, _I64, _I32, _I32, _I32, _P, _P, _I64, _P]),
    "gla_kv_cache_alloc_q8": (_I32, [_P, _I32, _I32, _I32, _I32, _P, _P, _P]),
    "gla_kv_cache_free_q8": (_I32, [_P, _P, _P, _P]),
    "gla_rope_append_q8": (_I32, [_P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _P, _I32, _F,
                                  _I32]),
    "gla_ingest_prompt_f32": (_I32, [_P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32,
                                     _I32, _F, _I32]),
    "gla_ingest_prompt_f16kv": (_I32, [_P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32,
                                       _I32, _F, _I32]),
}

EXPORTED_SYMBOLS = tuple(_SIGS)

_lib = None


def lib():
    """Loads the shared library (raises ImportError when it is missing)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with python gpullama3.java_b200/build_lib.py")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


class GlaError(RuntimeError):
    """A libgpullama_attn call returned a negative status."""

    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")


def _ptr(x) -> int | None:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    dp = getattr(x, "data_ptr", None)
    if dp is not None:
        return int(dp())
    raise TypeError(f"expected a device tensor or an address, got {type(x)!r}")


def device_view(address: int, shape, dtype):
    """A torch CUDA tensor viewing `address` (device memory the library
    allocated, e.g. a KV cache from gla_kv_cache_alloc) without copying; it
    must not outlive the allocation."""
    import torch

    typestr = {torch.float32: "<f4", torch.float16: "<f2", torch.int8: "|i1",
               torch.int16: "<i2", torch.int32: "<i4", torch.uint8: "|u1"}[dtype]

    class _View:
        __cuda_array_interface__ = {"shape": tuple(int(x) for x in shape), "typestr": typestr,
                                    "data": (int(address), False), "version": 3,
                                    "strides": None}

    return torch.as_tensor(_View(), device="cuda")


def debug_partition(n_pos, n_kv_heads, tile, n_ctas, unit_rows=64):
    """Host run of the decode work partition (no GPU). Returns a dict of arrays."""
    import numpy as np

    n_pos = np.ascontiguousarray(n_pos, dtype=np.int32)
    units = int(sum((max(int(x), 0) + unit_rows - 1) // unit_rows for x in n_pos)) * n_kv_heads
    cap = max(units + n_ctas + len(n_pos) * n_kv_heads, 1)
    arrs = [np.zeros(cap, dtype=np.int32) for _ in range(8)]
    rc = lib().gla_debug_partition(n_pos.ctypes.data, len(n_pos), n_kv_heads, tile, unit_rows,
                                   n_ctas, *[a.ctypes.data for a in arrs], cap)
    if rc < 0:
        raise GlaError(int(rc), "gla_debug_partition")
    names = ("cta", "seq", "kv_head", "row0", "rows", "slot", "first_cta", "npieces")
    return {k: a[:rc] for k, a in zip(names, arrs)}


class Context:
    """Owns one gla_ctx (device, stream, workspace)."""

    def __init__(self, device: int = 0, stream=None):
        self._L = lib()
        self._h = _P()
        if stream is None:
            try:
                import torch

                stream = torch.cuda.current_stream(device).cuda_stream
            except Exception:  # pragma: no cover - torch without CUDA
                stream = 0
        rc = self._L.gla_create(device, _P(int(stream) if stream else None), ctypes.byref(self._h))
        if rc != GLA_OK:
            raise GlaError(rc, "gla_create failed")
        self.device = device

    # -- plumbing ---------------------------------------------------------
    def _check(self, rc: int, what: str):
        if rc != GLA_OK:
            msg = self._L.gla_last_error(self._h)
            raise GlaError(rc, f"{what}: {msg.decode() if msg else ''}")

    def close(self):
        if self._h:
            self._L.gla_destroy(self._h)
            self._h = _P()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def set_stream(self, stream):
        self._check(self._L.gla_set_stream(self._h, _P(int(stream) if stream else None)),
                    "gla_set_stream")

    def num_sms(self) -> int:
        return int(self._L.gla_num_sms(self._h))

    def set_option(self, option: int, value: int):
        self._check(self._L.gla_set_option(self._h, option, value), "gla_set_option")

    def device_status(self) -> int:
        st = _I32(0)
        self._check(self._L.gla_device_status(self._h, ctypes.byref(st)), "gla_device_status")
        return int(st.value)

    def debug_trace(self):
        """Phase stamps of the last decode launch: uint64 array [CTA][16]
        (GLA_OPT_TRACE must be on)."""
        import numpy as np

        cap = 2 * self.num_sms() * 16
        out = np.zeros(cap, dtype=np.uint64)
        n = self._L.gla_debug_trace(self._h, out.ctypes.data, cap)
        if n < 0:
            self._check(int(n), "gla_debug_trace")
        return out[:n].reshape(-1, 16)

    def debug_advance_position(self, position_holder, delta, delay_us=20):
        """Test hook: a PDL kernel that adds delta to the device position."""
        self._check(self._L.gla_debug_advance_position(self._h, _ptr(position_holder), delta,
                                                       delay_us), "gla_debug_advance_position")

    def debug_xch_loopback(self, world):
        """Test hook: a one-process peer exchange whose other ranks never write."""
        self._check(self._L.gla_debug_xch_loopback(self._h, world), "gla_debug_xch_loopback")

    def reserve(self, max_batch, max_kv_heads, max_heads, max_head_dim):
        self._check(self._L.gla_reserve(self._h, max_batch, max_kv_heads, max_heads, max_head_dim),
                    "gla_reserve")

    # -- KV cache ---------------------------------------------------------
    def kv_cache_alloc(self, n_layers, context_length, kv_dim, dtype=DTYPE_F32):
        k, v = _P(), _P()
        self._check(self._L.gla_kv_cache_alloc(self._h, n_layers, context_length, kv_dim, dtype,
                                               ctypes.byref(k), ctypes.byref(v)),
                    "gla_kv_cache_alloc")
        return k.value, v.value

    def kv_cache_free(self, k, v):
        self._check(self._L.gla_kv_cache_free(self._h, _P(k), _P(v)), "gla_kv_cache_free")

    # -- the reference task -------------------------------------------------
    def process_heads_flash_attention(self, q, key_cache, value_cache, xb, n_heads, head_size,
                                      kv_dim, kv_mul, position_holder, layer, context_length,
                                      f16_cache=False):
        fn = (self._L.gla_process_heads_flash_attention_f16kv if f16_cache
              else self._L.gla_process_heads_flash_attention)
        self._check(fn(self._h, _ptr(q), _ptr(key_cache), _ptr(value_cache), _ptr(xb), n_heads,
                       head_size, kv_dim, kv_mul, _ptr(position_holder), layer, context_length),
                    "gla_process_heads_flash_attention")

    # -- decode -------------------------------------------------------------
    def decode(self, q, k, v, xb, n_heads, n_kv_heads, head_dim, n_pos, scale=None,
               kv_stride=None, f16_cache=False):
        if scale is None:
            scale = 1.0 / math.sqrt(head_dim)
        if kv_stride is None:
            kv_stride = n_kv_heads * head_dim
        fn = self._L.gla_decode_f16kv if f16_cache else self._L.gla_decode_f32kv
        self._check(fn(self._h, _ptr(q), _ptr(k), _ptr(v), _ptr(xb), n_heads, n_kv_heads,
                       head_dim, kv_stride, n_pos, scale), "gla_decode")

    def decode_partial(self, q, k, v, part, n_heads, n_kv_heads, head_dim, n_pos, scale=None,
                       kv_stride=None, f16_cache=False):
        if scale is None:
            scale = 1.0 / math.sqrt(head_dim)
        if kv_stride is None:
            kv_stride = n_kv_heads * head_dim
        fn = self._L.gla_decode_partial_f16kv if f16_cache else self._L.gla_decode_partial_f32kv
        self._check(fn(self._h, _ptr(q), _ptr(k), _ptr(v), _ptr(part), n_heads, n_kv_heads,
                       head_dim, kv_stride, n_pos, scale), "gla_decode_partial")

    def decode_batched(self, q, k_ptrs, v_ptrs, n_pos, max_n_pos, xb, batch, n_heads,
                       n_kv_heads, head_dim, scale=None, kv_stride=None, f16_cache=False):
        if scale is None:
            scale = 1.0 / math.sqrt(head_dim)
        if kv_stride is None:
            kv_stride = n_kv_heads * head_dim
        fn = self._L.gla_decode_batched_f16kv if f16_cache else self._L.gla_decode_batched_f32kv
        self._check(fn(self._h, _ptr(q), _ptr(k_ptrs), _ptr(v_ptrs), _ptr(n_pos), max_n_pos,
                       _ptr(xb), batch, n_heads, n_kv_heads, head_dim, kv_stride, scale),
                    "gla_decode_batched")

    def lse_combine(self, parts, n_parts, n_heads, head_dim, xb):
        self._check(self._L.gla_lse_combine(self._h, _ptr(parts), n_parts, n_heads, head_dim,
                                            _ptr(xb)), "gla_lse_combine")

    # -- multi-GPU ----------------------------------------------------------
    @staticmethod
    def comm_unique_id() -> bytes:
        L = lib()
        n = L.gla_comm_unique_id_size()
        buf = ctypes.create_string_buffer(n)
        rc = L.gla_comm_get_unique_id(buf)
        if rc != GLA_OK:
            raise GlaError(rc, "gla_comm_get_unique_id")
        return buf.raw

    def comm_init(self, nranks: int, rank: int, unique_id: bytes):
        buf = ctypes.create_string_buffer(unique_id, len(unique_id))
        self._check(self._L.gla_comm_init(self._h, nranks, rank, buf), "gla_comm_init")

    def comm_wait(self):
        """gla_comm_wait: bounded stream drain (aborts a stuck communicator)."""
        self._check(self._L.gla_comm_wait(self._h), "gla_comm_wait")

    def comm_resync(self):
        """gla_comm_resync: collective reset of the peer exchange epochs."""
        self._check(self._L.gla_comm_resync(self._h), "gla_comm_resync")

    @property
    def peer_exchange(self) -> bool:
        """True if sharded decode merges over the peer exchange (else NCCL)."""
        return bool(self._L.gla_comm_peer_exchange(self._h))

    def decode_sharded(self, q, k, v, xb, n_heads, n_kv_heads, head_dim, n_pos_local,
                       scale=None, kv_stride=None, f16_cache=True):
        if scale is None:
            scale = 1.0 / math.sqrt(head_dim)
        if kv_stride is None:
            kv_stride = n_kv_heads * head_dim
        fn = self._L.gla_decode_sharded_f16kv if f16_cache else self._L.gla_decode_sharded_f32kv
        self._check(fn(self._h, _ptr(q), _ptr(k), _ptr(v), _ptr(xb), n_heads, n_kv_heads,
                       head_dim, kv_stride, n_pos_local, scale), "gla_decode_sharded")

    # -- prefill / producers --------------------------------------------------
    def prefill_causal(self, q, k, v, out, L, n_heads, n_kv_heads, head_dim, scale=None):
        if scale is None:
            scale = 1.0 / math.sqrt(head_dim)
        self._check(self._L.gla_prefill_causal_f16(self._h, _ptr(q), _ptr(k), _ptr(v), _ptr(out),
                                                   L, n_heads, n_kv_heads, head_dim, scale),
                    "gla_prefill_causal_f16")

    def rope_append_attention(self, q, k, v, key_cache, value_cache, xb, n_heads, head_size,
                              kv_dim, kv_mul, position_holder, layer, context_length, theta,
                              style=ROPE_INTERLEAVED):
        """gla_rope_append_attention_f32: RoPE + KV append + attention, one launch."""
        self._check(self._L.gla_rope_append_attention_f32(
            self._h, _ptr(q), _ptr(k), _ptr(v), _ptr(key_cache), _ptr(value_cache), _ptr(xb),
            n_heads, head_size, kv_dim, kv_mul, _ptr(position_holder), layer, context_length,
            theta, style), "gla_rope_append_attention_f32")

    def decode_q8(self, q, k, v, scales, xb, n_heads, n_kv_heads, head_dim, n_pos,
                  kv_stride=None, scale=None):
        """gla_decode_q8kv: decode over a Q8 cache (int8 k/v, FP16 block scales)."""
        if kv_stride is None:
            kv_stride = n_kv_heads * head_dim
        if scale is None:
            scale = 1.0 / math.sqrt(head_dim)
        self._check(self._L.gla_decode_q8kv(self._h, _ptr(q), _ptr(k), _ptr(v), _ptr(scales),
                                            _ptr(xb), n_heads, n_kv_heads, head_dim, kv_stride,
                                            n_pos, scale), "gla_decode_q8kv")

    def quantize_q8(self, k, v, n_rows, n_kv_heads, head_dim, kq, vq, scales, src_stride=None,
                    kv_stride=None):
        """gla_kv_quantize_q8: FP32 K/V rows into Q8 cache rows."""
        if src_stride is None:
            src_stride = n_kv_heads * head_dim
        if kv_stride is None:
            kv_stride = n_kv_heads * head_dim
        self._check(self._L.gla_kv_quantize_q8(self._h, _ptr(k), _ptr(v), src_stride, n_rows,
                                               n_kv_heads, head_dim, _ptr(kq), _ptr(vq),
                                               kv_stride, _ptr(scales)), "gla_kv_quantize_q8")

    def rope_append_q8(self, q, k, v, kq, vq, scales, n_heads, n_kv_heads, head_dim,
                       position_holder, context_length, theta, style=ROPE_INTERLEAVED):
        """gla_rope_append_q8: RoPE of the new token, k/v quantised into a Q8 cache row."""
        self._check(self._L.gla_rope_append_q8(self._h, _ptr(q), _ptr(k), _ptr(v), _ptr(kq),
                                               _ptr(vq), _ptr(scales), n_heads, n_kv_heads,
                                               head_dim, _ptr(position_holder), context_length,
                                               theta, style), "gla_rope_append_q8")

    def kv_cache_alloc_q8(self, n_layers, context_length, n_kv_heads, head_dim):
        """gla_kv_cache_alloc_q8: returns (k, v, scales) device addresses."""
        k, v, s = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        self._check(self._L.gla_kv_cache_alloc_q8(self._h, n_layers, context_length, n_kv_heads,
                                                  head_dim, ctypes.byref(k), ctypes.byref(v),
                                                  ctypes.byref(s)), "gla_kv_cache_alloc_q8")
        return k.value, v.value, s.value

    def kv_cache_free_q8(self, k, v, scales):
        self._check(self._L.gla_kv_cache_free_q8(self._h, ctypes.c_void_p(k), ctypes.c_void_p(v),
                                                 ctypes.c_void_p(scales)), "gla_kv_cache_free_q8")

    def wo_residual(self, xb, x, w, n, d):
        """gla_wo_residual_f16: x += w . xb (w FP16 [d][n])."""
        self._check(self._L.gla_wo_residual_f16(self._h, _ptr(xb), _ptr(x), _ptr(w), n, d),
                    "gla_wo_residual_f16")

    def ingest_prompt(self, q, k, v, key_cache, value_cache, xb, start_pos, n_rows, n_heads,
                      n_kv_heads, head_dim, context_length, theta, style=ROPE_INTERLEAVED,
                      f16_cache=False):
        """gla_ingest_prompt_f32/_f16kv: RoPE, KV append and causal attention of
        positions start_pos..start_pos+n_rows-1 of one layer."""
        name = "gla_ingest_prompt_f16kv" if f16_cache else "gla_ingest_prompt_f32"
        self._check(getattr(self._L, name)(
            self._h, _ptr(q), _ptr(k), _ptr(v), _ptr(key_cache), _ptr(value_cache), _ptr(xb),
            start_pos, n_rows, n_heads, n_kv_heads, head_dim, context_length, theta, style), name)

    def rope_append(self, q, k, v, key_cache, value_cache, n_heads, n_kv_heads, head_dim,
                    position_holder, theta, style=ROPE_INTERLEAVED):
        self._check(self._L.gla_rope_append_f32(self._h, _ptr(q), _ptr(k), _ptr(v),
                                                _ptr(key_cache), _ptr(value_cache), n_heads,
                                                n_kv_heads, head_dim, _ptr(position_holder),
                                                theta, style), "gla_rope_append_f32")
