"""C ABI: the library loads, exports every declared symbol, and rejects bad
arguments without touching a GPU."""
import ctypes
import os
import re

import numpy as np
import pytest

import gpullama_attn as gla

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "gpullama_attn.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gla_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = gla.lib()
    names = declared_symbols()
    assert len(names) >= 25
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    # the binding covers the whole header too
    assert sorted(gla.EXPORTED_SYMBOLS) == names


def test_version_and_status_strings():
    L = gla.lib()
    assert L.gla_version() == 100
    assert L.gla_status_string(0) == b"GLA_OK"
    assert L.gla_status_string(-5) == b"GLA_ERR_TIMEOUT"
    assert L.gla_status_string(-99) == b"GLA_ERR_UNKNOWN"


def test_null_context_is_rejected():
    L = gla.lib()
    assert L.gla_decode_f32kv(None, None, None, None, None, 8, 2, 64, 128, 1, 0.125) == -1
    assert L.gla_decode_f16kv(None, None, None, None, None, 8, 2, 64, 128, 1, 0.125) == -1
    assert L.gla_process_heads_flash_attention(None, None, None, None, None, 8, 64, 128, 4, None,
                                               0, 16) == -1
    assert L.gla_lse_combine(None, None, 1, 1, 1, None) == -1
    assert L.gla_prefill_causal_f16(None, None, None, None, None, 8, 4, 4, 64, 0.1) == -1
    assert L.gla_ingest_prompt_f32(None, None, None, None, None, None, None, 0, 4, 8, 2, 64, 16,
                                   1e4, 0) == -1
    assert L.gla_ingest_prompt_f16kv(None, None, None, None, None, None, None, 0, 4, 8, 2, 64,
                                     16, 1e4, 0) == -1
    assert L.gla_wo_residual_f16(None, None, None, None, 64, 64) == -1
    assert L.gla_decode_q8kv(None, None, None, None, None, None, 8, 2, 64, 128, 1, 0.125) == -1
    assert L.gla_kv_quantize_q8(None, None, None, 128, 1, 2, 64, None, None, 128, None) == -1
    assert L.gla_kv_cache_alloc_q8(None, 1, 16, 2, 64, None, None, None) == -1
    assert L.gla_kv_cache_free_q8(None, None, None, None) == -1
    assert L.gla_rope_append_q8(None, None, None, None, None, None, None, 8, 2, 64, None, 16, 1e4,
                                0) == -1
    assert L.gla_destroy(None) == -1
    assert L.gla_device_status(None, None) == -1
    assert L.gla_last_error(None) == b""


def test_create_without_gpu_reports_no_device():
    try:
        import torch

        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    h = ctypes.c_void_p()
    assert gla.lib().gla_create(0, None, ctypes.byref(h)) == -7
    assert not h.value
    assert gla.lib().gla_create(0, None, None) == -1


def test_comm_unique_id_size():
    assert gla.lib().gla_comm_unique_id_size() == 128
