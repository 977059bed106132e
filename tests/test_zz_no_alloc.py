"""gla_decode_f32kv_noalloc: decode attention for callers that cannot
allocate device memory (its scratch is a static device array of the library).

The file name sorts last so that a run stopping at the first failure has
already run every other test.  It needs nothing from other tests: it runs
alone in a fresh process as well as after them.
"""
import ctypes
import math

import numpy as np
import pytest

import gpullama_attn as gla
import inputs

pytestmark = pytest.mark.gpu

TOL_F32 = 1e-3


def _close(got, ref):
    err = float(np.abs(got.astype(np.float64) - ref.astype(np.float64)).max())
    scale = float(np.abs(ref).max())
    return err <= TOL_F32 and err / scale <= TOL_F32, err


def test_noalloc_matches_context_entry_point_on_two_calls_in_a_row(oracle):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    L = gla.lib()
    stream = torch.cuda.current_stream().cuda_stream
    ctx = gla.Context(0, stream)  # the existing entry point, for comparison
    # different shapes back to back: every call reuses the scratch the one
    # before it left behind.  Config-2 layer (many pieces a kv head), config
    # 1, kvMul 8 with head_dim 96, and 4 kv heads over 37 CTAs each.
    cases = [(24, 8, 128, 4096, 61), (32, 8, 64, 512, 62), (16, 2, 96, 3000, 63),
             (16, 4, 128, 20000, 64)]
    for nh, nkv, hd, n, seed in cases:
        q, k, v = inputs.decode_case(seed, nh, nkv, hd, n)
        qd, kd, vd = (torch.from_numpy(x).cuda() for x in (q, k, v))
        want = torch.empty(nh * hd, device="cuda")
        got = torch.full((nh * hd,), float("nan"), device="cuda")
        ctx.decode(qd, kd, vd, want, nh, nkv, hd, n)
        # the context call's own status (its scratch is the context workspace)
        assert ctx.device_status() == 0
        rc = L.gla_decode_f32kv_noalloc(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(),
                                        got.data_ptr(), nh, nkv, hd, nkv * hd, n,
                                        1.0 / math.sqrt(hd), ctypes.c_void_p(stream))
        assert rc == 0, gla.STATUS_NAMES.get(rc, rc)
        torch.cuda.synchronize()
        got_np = got.cpu().numpy()
        ok, err = _close(got_np, want.cpu().numpy())
        assert ok, f"shape {(nh, nkv, hd, n)}: max abs err {err:.3e} against gla_decode_f32kv"
        ok, err = _close(got_np, oracle.decode_f32(q, k, v, nh, nkv, hd, n))
        assert ok, f"shape {(nh, nkv, hd, n)}: max abs err {err:.3e} against the oracle"
    ctx.close()


def test_noalloc_rejects_sizes_beyond_its_scratch():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    L = gla.lib()
    # 2048 kv heads exceed the 1024 arrival counters: refused before any launch
    nh = nkv = 2048
    hd = 64
    q = torch.zeros(nh * hd, device="cuda")
    k = torch.zeros(4, nkv * hd, device="cuda")
    rc = L.gla_decode_f32kv_noalloc(q.data_ptr(), k.data_ptr(), k.data_ptr(), q.data_ptr(), nh,
                                    nkv, hd, nkv * hd, 4, 0.125, None)
    assert rc == -3  # GLA_ERR_NOT_SUPPORTED
    rc = L.gla_decode_f32kv_noalloc(None, k.data_ptr(), k.data_ptr(), q.data_ptr(), 8, 2, 64,
                                    128, 4, 0.125, None)
    assert rc == -1  # GLA_ERR_INVALID_ARG
