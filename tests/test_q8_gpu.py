"""Q8 KV cache (gla_kv_quantize_q8, gla_decode_q8kv) through the C ABI.

Quantisation is integer/byte work: the kernel's int8 values and FP16 scales
must equal the oracle's (GGML's Q8_0 reference quantiser restated in C) bit
for bit.  Decode computes attention over the dequantised values q * scale,
so it is checked against the FP32 oracle run on exactly those values with the
FP32 tolerance 1e-3 (max |err| and max |err| / max |ref|).
"""
import numpy as np
import pytest

import inputs

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _torch():
    import torch

    return torch


def _dev(x):
    torch = _torch()
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _quantize_gpu(ctx, k, v, n_kv, hd, kv_stride=None):
    torch = _torch()
    rows = k.shape[0]
    kv_stride = kv_stride or n_kv * hd
    kq = torch.full((rows, kv_stride), 99, dtype=torch.int8, device="cuda")
    vq = torch.full_like(kq, 99)
    sc = torch.full((rows, n_kv, 8), 12345, dtype=torch.int16, device="cuda")
    ctx.quantize_q8(_dev(k), _dev(v), rows, n_kv, hd, kq, vq, sc, kv_stride=kv_stride)
    assert ctx.device_status() == 0
    return kq.cpu().numpy(), vq.cpu().numpy(), sc.cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("rows,n_kv,hd,pad", [(300, 8, 128, 0), (77, 2, 64, 32), (5, 4, 128, 16)])
def test_quantize_matches_oracle_bitwise(gla_ctx, oracle, rows, n_kv, hd, pad):
    rng = np.random.Generator(np.random.PCG64(rows + hd))
    k = rng.standard_normal((rows, n_kv * hd), dtype=np.float32) * 3
    v = rng.standard_normal((rows, n_kv * hd), dtype=np.float32)
    k[0, :32] = 0.0           # an all-zero block: d = 0, q = 0
    k[1, 32:64] = 1e-30       # tiny values
    v[2, :hd] *= 1e4          # large values
    k[3, 5] = -127.5          # exact ties
    kq, vq, sc = _quantize_gpu(gla_ctx, k, v, n_kv, hd, n_kv * hd + pad)
    rq, rv, rs = oracle.quantize_q8(k, v, n_kv, hd)
    np.testing.assert_array_equal(kq[:, :n_kv * hd], rq)
    np.testing.assert_array_equal(vq[:, :n_kv * hd], rv)
    np.testing.assert_array_equal(sc, rs)
    if pad:  # the padding columns are not touched
        assert (kq[:, n_kv * hd:] == 99).all() and (vq[:, n_kv * hd:] == 99).all()


CASES = [
    # nh, nkv, hd, T
    (24, 8, 128, 4096),   # Llama-3.2-3B shape
    (28, 4, 128, 20000),  # Qwen2.5-7B shape
    (32, 8, 64, 777),     # hd 64
    (8, 8, 128, 300),     # MHA
    (24, 8, 128, 1),
    (24, 8, 128, 63),
    (24, 8, 128, 65),
    (14, 2, 64, 129),
]


@pytest.mark.parametrize("nh,nkv,hd,T", CASES)
def test_decode_q8_matches_oracle_on_dequantised_cache(gla_ctx, oracle, nh, nkv, hd, T):
    torch = _torch()
    q, k, v = inputs.decode_case(T + nh, nh, nkv, hd, T)
    kq, vq, sc = oracle.quantize_q8(k, v, nkv, hd)
    kd, vd = oracle.dequantize_q8(kq, vq, sc, nkv, hd)
    xb = torch.full((nh * hd,), float("nan"), device="cuda")
    gla_ctx.decode_q8(_dev(q), _dev(kq), _dev(vq), _dev(sc.view(np.int16)), xb, nh, nkv, hd, T)
    assert gla_ctx.device_status() == 0
    got = xb.cpu().numpy()
    ref = oracle.decode_f32(q, kd, vd, nh, nkv, hd, T)
    err = np.abs(got - ref).max()
    assert np.isfinite(got).all()
    assert err <= TOL and err / np.abs(ref).max() <= TOL, err
    # and it stays close to attention over the unquantised cache
    ref32 = oracle.decode_f32(q, k, v, nh, nkv, hd, T)
    assert np.abs(got - ref32).max() <= 0.05 * np.abs(ref32).max()


def test_decode_q8_strided_cache_and_gpu_quantiser(gla_ctx, oracle):
    """A padded Q8 cache filled by the GPU quantiser, read through kv_stride."""
    torch = _torch()
    nh, nkv, hd, T, pad = 16, 4, 128, 1500, 64
    q, k, v = inputs.decode_case(3, nh, nkv, hd, T)
    stride = nkv * hd + pad
    kq = torch.zeros((T, stride), dtype=torch.int8, device="cuda")
    vq = torch.zeros_like(kq)
    sc = torch.zeros((T, nkv, 8), dtype=torch.int16, device="cuda")
    gla_ctx.quantize_q8(_dev(k), _dev(v), T, nkv, hd, kq, vq, sc, kv_stride=stride)
    xb = torch.empty(nh * hd, device="cuda")
    gla_ctx.decode_q8(_dev(q), kq, vq, sc, xb, nh, nkv, hd, T, kv_stride=stride)
    assert gla_ctx.device_status() == 0
    rq, rv, rs = oracle.quantize_q8(k, v, nkv, hd)
    kd, vd = oracle.dequantize_q8(rq, rv, rs, nkv, hd)
    ref = oracle.decode_f32(q, kd, vd, nh, nkv, hd, T)
    got = xb.cpu().numpy()
    err = np.abs(got - ref).max()
    assert err <= TOL and err / np.abs(ref).max() <= TOL, err


def test_decode_q8_rejects_bad_arguments(gla_ctx):
    import gpullama_attn as gla

    torch = _torch()
    q = torch.zeros(8 * 96, device="cuda")
    kq = torch.zeros((64, 8 * 128), dtype=torch.int8, device="cuda")
    sc = torch.zeros((64, 8, 8), dtype=torch.int16, device="cuda")
    xb = torch.zeros(8 * 128, device="cuda")
    with pytest.raises(gla.GlaError):  # head_dim 96
        gla_ctx.decode_q8(q, kq, kq, sc, xb, 8, 8, 96, 10)
    with pytest.raises(gla.GlaError):  # kv_stride not a multiple of 16
        gla_ctx.decode_q8(xb, kq, kq, sc, xb, 8, 8, 128, 10, kv_stride=8 * 128 + 8)
    with pytest.raises(gla.GlaError):  # scales not 16-byte aligned
        gla_ctx.decode_q8(xb, kq, kq, sc.view(-1)[1:], xb, 8, 8, 128, 10)
