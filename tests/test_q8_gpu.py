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
    v[4, 32:64] = 1e-39       # subnormal block: 1/d overflows, q = 0
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


def test_q8_token_flow_alloc_rope_append_decode(gla_ctx, oracle):
    """The per-token flow over a Q8 cache layer from gla_kv_cache_alloc_q8:
    history rows quantised, the new token's q/k rotated and k/v appended by
    gla_rope_append_q8 at the device position, then gla_decode_q8kv.  The
    appended row equals the oracle quantiser applied to the rotated k (bit for
    bit); q and k are rotated like the FP32 RoPE (atol 2e-6); attention matches
    the FP32 oracle on the dequantised cache; untouched rows stay zero."""
    import gpullama_attn as gla

    torch = _torch()
    nh, nkv, hd, T, ctx_len, layers, theta = 24, 8, 128, 700, 1024, 2, 500000.0
    kvd = nkv * hd
    kp, vp, sp = gla_ctx.kv_cache_alloc_q8(layers, ctx_len, nkv, hd)
    try:
        layer = 1
        kl = kp + layer * ctx_len * kvd
        vl = vp + layer * ctx_len * kvd
        sl = sp + layer * ctx_len * nkv * 8 * 2  # bytes
        rng = np.random.Generator(np.random.PCG64(77))
        hist_k = rng.standard_normal((T - 1, kvd), dtype=np.float32)
        hist_v = rng.standard_normal((T - 1, kvd), dtype=np.float32)
        gla_ctx.quantize_q8(_dev(hist_k), _dev(hist_v), T - 1, nkv, hd, kl, vl, sl)
        q = rng.standard_normal(nh * hd, dtype=np.float32)
        kn = rng.standard_normal(kvd, dtype=np.float32)
        vn = rng.standard_normal(kvd, dtype=np.float32)
        qd, kd, vd = _dev(q), _dev(kn), _dev(vn)
        ph = torch.tensor([T - 1], dtype=torch.int32, device="cuda")
        gla_ctx.rope_append_q8(qd, kd, vd, kl, vl, sl, nh, nkv, hd, ph, ctx_len, theta,
                               gla.ROPE_INTERLEAVED)
        xb = torch.empty(nh * hd, device="cuda")
        gla_ctx.decode_q8(qd, kl, vl, sl, xb, nh, nkv, hd, T)
        assert gla_ctx.device_status() == 0

        # the layer read back through views of the raw device addresses
        def view(ptr, shape, typestr):
            class _Mem:
                __cuda_array_interface__ = {"shape": shape, "typestr": typestr,
                                            "data": (ptr, False), "version": 3, "strides": None}
            return torch.as_tensor(_Mem(), device="cuda").cpu().numpy()

        ck = view(kl, (ctx_len, kvd), "|i1")
        cv = view(vl, (ctx_len, kvd), "|i1")
        cs = view(sl, (ctx_len, nkv, 8), "<u2")
        assert (ck[T:] == 0).all() and (cv[T:] == 0).all() and (cs[T:] == 0).all()
        q_rot, k_rot = qd.cpu().numpy(), kd.cpu().numpy()
        cr, ci = oracle.rope_freqs(ctx_len, hd, theta)
        qr, kr = q.copy(), kn.copy()
        oracle.rope_interleaved(qr, kr, hd, T - 1, cr, ci)
        np.testing.assert_allclose(q_rot, qr, rtol=0, atol=2e-6)
        np.testing.assert_allclose(k_rot, kr, rtol=0, atol=2e-6)
        rq, rv, rs = oracle.quantize_q8(k_rot[None], vn[None], nkv, hd)
        np.testing.assert_array_equal(ck[T - 1], rq[0])
        np.testing.assert_array_equal(cv[T - 1], rv[0])
        np.testing.assert_array_equal(cs[T - 1], rs[0])
        hq, hv, hs = oracle.quantize_q8(hist_k, hist_v, nkv, hd)
        np.testing.assert_array_equal(ck[:T - 1], hq)
        np.testing.assert_array_equal(cs[:T - 1], hs)
        kd_all, vd_all = oracle.dequantize_q8(ck[:T], cv[:T], cs[:T], nkv, hd)
        ref = oracle.decode_f32(q_rot, kd_all, vd_all, nh, nkv, hd, T)
        got = xb.cpu().numpy()
        err = np.abs(got - ref).max()
        assert err <= TOL and err / np.abs(ref).max() <= TOL, err
        # a position past the context writes nothing and latches an error
        ph_bad = torch.tensor([ctx_len], dtype=torch.int32, device="cuda")
        gla_ctx.rope_append_q8(qd, kd, vd, kl, vl, sl, nh, nkv, hd, ph_bad, ctx_len, theta,
                               gla.ROPE_INTERLEAVED)
        assert gla_ctx.device_status() == -1  # GLA_ERR_INVALID_ARG, then cleared
        assert gla_ctx.device_status() == 0
    finally:
        gla_ctx.kv_cache_free_q8(kp, vp, sp)
