"""Decode attention on the GPU (through the C ABI) against the CPU oracle.

Tolerances: max |err| <= 1e-3 and max |err| / max |ref|
<= 1e-3 with an FP32 cache; 5e-3 for both with an FP16 cache.
"""
import math

import numpy as np
import pytest

import inputs
import reference64

pytestmark = pytest.mark.gpu

TOL_F32 = 1e-3
TOL_F16 = 5e-3


def _torch():
    import torch

    return torch


def dev(x):
    torch = _torch()
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def assert_close(got, ref, tol, what=""):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(got - ref).max()
    scale = max(np.abs(ref).max(), 1e-30)
    assert err <= tol and err / scale <= tol, f"{what}: max abs err {err:.3e}, rel {err / scale:.3e}"


def gpu_decode(ctx, q, k, v, nh, nkv, hd, n_pos, f16=False, kv_stride=None):
    torch = _torch()
    if f16:
        k, v = inputs.to_f16_bits(k), inputs.to_f16_bits(v)
    qd, kd, vd = dev(q), dev(k.view(np.int16) if f16 else k), dev(v.view(np.int16) if f16 else v)
    xb = torch.empty(nh * hd, dtype=torch.float32, device="cuda")
    ctx.decode(qd, kd, vd, xb, nh, nkv, hd, n_pos, kv_stride=kv_stride, f16_cache=f16)
    assert ctx.device_status() == 0
    return xb.cpu().numpy(), k, v


SWEEP_POS = [0, 1, 7, 8, 31, 32, 33, 511, 4095]


@pytest.mark.parametrize("f16", [False, True], ids=["f32kv", "f16kv"])
@pytest.mark.parametrize("hd", [64, 96, 128])
@pytest.mark.parametrize("kv_mul", [1, 3, 4, 7, 8])
def test_decode_sweep(gla_ctx, oracle, f16, hd, kv_mul):
    nkv = 2
    nh = nkv * kv_mul
    n_rows = max(SWEEP_POS) + 1
    q, k, v = inputs.decode_case(1000 + hd + kv_mul, nh, nkv, hd, n_rows)
    for pos in SWEEP_POS:
        xb, kk, vv = gpu_decode(gla_ctx, q, k, v, nh, nkv, hd, pos + 1, f16=f16)
        if f16:
            ref = oracle.decode_f16(q, kk, vv, nh, nkv, hd, pos + 1)
        else:
            ref = oracle.decode_f32(q, k, v, nh, nkv, hd, pos + 1)
        assert_close(xb, ref, TOL_F16 if f16 else TOL_F32, f"pos={pos}")


def test_golden_fixtures_on_gpu(gla_ctx):
    import os

    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "attention_golden.npz"))
    names = sorted({k.split("/")[0] for k in g.files if k.endswith("/xb")})
    for name in names:
        seed, nh, nkv, hd, npos, f16 = (int(x) for x in g[f"{name}/meta"])
        if f"{name}/q" in g.files:
            q, k, v = g[f"{name}/q"], g[f"{name}/k"], g[f"{name}/v"]
            if f16:
                k = k.view(np.float16).astype(np.float32)
                v = v.view(np.float16).astype(np.float32)
        else:
            q, k, v = inputs.decode_case(seed, nh, nkv, hd, npos)
        xb, _, _ = gpu_decode(gla_ctx, q, k, v, nh, nkv, hd, npos, f16=bool(f16))
        assert_close(xb, g[f"{name}/xb"], TOL_F16 if f16 else TOL_F32, name)


def test_c1_llama32_1b_exact_config(gla_ctx, oracle):
    # nHeads 32, nKVHeads 8, hd 64, position 511, seed 0
    q, k, v = inputs.decode_case(0, 32, 8, 64, 512)
    xb, _, _ = gpu_decode(gla_ctx, q, k, v, 32, 8, 64, 512)
    assert_close(xb, oracle.decode_f32(q, k, v, 32, 8, 64, 512), TOL_F32, "C1")


@pytest.mark.parametrize("f16", [False, True])
def test_padded_kv_stride(gla_ctx, oracle, f16):
    nh, nkv, hd, n = 8, 2, 128, 300
    stride = nkv * hd + 64
    q, k, v = inputs.decode_case(21, nh, nkv, hd, n, kv_stride=stride)
    xb, kk, vv = gpu_decode(gla_ctx, q, k, v, nh, nkv, hd, n, f16=f16, kv_stride=stride)
    if f16:
        ref = oracle.decode_f16(q, kk, vv, nh, nkv, hd, n, kv_stride=stride)
    else:
        ref = oracle.decode_f32(q, k, v, nh, nkv, hd, n, kv_stride=stride)
    assert_close(xb, ref, TOL_F16 if f16 else TOL_F32)


def test_repeated_calls_are_identical(gla_ctx):
    # the piece counters reset themselves: back-to-back calls agree bit for bit
    q, k, v = inputs.decode_case(22, 24, 8, 128, 4096)
    a, _, _ = gpu_decode(gla_ctx, q, k, v, 24, 8, 128, 4096)
    for _ in range(3):
        b, _, _ = gpu_decode(gla_ctx, q, k, v, 24, 8, 128, 4096)
        np.testing.assert_array_equal(a, b)


def test_process_heads_flash_attention_mirror(gla_ctx, oracle):
    """The reference task signature: flat [layer][ctx][kvDim] caches, device position."""
    torch = _torch()
    n_layers, ctx_len, nh, nkv, hd = 3, 256, 16, 4, 64
    kv_dim = nkv * hd
    rng = np.random.Generator(np.random.PCG64(23))
    kc = rng.standard_normal((n_layers, ctx_len, kv_dim), dtype=np.float32)
    vc = rng.standard_normal((n_layers, ctx_len, kv_dim), dtype=np.float32)
    q = rng.standard_normal(nh * hd, dtype=np.float32)
    kd, vd, qd = dev(kc), dev(vc), dev(q)
    xb = torch.empty(nh * hd, device="cuda")
    for layer in range(n_layers):
        for pos in (0, 100, ctx_len - 1):
            ph = torch.tensor([pos], dtype=torch.int32, device="cuda")
            gla_ctx.process_heads_flash_attention(qd, kd, vd, xb, nh, hd, kv_dim, nh // nkv, ph,
                                                  layer, ctx_len)
            assert gla_ctx.device_status() == 0
            ref = oracle.decode_f32(q, kc[layer], vc[layer], nh, nkv, hd, pos + 1)
            assert_close(xb.cpu().numpy(), ref, TOL_F32, f"layer {layer} pos {pos}")


def test_process_heads_position_beyond_context_is_latched(gla_ctx):
    torch = _torch()
    nh, nkv, hd, ctx_len = 8, 2, 64, 64
    kd = torch.zeros(ctx_len, nkv * hd, device="cuda")
    vd = torch.zeros_like(kd)
    qd = torch.zeros(nh * hd, device="cuda")
    xb = torch.empty_like(qd)
    ph = torch.tensor([ctx_len + 5], dtype=torch.int32, device="cuda")
    gla_ctx.process_heads_flash_attention(qd, kd, vd, xb, nh, hd, nkv * hd, nh // nkv, ph, 0,
                                          ctx_len)
    assert gla_ctx.device_status() == -1  # GLA_ERR_INVALID_ARG, rows clamped to the cache
    assert gla_ctx.device_status() == 0   # cleared by the read


@pytest.mark.parametrize("f16", [False, True])
def test_batched_ragged(gla_ctx, oracle, f16):
    torch = _torch()
    nh, nkv, hd = 32, 8, 128
    lengths = [1, 17, 64, 65, 1000, 3333, 128]
    B = len(lengths)
    qs, ks, vs, refs = [], [], [], []
    for b, n in enumerate(lengths):
        q, k, v = inputs.decode_case(300 + b, nh, nkv, hd, n)
        if f16:
            k16, v16 = inputs.to_f16_bits(k), inputs.to_f16_bits(v)
            refs.append(oracle.decode_f16(q, k16, v16, nh, nkv, hd, n))
            ks.append(dev(k16.view(np.int16)))
            vs.append(dev(v16.view(np.int16)))
        else:
            refs.append(oracle.decode_f32(q, k, v, nh, nkv, hd, n))
            ks.append(dev(k))
            vs.append(dev(v))
        qs.append(q)
    qd = dev(np.stack(qs))
    kp = torch.tensor([t.data_ptr() for t in ks], dtype=torch.int64, device="cuda")
    vp = torch.tensor([t.data_ptr() for t in vs], dtype=torch.int64, device="cuda")
    npd = torch.tensor(lengths, dtype=torch.int32, device="cuda")
    xb = torch.empty(B, nh * hd, device="cuda")
    gla_ctx.decode_batched(qd, kp, vp, npd, max(lengths), xb, B, nh, nkv, hd, f16_cache=f16)
    assert gla_ctx.device_status() == 0
    out = xb.cpu().numpy()
    for b in range(B):
        assert_close(out[b], refs[b], TOL_F16 if f16 else TOL_F32, f"seq {b}")


@pytest.mark.parametrize("f16", [False, True])
def test_partial_records_and_combine(gla_ctx, oracle, f16):
    """KV-sequence sharding emulated on one GPU: shard records merge to the full result."""
    torch = _torch()
    nh, nkv, hd, n = 28, 4, 128, 5000
    q, k, v = inputs.decode_case(31, nh, nkv, hd, n)
    bounds = [0, 1, 1700, 3001, n]  # includes a one-row shard
    S = len(bounds) - 1
    parts = torch.empty(S, nh, hd + 2, device="cuda")
    if f16:
        k16, v16 = inputs.to_f16_bits(k), inputs.to_f16_bits(v)
        kq = k16.view(np.float16).astype(np.float32)
        vq = v16.view(np.float16).astype(np.float32)
    else:
        kq, vq = k, v
    qd = dev(q)
    keep = []
    for s in range(S):
        lo, hi = bounds[s], bounds[s + 1]
        if f16:
            ks = dev(k16[lo:hi].view(np.int16))
            vs = dev(v16[lo:hi].view(np.int16))
        else:
            ks, vs = dev(k[lo:hi]), dev(v[lo:hi])
        keep += [ks, vs]
        gla_ctx.decode_partial(qd, ks, vs, parts[s], nh, nkv, hd, hi - lo, f16_cache=f16)
        assert gla_ctx.device_status() == 0
        rec = parts[s].cpu().numpy()
        want = reference64.records64(q, kq, vq, nh, nkv, hd, slice(lo, hi))
        tol = TOL_F16 if f16 else TOL_F32
        assert_close(rec[:, :hd], want[:, :hd], tol, f"o shard {s}")
        np.testing.assert_allclose(rec[:, hd], want[:, hd], atol=tol * 10)
        np.testing.assert_allclose(rec[:, hd + 1], want[:, hd + 1], rtol=tol * 10)
    xb = torch.empty(nh * hd, device="cuda")
    gla_ctx.lse_combine(parts, S, nh, hd, xb)
    ref = (oracle.decode_f16(q, k16, v16, nh, nkv, hd, n) if f16
           else oracle.decode_f32(q, k, v, nh, nkv, hd, n))
    assert_close(xb.cpu().numpy(), ref, TOL_F16 if f16 else TOL_F32, "combined")


def test_argument_errors_with_context(gla_ctx):
    torch = _torch()
    import gpullama_attn as gla

    q = torch.zeros(8 * 64 + 4, device="cuda")
    k = torch.zeros(64, 128, device="cuda")
    xb = torch.zeros(8 * 64, device="cuda")
    with pytest.raises(gla.GlaError) as e:  # misaligned q
        gla_ctx.decode(q.data_ptr() + 4, k, k, xb, 8, 2, 64, 10)
    assert e.value.status == -4
    with pytest.raises(gla.GlaError) as e:  # unsupported head_dim
        gla_ctx.decode(q, k, k, xb, 8, 2, 80, 10, kv_stride=160)
    assert e.value.status == -3
    with pytest.raises(gla.GlaError) as e:  # kvMul 16 > 8
        gla_ctx.decode(q, k, k, xb, 16, 1, 64, 10, kv_stride=128)
    assert e.value.status == -3
    with pytest.raises(gla.GlaError) as e:  # n_pos 0
        gla_ctx.decode(q, k, k, xb, 8, 2, 64, 0)
    assert e.value.status == -1
    assert "n_pos" in str(e.value)
    assert gla_ctx.device_status() == 0


def test_c2_layer_full_size(gla_ctx, oracle):
    # Llama-3.2-3B shape, context 4096, FP32 cache, RoPE'd inputs (theta 500000)
    nh, nkv, hd, T = 24, 8, 128, 4096
    q, k, v = inputs.decode_case(41, nh, nkv, hd, T)
    cr, ci = oracle.rope_freqs(T, hd, 500000.0)
    oracle.rope_interleaved(q, k[T - 1], hd, T - 1, cr, ci)  # q and the new key at pos T-1
    scratch = np.zeros(nh * hd, np.float32)
    for t in range(T - 1):  # every cached key was rotated at its own position
        oracle.rope_interleaved(scratch, k[t], hd, t, cr, ci)
    xb, _, _ = gpu_decode(gla_ctx, q, k, v, nh, nkv, hd, T)
    assert_close(xb, oracle.decode_f32(q, k, v, nh, nkv, hd, T), TOL_F32, "C2")


def test_c4_long_context_full_size(gla_ctx, oracle):
    # Qwen2.5-7B shape, context 131072, FP16 cache
    nh, nkv, hd, T = 28, 4, 128, 131072
    q, k, v = inputs.decode_case(42, nh, nkv, hd, T)
    k16, v16 = inputs.to_f16_bits(k), inputs.to_f16_bits(v)
    del k, v
    xb, _, _ = gpu_decode(gla_ctx, q, k16.view(np.float16).astype(np.float32),
                          v16.view(np.float16).astype(np.float32), nh, nkv, hd, T, f16=True)
    assert_close(xb, oracle.decode_f16(q, k16, v16, nh, nkv, hd, T), TOL_F16, "C4")


def test_rope_append_matches_oracle(gla_ctx, oracle):
    import os

    torch = _torch()
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "attention_golden.npz"))
    for name in ("rope_llama3_theta5e5_pos123", "rope_neox_theta1e6_pos77"):
        seed, nh, nkv, hd, pos, style = (int(x) for x in g[f"{name}/meta"])
        theta = float(g[f"{name}/theta"])
        qd, kd = dev(g[f"{name}/q_in"]), dev(g[f"{name}/k_in"])
        rng = np.random.Generator(np.random.PCG64(seed + 1))
        vin = rng.standard_normal(nkv * hd, dtype=np.float32)
        vd = dev(vin)
        kc = torch.zeros(pos + 1, nkv * hd, device="cuda")
        vc = torch.zeros_like(kc)
        ph = torch.tensor([pos], dtype=torch.int32, device="cuda")
        gla_ctx.rope_append(qd, kd, vd, kc, vc, nh, nkv, hd, ph, theta, style)
        assert gla_ctx.device_status() == 0
        np.testing.assert_allclose(qd.cpu().numpy(), g[f"{name}/q_out"], rtol=0, atol=2e-6)
        np.testing.assert_allclose(kd.cpu().numpy(), g[f"{name}/k_out"], rtol=0, atol=2e-6)
        np.testing.assert_array_equal(kc[pos].cpu().numpy(), kd.cpu().numpy())
        np.testing.assert_array_equal(vc[pos].cpu().numpy(), vin)
        assert float(kc[:pos].abs().sum()) == 0.0


def test_early_prefetch_sees_the_row_appended_just_before(gla_ctx, oracle):
    """RoPE + KV append writes row `pos`, then a decode over rows 0..pos runs
    right after it on the same stream: the early history prefetch must not
    read the newest row before the append has finished, and the result must
    not depend on the option."""
    import gpullama_attn as gla

    torch = _torch()
    nh, nkv, hd, T = 24, 8, 128, 2000
    pos = T - 1
    q0, k, v = inputs.decode_case(51, nh, nkv, hd, T)
    rng = np.random.Generator(np.random.PCG64(52))
    knew = rng.standard_normal(nkv * hd, dtype=np.float32)
    vnew = rng.standard_normal(nkv * hd, dtype=np.float32)
    k[pos] = 7.0  # stale row contents the append must replace
    v[pos] = -7.0
    outs, outs_dev = [], []
    for opt in (2, 1, 0):
        gla_ctx.set_option(gla.OPT_EARLY_KV_PREFETCH, opt)
        kc, vc = dev(k), dev(v)
        qd, kd, vd = dev(q0), dev(knew), dev(vnew)
        ph = torch.tensor([pos], dtype=torch.int32, device="cuda")
        xb = torch.empty(nh * hd, device="cuda")
        xb2 = torch.empty(nh * hd, device="cuda")
        for _ in range(3):  # back-to-back decodes: PDL overlap between them
            gla_ctx.decode(qd, kc, vc, xb, nh, nkv, hd, pos)
        gla_ctx.rope_append(qd, kd, vd, kc, vc, nh, nkv, hd, ph, 500000.0)
        gla_ctx.decode(qd, kc, vc, xb, nh, nkv, hd, pos + 1)
        # the device-position path right behind a decode (PDL overlap), as a
        # layer plan issues it: position holder = pos, rows 0..pos
        gla_ctx.process_heads_flash_attention(qd, kc, vc, xb2, nh, hd, nkv * hd, nh // nkv, ph,
                                              0, T)
        assert gla_ctx.device_status() == 0
        outs.append(xb.cpu().numpy())
        outs_dev.append(xb2.cpu().numpy())
        kk, vv, qq = kc.cpu().numpy(), vc.cpu().numpy(), qd.cpu().numpy()
        ref = oracle.decode_f32(qq, kk, vv, nh, nkv, hd, pos + 1)
        assert_close(outs[-1], ref, TOL_F32, f"option {opt}")
        assert_close(outs_dev[-1], ref, TOL_F32, f"option {opt}, device position")
        assert np.abs(kk[pos]).max() < 7.0 and vv[pos][0] == vnew[0]
    gla_ctx.set_option(gla.OPT_EARLY_KV_PREFETCH, 2)
    np.testing.assert_array_equal(outs[0], outs[1])
    np.testing.assert_array_equal(outs[0], outs[2])
    np.testing.assert_array_equal(outs_dev[0], outs_dev[2])


@pytest.mark.parametrize("style,hd,nh,nkv", [(0, 128, 24, 8), (1, 96, 32, 32), (0, 64, 32, 8),
                                             (1, 128, 28, 4)])
def test_fused_rope_append_attention_equals_separate_calls(gla_ctx, style, hd, nh, nkv):
    """gla_rope_append_attention_f32 = gla_rope_append_f32 followed by
    gla_process_heads_flash_attention, bit for bit: the output, the written
    cache row (and nothing else), and the caller's q left unrotated.  Run
    behind back-to-back decodes so its early history reads overlap them."""
    import gpullama_attn as gla

    torch = _torch()
    n_layers, ctxlen, pos, layer, theta = 2, 700, 515, 1, 500000.0
    kvd = nkv * hd
    rng = np.random.Generator(np.random.PCG64(77 + hd + style))
    kc0 = rng.standard_normal((n_layers, ctxlen, kvd), dtype=np.float32)
    vc0 = rng.standard_normal((n_layers, ctxlen, kvd), dtype=np.float32)
    q0 = rng.standard_normal(nh * hd, dtype=np.float32)
    k0 = rng.standard_normal(kvd, dtype=np.float32)
    v0 = rng.standard_normal(kvd, dtype=np.float32)
    ph = torch.tensor([pos], dtype=torch.int32, device="cuda")
    kc1, vc1, q1, k1, v1 = dev(kc0), dev(vc0), dev(q0), dev(k0), dev(v0)
    xb1 = torch.empty(nh * hd, device="cuda")
    gla_ctx.rope_append(q1, k1, v1, kc1[layer], vc1[layer], nh, nkv, hd, ph, theta, style)
    gla_ctx.process_heads_flash_attention(q1, kc1, vc1, xb1, nh, hd, kvd, nh // nkv, ph, layer,
                                          ctxlen)
    # every early-prefetch level: 2 patches the newest row into the tile
    # copied early, 0 and 1 (position on the device) append it to the cache
    # and copy the tile after the wait
    try:
        for opt in (2, 1, 0):
            gla_ctx.set_option(gla.OPT_EARLY_KV_PREFETCH, opt)
            kc2, vc2, q2, k2, v2 = dev(kc0), dev(vc0), dev(q0), dev(k0), dev(v0)
            xb2 = torch.empty(nh * hd, device="cuda")
            scratch = torch.empty(nh * hd, device="cuda")
            for _ in range(3):  # decodes that release their dependents early
                gla_ctx.decode(q2, kc2[0], vc2[0], scratch, nh, nkv, hd, ctxlen)
            gla_ctx.rope_append_attention(q2, k2, v2, kc2, vc2, xb2, nh, hd, kvd, nh // nkv, ph,
                                          layer, ctxlen, theta, style)
            assert gla_ctx.device_status() == 0
            np.testing.assert_array_equal(xb2.cpu().numpy(), xb1.cpu().numpy())
            np.testing.assert_array_equal(kc2.cpu().numpy(), kc1.cpu().numpy())
            np.testing.assert_array_equal(vc2.cpu().numpy(), vc1.cpu().numpy())
            np.testing.assert_array_equal(q2.cpu().numpy(), q0)
            changed = np.argwhere(np.any(kc2.cpu().numpy() != kc0, axis=-1))
            assert changed.tolist() == [[layer, pos]]
    finally:
        gla_ctx.set_option(gla.OPT_EARLY_KV_PREFETCH, 2)
    with pytest.raises(gla.GlaError):
        gla_ctx.rope_append_attention(q2, k2, v2, kc2, vc2, xb2, nh, hd, kvd, nh // nkv, ph,
                                      layer, ctxlen, theta, 7)


def _foreign_pdl_case(gla_ctx, oracle, delta, fused):
    import gpullama_attn as gla

    torch = _torch()
    nh, nkv, hd, ctxlen = 24, 8, 128, 2048
    pos0 = 700
    q0, k, v = inputs.decode_case(61 + delta, nh, nkv, hd, ctxlen)
    rng = np.random.Generator(np.random.PCG64(62))
    knew = rng.standard_normal(nkv * hd, dtype=np.float32)
    vnew = rng.standard_normal(nkv * hd, dtype=np.float32)
    kc, vc = dev(k), dev(v)
    qd, kd, vd = dev(q0), dev(knew), dev(vnew)
    ph = torch.tensor([pos0], dtype=torch.int32, device="cuda")
    xb = torch.empty(nh * hd, device="cuda")
    scratch = torch.empty(nh * hd, device="cuda")
    assert gla_ctx.device_status() == 0
    for _ in range(3):  # decodes that release their dependents early, ahead of it
        gla_ctx.decode(qd, kc, vc, scratch, nh, nkv, hd, pos0 + 1)
    gla_ctx.debug_advance_position(ph, delta, delay_us=30)
    if fused:
        gla_ctx.rope_append_attention(qd, kd, vd, kc, vc, xb, nh, hd, nkv * hd, nh // nkv, ph, 0,
                                      ctxlen, 500000.0)
    else:
        gla_ctx.process_heads_flash_attention(qd, kc, vc, xb, nh, hd, nkv * hd, nh // nkv, ph, 0,
                                              ctxlen)
    assert gla_ctx.device_status() == 0
    assert int(ph.item()) == pos0 + delta
    pos = pos0 + delta
    kk, vv = kc.cpu().numpy(), vc.cpu().numpy()
    if fused:
        # the reference: RoPE of q and the new key at `pos`, append, attend
        cr, ci = oracle.rope_freqs(ctxlen, hd, 500000.0)
        qq, kn = q0.copy(), knew.copy()
        oracle.rope_interleaved(qq, kn, hd, pos, cr, ci)
        np.testing.assert_allclose(kk[pos], kn, rtol=0, atol=2e-6)
        np.testing.assert_array_equal(vv[pos], vnew)
    else:
        qq = q0
    ref = oracle.decode_f32(qq, kk, vv, nh, nkv, hd, pos + 1)
    assert_close(xb.cpu().numpy(), ref, TOL_F32, f"delta {delta}, fused {fused}")


@pytest.mark.parametrize("fused", [False, True], ids=["task", "fused-rope"])
@pytest.mark.parametrize("delta", [1, 64, 300])
def test_decode_after_foreign_pdl_position_update(gla_ctx, oracle, delta, fused):
    import gpullama_attn as gla

    gla_ctx.set_option(gla.OPT_EARLY_KV_PREFETCH, 2)  # the default level
    _foreign_pdl_case(gla_ctx, oracle, delta, fused)


def test_phase_trace_option(gla_ctx):
    """GLA_OPT_TRACE: every CTA of the last decode launch leaves ordered
    %globaltimer stamps; the tiles it reports add up to the launch's tiles
    (C2 layer shape: 8 kv heads x 64 tiles) and, with more than one CTA per
    kv head holding a piece, the last G CTAs of a kv head to finish merge it
    (one q head each: 8 kv heads x 3)."""
    import gpullama_attn as gla

    torch = _torch()
    nh, nkv, hd, n = 24, 8, 128, 4096
    q, k, v = inputs.decode_case(5, nh, nkv, hd, n)
    qd, kd, vd = dev(q), dev(k), dev(v)
    xb = torch.empty(nh * hd, device="cuda")
    gla_ctx.set_option(gla.OPT_TRACE, 1)
    try:
        gla_ctx.decode(qd, kd, vd, xb, nh, nkv, hd, n)
        tr = gla_ctx.debug_trace()
    finally:
        gla_ctx.set_option(gla.OPT_TRACE, 0)
    assert gla_ctx.device_status() == 0
    ctas = gla_ctx.num_sms()
    tr = tr[:ctas]
    info = tr[:, 10]
    tiles = (info & 0xFFFF).astype(np.int64)
    merger = (info >> 24) & 0xFF
    assert int(tiles.sum()) == nkv * (n // 64)
    assert int(merger.sum()) == nkv * (nh // nkv)
    work = tiles > 0
    for col_a, col_b in ((0, 1), (1, 2), (2, 3), (3, 4), (4, 5), (5, 11)):
        assert np.all(tr[work, col_a] <= tr[work, col_b]), (col_a, col_b)
    assert np.all(tr[merger == 1, 5] <= tr[merger == 1, 6])
