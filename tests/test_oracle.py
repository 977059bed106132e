"""CPU oracle: known answers, float64 agreement, golden fixtures, RoPE."""
import os

import numpy as np
import pytest

import inputs
import reference64

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "attention_golden.npz")


def test_kat_uniform_scores_give_mean_of_v(oracle):
    # q = 0 -> every score is 0 -> softmax is uniform -> xb = mean of V rows
    nh, nkv, hd, n = 8, 2, 64, 37
    _, k, v = inputs.decode_case(7, nh, nkv, hd, n)
    q = np.zeros(nh * hd, dtype=np.float32)
    xb = oracle.decode_f32(q, k, v, nh, nkv, hd, n).reshape(nh, hd)
    vm = v.reshape(n, nkv, hd).astype(np.float64).mean(axis=0)
    for h in range(nh):
        np.testing.assert_allclose(xb[h], vm[h // (nh // nkv)], rtol=0, atol=2e-6)


def test_kat_single_row_returns_that_row(oracle):
    nh, nkv, hd = 6, 3, 128
    q, k, v = inputs.decode_case(8, nh, nkv, hd, 1)
    xb = oracle.decode_f32(q, k, v, nh, nkv, hd, 1).reshape(nh, hd)
    for h in range(nh):
        np.testing.assert_array_equal(xb[h], v[0].reshape(nkv, hd)[h // 2])


@pytest.mark.parametrize("nh,nkv,hd,n", [(8, 2, 64, 40), (14, 2, 128, 300), (4, 4, 96, 17),
                                         (32, 8, 64, 512), (24, 8, 128, 1000)])
def test_oracle_matches_float64(oracle, nh, nkv, hd, n):
    q, k, v = inputs.decode_case(n + hd, nh, nkv, hd, n)
    xb = oracle.decode_f32(q, k, v, nh, nkv, hd, n)
    ref = reference64.decode64(q, k, v, nh, nkv, hd, n)
    np.testing.assert_allclose(xb, ref, rtol=0, atol=2e-5)


def test_oracle_independent_of_thread_count(oracle):
    q, k, v = inputs.decode_case(3, 16, 4, 128, 200)
    a = oracle.decode_f32(q, k, v, 16, 4, 128, 200, n_threads=1)
    b = oracle.decode_f32(q, k, v, 16, 4, 128, 200, n_threads=5)
    np.testing.assert_array_equal(a, b)


def test_oracle_kv_stride(oracle):
    # a padded row stride reads the same rows as the packed layout
    nh, nkv, hd, n = 8, 2, 64, 20
    q, k, v = inputs.decode_case(4, nh, nkv, hd, n, kv_stride=160)
    a = oracle.decode_f32(q, k, v, nh, nkv, hd, n, kv_stride=160)
    kp = np.ascontiguousarray(k[:, : nkv * hd])
    vp = np.ascontiguousarray(v[:, : nkv * hd])
    b = oracle.decode_f32(q, kp, vp, nh, nkv, hd, n)
    np.testing.assert_array_equal(a, b)


def test_half_to_float_matches_numpy(oracle):
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    got = oracle.half_to_float(bits)
    want = bits.view(np.float16).astype(np.float32)
    finite = np.isfinite(want)
    np.testing.assert_array_equal(got[finite], want[finite])
    assert np.all(np.isnan(got[np.isnan(want)]))
    np.testing.assert_array_equal(got[np.isinf(want)], want[np.isinf(want)])


def test_f16_oracle_is_f32_oracle_on_decoded_values(oracle):
    nh, nkv, hd, n = 8, 2, 128, 64
    q, k, v = inputs.decode_case(9, nh, nkv, hd, n)
    k16, v16 = inputs.to_f16_bits(k), inputs.to_f16_bits(v)
    a = oracle.decode_f16(q, k16, v16, nh, nkv, hd, n)
    b = oracle.decode_f32(q, k16.view(np.float16).astype(np.float32),
                          v16.view(np.float16).astype(np.float32), nh, nkv, hd, n)
    np.testing.assert_array_equal(a, b)


def test_golden_fixtures_reproduce(oracle):
    g = np.load(GOLDEN)
    names = sorted({k.split("/")[0] for k in g.files if k.endswith("/xb")})
    assert len(names) >= 6
    for name in names:
        seed, nh, nkv, hd, npos, f16 = (int(x) for x in g[f"{name}/meta"])
        if f"{name}/q" in g.files:
            q, k, v = g[f"{name}/q"], g[f"{name}/k"], g[f"{name}/v"]
        else:
            q, k, v = inputs.decode_case(seed, nh, nkv, hd, npos)
            if f16:
                k, v = inputs.to_f16_bits(k), inputs.to_f16_bits(v)
            import hashlib

            h = hashlib.sha256()
            for a in (q, k, v):
                h.update(np.ascontiguousarray(a).tobytes())
            assert h.hexdigest() == str(g[f"{name}/sha256"]), f"{name}: input generator drifted"
        if f16:
            xb = oracle.decode_f16(q, k, v, nh, nkv, hd, npos)
        else:
            xb = oracle.decode_f32(q, k, v, nh, nkv, hd, npos)
        np.testing.assert_array_equal(xb, g[f"{name}/xb"], err_msg=name)


def test_rope_golden_and_float64(oracle):
    g = np.load(GOLDEN)
    for name in ("rope_llama3_theta5e5_pos123", "rope_neox_theta1e6_pos77"):
        seed, nh, nkv, hd, pos, style = (int(x) for x in g[f"{name}/meta"])
        theta = float(g[f"{name}/theta"])
        cr, ci = oracle.rope_freqs(pos + 1, hd, theta)
        q, k = g[f"{name}/q_in"].copy(), g[f"{name}/k_in"].copy()
        if style == 0:
            oracle.rope_interleaved(q, k, hd, pos, cr, ci)
        else:
            oracle.rope_neox(q, k, nh, nkv, hd, pos, cr, ci)
        np.testing.assert_array_equal(q, g[f"{name}/q_out"])
        np.testing.assert_array_equal(k, g[f"{name}/k_out"])
        # float64 restatement of the rotation
        i = np.arange(hd // 2)
        freq = (1.0 / theta ** (2 * i / hd)).astype(np.float32).astype(np.float64)
        ang = np.float32(pos) * freq.astype(np.float32)
        c, s = np.cos(ang.astype(np.float64)), np.sin(ang.astype(np.float64))
        q0 = g[f"{name}/q_in"].astype(np.float64).reshape(nh, hd)
        if style == 0:
            a, b = q0[:, 0::2], q0[:, 1::2]
        else:
            a, b = q0[:, : hd // 2], q0[:, hd // 2:]
        ra, rb = a * c - b * s, a * s + b * c
        qo = g[f"{name}/q_out"].reshape(nh, hd)
        got_a, got_b = (qo[:, 0::2], qo[:, 1::2]) if style == 0 else (qo[:, : hd // 2], qo[:, hd // 2:])
        np.testing.assert_allclose(got_a, ra, atol=1e-5)
        np.testing.assert_allclose(got_b, rb, atol=1e-5)


def test_prefill_oracle_is_decode_per_row(oracle):
    L, nh, nkv, hd = 12, 4, 2, 64
    rng = np.random.Generator(np.random.PCG64(5))
    q = rng.standard_normal((L, nh * hd), dtype=np.float32)
    k = rng.standard_normal((L, nkv * hd), dtype=np.float32)
    v = rng.standard_normal((L, nkv * hd), dtype=np.float32)
    out = oracle.prefill_causal_f32(q, k, v, L, nh, nkv, hd)
    for p in (0, 5, L - 1):
        xb = oracle.decode_f32(q[p], k, v, nh, nkv, hd, p + 1)
        np.testing.assert_array_equal(out[p], xb)


def test_wo_residual_oracle_known_answers_and_float64(oracle):
    """matrixVectorGenericWithResidual restatement: identity weights add xb to
    the residual exactly; random weights agree with float64 to FP32 rounding;
    the 32-lane tree order is what makes it differ from a plain loop."""
    n = d = 64
    eye = np.eye(d, n, dtype=np.float16)
    xb = np.arange(n, dtype=np.float32) * 0.5
    x = np.ones(d, dtype=np.float32)
    np.testing.assert_array_equal(oracle.wo_residual_f16(xb, x, eye, n, d), x + xb)
    rng = np.random.Generator(np.random.PCG64(9))
    for n, d in ((3072, 40), (8, 3), (4104, 5)):
        w = (rng.standard_normal((d, n), dtype=np.float32) * 0.05).astype(np.float16)
        xb = rng.standard_normal(n, dtype=np.float32)
        x = rng.standard_normal(d, dtype=np.float32)
        got = oracle.wo_residual_f16(xb, x, w, n, d)
        w64 = w.astype(np.float64)
        exact = x + w64 @ xb.astype(np.float64)
        scale = np.abs(x) + np.abs(w64) @ np.abs(xb.astype(np.float64))
        assert (np.abs(got - exact) <= 4e-6 * scale).all()
    # a one-lane workgroup is a plain sequential FP32 dot product per row
    n, d = 40, 3
    w = (rng.standard_normal((d, n), dtype=np.float32) * 0.05).astype(np.float16)
    xb = rng.standard_normal(n, dtype=np.float32)
    x = rng.standard_normal(d, dtype=np.float32)
    plain = np.empty(d, dtype=np.float32)
    for i in range(d):
        acc = np.float32(0.0)
        for j in range(n):
            acc = np.float32(acc + np.float32(np.float32(w[i, j]) * xb[j]))
        plain[i] = np.float32(x[i] + acc)
    np.testing.assert_array_equal(oracle.wo_residual_f16(xb, x, w, n, d, local_size=1), plain)


def test_float_to_half_and_q8_quantiser(oracle):
    """The oracle's FP16 rounding equals numpy's (round to nearest even, edge
    cases included), and its Q8_0 quantiser equals a numpy restatement of
    GGML's: d = amax/127, q = round-half-away(x * (1/d)), d stored as FP16;
    dequantised values are within half a step of the input."""
    rng = np.random.Generator(np.random.PCG64(4))
    x = np.concatenate([rng.standard_normal(20000, dtype=np.float32) * s
                        for s in (1e-8, 1e-5, 1e-3, 1.0, 1e2, 1e4, 6e4)])
    x = np.concatenate([x, np.array([65504, 65519.99, 65520, -65520, 5.96e-8, 2.98e-8, 2.99e-8,
                                     0.0, -0.0, np.inf, -np.inf], dtype=np.float32)])
    with np.errstate(over="ignore"):
        np.testing.assert_array_equal(oracle.float_to_half(x), x.astype(np.float16).view(np.uint16))
    n_kv, hd, rows = 3, 128, 40
    k = rng.standard_normal((rows, n_kv * hd), dtype=np.float32) * 2
    v = rng.standard_normal((rows, n_kv * hd), dtype=np.float32)
    k[0, :32] = 0.0
    kq, vq, sc = oracle.quantize_q8(k, v, n_kv, hd)
    for src, q, lo in ((k, kq, 0), (v, vq, 4)):
        b = src.reshape(rows, n_kv, 4, 32)
        amax = np.abs(b).max(axis=3)
        d = (amax / np.float32(127)).astype(np.float32)
        inv = np.where(d != 0, np.float32(1) / np.where(d != 0, d, 1), 0).astype(np.float32)
        y = (b * inv[..., None]).astype(np.float32)
        qn = np.where(y >= 0, np.floor(y + 0.5), -np.floor(-y + 0.5)).astype(np.int8)
        np.testing.assert_array_equal(q.reshape(rows, n_kv, 4, 32), qn)
        np.testing.assert_array_equal(sc[:, :, lo:lo + 4], d.astype(np.float16).view(np.uint16))
    assert (sc[0, 0, 0] == 0) and (kq[0, :32] == 0).all()
    kd, vd = oracle.dequantize_q8(kq, vq, sc, n_kv, hd)
    step = oracle.half_to_float(sc[:, :, :4]).repeat(32, axis=2).reshape(rows, n_kv * hd)
    # half a step, plus 127 times the FP16 rounding of the step (<= 2^-11 of it)
    assert (np.abs(kd - k) <= (0.5 + 127 * 2.0 ** -11) * step * (1 + 1e-6) + 1e-30).all()
