"""Batched prompt ingestion (gla_ingest_prompt_f32 / _f16kv) through the C ABI.

The oracle is the reference's ingestion loop run position by position
(InferenceEngine.java:88-99): RoPE of q and k (InferenceCore.java:82-94 or
:210-225), the k/v row appended to the cache (:99-100), then the attention
block over rows 0..p (:105-144), all in FP32.  The product computes attention
on tensor cores with FP16 operands, so the tolerance is the FP16 bound 5e-3
(max |err| and max |err| / max |ref|).  The rotated k rows in the cache are
checked like the single-position RoPE kernel (atol 2e-6: the GPU's double
cos/sin against the C library's; FP16 caches within half an FP16 ulp more).
"""
import numpy as np
import pytest

import gpullama_attn as gla

pytestmark = pytest.mark.gpu

TOL = 5e-3
SENTINEL = 7.0


def _torch():
    import torch

    return torch


def _inputs(seed, total, nh, nkv, hd):
    rng = np.random.Generator(np.random.PCG64(seed))
    q = rng.standard_normal((total, nh * hd), dtype=np.float32)
    k = rng.standard_normal((total, nkv * hd), dtype=np.float32)
    v = rng.standard_normal((total, nkv * hd), dtype=np.float32)
    return q, k, v


def _oracle_ingest(oracle, q, k, v, nh, nkv, hd, ctx_len, theta, style):
    """Sequential ingestion on the CPU: rotated q/k, caches and xb per position."""
    total = q.shape[0]
    cr, ci = oracle.rope_freqs(ctx_len, hd, theta)
    qr, kr = q.copy(), k.copy()
    kc = np.zeros((ctx_len, nkv * hd), np.float32)
    vc = np.zeros_like(kc)
    xb = np.zeros((total, nh * hd), np.float32)
    for p in range(total):
        if style == gla.ROPE_INTERLEAVED:
            oracle.rope_interleaved(qr[p], kr[p], hd, p, cr, ci)
        else:
            oracle.rope_neox(qr[p], kr[p], nh, nkv, hd, p, cr, ci)
        kc[p], vc[p] = kr[p], v[p]
        xb[p] = oracle.decode_f32(qr[p], kc, vc, nh, nkv, hd, p + 1)
    return qr, kr, xb


def _run_chunks(ctx, q, k, v, chunks, nh, nkv, hd, ctx_len, theta, style, f16):
    """Ingests the rows chunk by chunk; returns q and k as the call left them,
    the caches and xb (numpy)."""
    torch = _torch()
    total = q.shape[0]
    if f16:
        kc = torch.full((ctx_len, nkv * hd), SENTINEL, dtype=torch.float16, device="cuda")
    else:
        kc = torch.full((ctx_len, nkv * hd), SENTINEL, device="cuda")
    vc = torch.full_like(kc, SENTINEL)
    qo = np.zeros_like(q)
    ko = np.zeros_like(k)
    xb = np.full((total, nh * hd), np.nan, np.float32)
    for start, n in chunks:
        qd = torch.from_numpy(q[start:start + n].copy()).cuda()
        kd = torch.from_numpy(k[start:start + n].copy()).cuda()
        vd = torch.from_numpy(v[start:start + n].copy()).cuda()
        xd = torch.full((n, nh * hd), float("nan"), device="cuda")
        ctx.ingest_prompt(qd, kd, vd, kc, vc, xd, start, n, nh, nkv, hd, ctx_len, theta, style,
                          f16_cache=f16)
        qo[start:start + n] = qd.cpu().numpy()
        ko[start:start + n] = kd.cpu().numpy()
        xb[start:start + n] = xd.cpu().numpy()
    assert ctx.device_status() == 0
    return qo, ko, kc.float().cpu().numpy(), vc.float().cpu().numpy(), xb


def _check(got, ref, what):
    err = np.abs(got.astype(np.float64) - ref).max()
    scale = np.abs(ref).max()
    assert err <= TOL and err / scale <= TOL, f"{what}: max abs err {err:.3e} rel {err / scale:.3e}"


CASES = [
    # nh, nkv, hd, style, theta, chunks (start, rows), context length
    (8, 2, 128, gla.ROPE_INTERLEAVED, 500000.0, [(0, 200), (200, 1), (201, 180)], 400),
    (4, 4, 96, gla.ROPE_NEOX, 10000.0, [(0, 130), (130, 300)], 512),
    (6, 2, 64, gla.ROPE_NEOX, 1000000.0, [(0, 1), (1, 127), (128, 256)], 384),
    (2, 1, 64, gla.ROPE_INTERLEAVED, 10000.0, [(0, 7)], 7),
]


@pytest.mark.parametrize("f16", [False, True], ids=["f32kv", "f16kv"])
@pytest.mark.parametrize("case", range(len(CASES)))
def test_ingest_matches_sequential_oracle(gla_ctx, oracle, case, f16):
    nh, nkv, hd, style, theta, chunks, ctx_len = CASES[case]
    total = sum(n for _, n in chunks)
    q, k, v = _inputs(100 + case, total, nh, nkv, hd)
    qo, ko, kc, vc, xb = _run_chunks(gla_ctx, q, k, v, chunks, nh, nkv, hd, ctx_len, theta,
                                     style, f16)
    qr, kr, ref = _oracle_ingest(oracle, q, k, v, nh, nkv, hd, ctx_len, theta, style)
    np.testing.assert_array_equal(qo, q)  # inputs are read only
    np.testing.assert_array_equal(ko, k)
    if f16:
        bound = np.abs(kr) * 2.0 ** -11 + 2e-6
        assert (np.abs(kc[:total] - kr) <= bound).all()
        np.testing.assert_array_equal(vc[:total], v.astype(np.float16).astype(np.float32))
    else:
        np.testing.assert_allclose(kc[:total], kr, rtol=0, atol=2e-6)
        np.testing.assert_array_equal(vc[:total], v)
    assert (kc[total:] == SENTINEL).all() and (vc[total:] == SENTINEL).all()
    assert np.isfinite(xb).all()
    _check(xb, ref, f"case {case} f16={f16}")


def test_ingest_f32_and_f16_caches_give_identical_rows(gla_ctx):
    """Both variants feed the tensor cores the same FP16 operands: the FP16
    cache is the FP32 cache rounded, and xb is bit-identical."""
    nh, nkv, hd, style, theta, chunks, ctx_len = CASES[0]
    total = sum(n for _, n in chunks)
    q, k, v = _inputs(7, total, nh, nkv, hd)
    a = _run_chunks(gla_ctx, q, k, v, chunks, nh, nkv, hd, ctx_len, theta, style, False)
    b = _run_chunks(gla_ctx, q, k, v, chunks, nh, nkv, hd, ctx_len, theta, style, True)
    np.testing.assert_array_equal(a[2].astype(np.float16).astype(np.float32), b[2])
    np.testing.assert_array_equal(a[3].astype(np.float16).astype(np.float32), b[3])
    np.testing.assert_array_equal(a[4], b[4])


def test_ingest_chunked_equals_one_call_c5_shape(gla_ctx, oracle):
    """BASELINE config 5 shape (32 heads, hd 96, 4096 positions): ingesting in
    three chunks gives the same rows as one call (every row walks the same key
    blocks in the same order), and sampled rows match the sequential oracle."""
    nh, nkv, hd, L, theta = 32, 32, 96, 4096, 10000.0
    style = gla.ROPE_NEOX
    q, k, v = _inputs(5, L, nh, nkv, hd)
    one = _run_chunks(gla_ctx, q, k, v, [(0, L)], nh, nkv, hd, L, theta, style, True)
    three = _run_chunks(gla_ctx, q, k, v, [(0, 1000), (1000, 77), (1077, L - 1077)], nh, nkv, hd,
                        L, theta, style, True)
    for x, y in zip(one, three):
        np.testing.assert_array_equal(x, y)
    qo, ko, kc, vc, xb = one
    cr, ci = oracle.rope_freqs(L, hd, theta)
    kr = k.copy()
    qs = {}
    for p in range(L):  # rotate k rows (cheap) to build the FP32 cache
        qq = q[p].copy()
        oracle.rope_neox(qq, kr[p], nh, nkv, hd, p, cr, ci)
        qs[p] = qq
    for p in (0, 1, 127, 128, 999, 1000, 1076, 1077, 2047, 4095):
        ref = oracle.decode_f32(qs[p], kr, v, nh, nkv, hd, p + 1)
        _check(xb[p], ref, f"row {p}")


def test_ingest_then_decode_next_token(gla_ctx, oracle):
    """A prompt ingested in one call, then the next token decoded through the
    fused RoPE + append + attention call on the same FP32 cache."""
    torch = _torch()
    nh, nkv, hd, theta = 8, 2, 128, 500000.0
    style = gla.ROPE_INTERLEAVED
    L, ctx_len = 333, 400
    q, k, v = _inputs(21, L + 1, nh, nkv, hd)
    kc = torch.zeros((1, ctx_len, nkv * hd), device="cuda")  # layer 0 of a 1-layer cache
    vc = torch.zeros_like(kc)
    qd, kd, vd = (torch.from_numpy(x[:L].copy()).cuda() for x in (q, k, v))
    xd = torch.empty((L, nh * hd), device="cuda")
    gla_ctx.ingest_prompt(qd, kd, vd, kc, vc, xd, 0, L, nh, nkv, hd, ctx_len, theta, style)
    qn, kn, vn = (torch.from_numpy(x[L].copy()).cuda() for x in (q, k, v))
    xn = torch.empty(nh * hd, device="cuda")
    ph = torch.tensor([L], dtype=torch.int32, device="cuda")
    gla_ctx.rope_append_attention(qn, kn, vn, kc, vc, xn, nh, hd, nkv * hd, nh // nkv, ph, 0,
                                  ctx_len, theta, style)
    assert gla_ctx.device_status() == 0
    _, _, ref = _oracle_ingest(oracle, q, k, v, nh, nkv, hd, ctx_len, theta, style)
    got = xn.cpu().numpy()
    err = np.abs(got - ref[L]).max()
    assert err <= 1e-3 and err / np.abs(ref[L]).max() <= 1e-3, err  # FP32 decode bound
    _check(xd.cpu().numpy(), ref[:L], "prompt rows")


def test_ingest_rejects_bad_arguments(gla_ctx):
    torch = _torch()
    nh, nkv, hd = 2, 1, 64
    q = torch.zeros((4, nh * hd), device="cuda")
    k = torch.zeros((4, nkv * hd), device="cuda")
    kc = torch.zeros((8, nkv * hd), device="cuda")
    xb = torch.zeros_like(q)
    with pytest.raises(gla.GlaError):  # positions past the context
        gla_ctx.ingest_prompt(q, k, k, kc, kc.clone(), xb, 6, 4, nh, nkv, hd, 8, 1e4)
    with pytest.raises(gla.GlaError):  # unsupported head_dim
        gla_ctx.ingest_prompt(q, k, k, kc, kc.clone(), xb, 0, 2, 4, 1, 32, 8, 1e4)
    with pytest.raises(gla.GlaError):  # unknown rope style
        gla_ctx.ingest_prompt(q, k, k, kc, kc.clone(), xb, 0, 4, nh, nkv, hd, 8, 1e4, style=5)
    with pytest.raises(gla.GlaError):  # zero rows
        gla_ctx.ingest_prompt(q, k, k, kc, kc.clone(), xb, 0, 0, nh, nkv, hd, 8, 1e4)
