"""Output projection + residual (gla_wo_residual_f16) through the C ABI.

The oracle restates the reference's GPU task matrixVectorGenericWithResidual
(TransformerComputeKernelsLayered.java:715-733) with its 32-lane strided sums
and tree reduction.  The kernel sums in another order, so results are checked
against the exact (float64) value with an FP32 rounding bound,
|err| <= 4e-6 * (|x_i| + sum_j |w_ij xb_j|), which the oracle meets too.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL = 4e-6


def _torch():
    import torch

    return torch


def _case(seed, n, d):
    rng = np.random.Generator(np.random.PCG64(seed))
    w = (rng.standard_normal((d, n), dtype=np.float32) * 0.05).astype(np.float16)
    xb = rng.standard_normal(n, dtype=np.float32)
    x = rng.standard_normal(d, dtype=np.float32)
    return w, xb, x


def _bound_check(got, w, xb, x, what):
    w64 = w.astype(np.float64)
    exact = x.astype(np.float64) + w64 @ xb.astype(np.float64)
    scale = np.abs(x) + np.abs(w64) @ np.abs(xb.astype(np.float64))
    err = np.abs(got.astype(np.float64) - exact)
    assert (err <= REL * scale).all(), f"{what}: worst {np.max(err / scale):.3e} of scale"


def _run(ctx, w, xb, x):
    torch = _torch()
    wd = torch.from_numpy(w.view(np.int16)).cuda()
    xbd = torch.from_numpy(xb).cuda()
    xd = torch.from_numpy(x.copy()).cuda()
    ctx.wo_residual(xbd, xd, wd, w.shape[1], w.shape[0])
    assert ctx.device_status() == 0
    return xd.cpu().numpy()


@pytest.mark.parametrize("n,d", [
    (3072, 3072),   # Llama-3.2-3B wo
    (2048, 2048),   # Llama-3.2-1B
    (4096, 4096),   # Llama-3.1-8B
    (8, 1),         # smallest
    (5120, 100),    # two row passes (640 chunks > 512 a pass)
    (4104, 33),     # second pass of one chunk
    (3072, 1),
])
def test_wo_residual_matches_oracle(gla_ctx, oracle, n, d):
    w, xb, x = _case(n + d, n, d)
    got = _run(gla_ctx, w, xb, x)
    ref = oracle.wo_residual_f16(xb, x, w, n, d)
    _bound_check(ref, w, xb, x, "oracle")
    _bound_check(got, w, xb, x, f"n={n} d={d}")


def test_wo_residual_accumulates(gla_ctx):
    """Two calls add the projection twice (x is read and written in place)."""
    torch = _torch()
    n, d = 1024, 300
    w, xb, x = _case(3, n, d)
    wd = torch.from_numpy(w.view(np.int16)).cuda()
    xbd = torch.from_numpy(xb).cuda()
    xd = torch.from_numpy(x.copy()).cuda()
    gla_ctx.wo_residual(xbd, xd, wd, n, d)
    once = xd.cpu().numpy()
    gla_ctx.wo_residual(xbd, xd, wd, n, d)
    twice = xd.cpu().numpy()
    proj = once.astype(np.float64) - x
    np.testing.assert_allclose(twice - once, proj, rtol=0, atol=1e-5)


def test_wo_after_attention_chain_equals_step_by_step(gla_ctx):
    """The projection launched right behind the attention call (programmatic
    dependent launch) must read the finished xb: a chain of layers issued
    back to back, and the same chain captured in a CUDA graph, equal the
    calls run one at a time with a synchronize between them, bit for bit."""
    import gpullama_attn as gla

    torch = _torch()
    nh, nkv, hd, ctx_len, layers, pos = 24, 8, 128, 1024, 6, 700
    dim, kvd = nh * hd, nkv * hd
    rng = np.random.Generator(np.random.PCG64(11))
    kc0 = rng.standard_normal((layers, ctx_len, kvd), dtype=np.float32)
    vc0 = rng.standard_normal((layers, ctx_len, kvd), dtype=np.float32)
    wo = [(rng.standard_normal((dim, dim), dtype=np.float32) * 0.02).astype(np.float16)
          for _ in range(layers)]
    q0 = rng.standard_normal((layers, dim), dtype=np.float32)
    k0 = rng.standard_normal((layers, kvd), dtype=np.float32)
    v0 = rng.standard_normal((layers, kvd), dtype=np.float32)
    x0 = rng.standard_normal(dim, dtype=np.float32)
    wod = [torch.from_numpy(w.view(np.int16)).cuda() for w in wo]
    ph = torch.tensor([pos], dtype=torch.int32, device="cuda")

    def fresh():
        return (torch.from_numpy(kc0.copy()).cuda(), torch.from_numpy(vc0.copy()).cuda(),
                torch.from_numpy(q0.copy()).cuda(), torch.from_numpy(k0.copy()).cuda(),
                torch.from_numpy(v0.copy()).cuda(), torch.from_numpy(x0.copy()).cuda(),
                torch.empty(dim, device="cuda"))

    def chain(bufs, sync):
        kc, vc, q, k, v, x, xb = bufs
        for l in range(layers):
            gla_ctx.rope_append_attention(q[l], k[l], v[l], kc, vc, xb, nh, hd, kvd, nh // nkv,
                                          ph, l, ctx_len, 500000.0, gla.ROPE_INTERLEAVED)
            if sync:
                torch.cuda.synchronize()
            gla_ctx.wo_residual(xb, x, wod[l], dim, dim)
            if sync:
                torch.cuda.synchronize()
        return x

    ref = chain(fresh(), True).cpu().numpy()
    got = chain(fresh(), False).cpu().numpy()
    np.testing.assert_array_equal(got, ref)
    # the same chain replayed from a CUDA graph on the context's stream
    stream = torch.cuda.Stream()
    gla_ctx.set_stream(stream.cuda_stream)
    try:
        bufs = fresh()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            chain(bufs, False)
        kc, vc, q, k, v, x, xb = bufs
        for _ in range(2):  # replays start from the initial state each time
            for dst, src in zip((kc, vc, q, k, v, x), (kc0, vc0, q0, k0, v0, x0)):
                dst.copy_(torch.from_numpy(src))
            torch.cuda.synchronize()
            g.replay()
            torch.cuda.synchronize()
            np.testing.assert_array_equal(x.cpu().numpy(), ref)
    finally:
        gla_ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    assert gla_ctx.device_status() == 0


def test_wo_rejects_bad_arguments(gla_ctx):
    import gpullama_attn as gla

    torch = _torch()
    w = torch.zeros((4, 64), dtype=torch.int16, device="cuda")
    xb = torch.zeros(64, device="cuda")
    x = torch.zeros(4, device="cuda")
    with pytest.raises(gla.GlaError):  # n not a multiple of 8
        gla_ctx.wo_residual(xb, x, w, 60, 4)
    with pytest.raises(gla.GlaError):  # w not 16-byte aligned
        gla_ctx.wo_residual(xb, x, w.view(-1)[1:], 56, 4)
    with pytest.raises(gla.GlaError):  # empty output
        gla_ctx.wo_residual(xb, x, w, 64, 0)
