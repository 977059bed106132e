"""KV caches allocated by the library (gla_kv_cache_alloc, the device
counterpart of the State caches: inference/state/State.java:41-42,56-58 and
LlamaState.java:45-46,61-64 allocate [layer][contextLength][kvDim] FP32
arrays), filled by the library's own producers and decoded against the
oracle - the per-token flow of InferenceCore.forwardJava (RoPE :82-94, KV
append :99-100, attention :105-144) and prompt ingestion
(InferenceEngine.java:88-99)."""
import numpy as np
import pytest

import inputs

pytestmark = pytest.mark.gpu

TOL_F32 = 1e-3
TOL_F16 = 5e-3


def _close(got, ref, tol, what):
    err = float(np.abs(np.asarray(got, np.float64) - np.asarray(ref, np.float64)).max())
    scale = max(float(np.abs(ref).max()), 1e-30)
    assert err <= tol and err / scale <= tol, f"{what}: max abs err {err:.3e}"


def test_fp32_state_token_by_token(gla_ctx, oracle):
    """Llama layout: n_layers caches from gla_kv_cache_alloc (zeroed), then
    token by token and layer by layer the fused RoPE + append + attention
    task at the device position; every token's output against the oracle on
    a host replica built with the oracle's RoPE."""
    import torch

    import gpullama_attn as gla

    n_layers, ctxlen, nh, nkv, hd, theta = 2, 96, 8, 2, 64, 500000.0
    kvd = nkv * hd
    kp, vp = gla_ctx.kv_cache_alloc(n_layers, ctxlen, kvd, gla.DTYPE_F32)
    try:
        kc = gla.device_view(kp, (n_layers, ctxlen, kvd), torch.float32)
        vc = gla.device_view(vp, (n_layers, ctxlen, kvd), torch.float32)
        torch.cuda.synchronize()
        assert float(kc.abs().sum()) == 0.0 and float(vc.abs().sum()) == 0.0
        cr, ci = oracle.rope_freqs(ctxlen, hd, theta)
        hk = np.zeros((n_layers, ctxlen, kvd), np.float32)
        hv = np.zeros((n_layers, ctxlen, kvd), np.float32)
        ph = torch.zeros(1, dtype=torch.int32, device="cuda")
        rng = np.random.Generator(np.random.PCG64(17))
        for t in range(0, 70):
            ph.fill_(t)
            for layer in range(n_layers):
                q = rng.standard_normal(nh * hd, dtype=np.float32)
                k = rng.standard_normal(kvd, dtype=np.float32)
                v = rng.standard_normal(kvd, dtype=np.float32)
                xb = torch.empty(nh * hd, device="cuda")
                gla_ctx.rope_append_attention(torch.from_numpy(q).cuda(),
                                              torch.from_numpy(k).cuda(),
                                              torch.from_numpy(v).cuda(), kp, vp, xb, nh, hd,
                                              kvd, nh // nkv, ph, layer, ctxlen, theta)
                qr, kr = q.copy(), k.copy()
                oracle.rope_interleaved(qr, kr, hd, t, cr, ci)
                hk[layer, t], hv[layer, t] = kr, v
                if t in (0, 1, 63, 64, 69):
                    assert gla_ctx.device_status() == 0
                    ref = oracle.decode_f32(qr, hk[layer], hv[layer], nh, nkv, hd, t + 1)
                    _close(xb.cpu().numpy(), ref, TOL_F32, f"token {t} layer {layer}")
        assert gla_ctx.device_status() == 0
        np.testing.assert_allclose(kc.cpu().numpy(), hk, rtol=0, atol=2e-6)
        np.testing.assert_array_equal(vc.cpu().numpy(), hv)
    finally:
        gla_ctx.kv_cache_free(kp, vp)


def test_fp16_state_prompt_then_decode(gla_ctx, oracle):
    """FP16 caches from gla_kv_cache_alloc: a prompt ingested in two chunks
    (gla_ingest_prompt_f16kv), then the reference task over the cache at the
    last prompt position; the task's output against the oracle on the cache
    the library wrote (read back through a device view)."""
    import torch

    import gpullama_attn as gla

    n_layers, ctxlen, nh, nkv, hd, theta = 3, 512, 28, 4, 128, 1000000.0
    kvd = nkv * hd
    P, layer = 300, 2
    kp, vp = gla_ctx.kv_cache_alloc(n_layers, ctxlen, kvd, gla.DTYPE_F16)
    try:
        kc = gla.device_view(kp, (n_layers, ctxlen, kvd), torch.float16)
        vc = gla.device_view(vp, (n_layers, ctxlen, kvd), torch.float16)
        rng = np.random.Generator(np.random.PCG64(23))
        q = torch.from_numpy(rng.standard_normal((P, nh * hd), dtype=np.float32)).cuda()
        k = torch.from_numpy(rng.standard_normal((P, kvd), dtype=np.float32)).cuda()
        v = torch.from_numpy(rng.standard_normal((P, kvd), dtype=np.float32)).cuda()
        out = torch.empty(P, nh * hd, device="cuda")
        for lo, hi in ((0, 200), (200, P)):
            gla_ctx.ingest_prompt(q[lo:hi], k[lo:hi], v[lo:hi], kc[layer], vc[layer], out[lo:hi],
                                  lo, hi - lo, nh, nkv, hd, ctxlen, theta, gla.ROPE_NEOX,
                                  f16_cache=True)
        assert gla_ctx.device_status() == 0
        k16 = kc[layer, :P].view(torch.int16).cpu().numpy().view(np.uint16)
        v16 = vc[layer, :P].view(torch.int16).cpu().numpy().view(np.uint16)
        assert np.all(kc[layer, P:].cpu().numpy() == 0) and np.all(kc[0].cpu().numpy() == 0)
        # the ingested prompt's last row, as prefill computed it
        cr, ci = oracle.rope_freqs(ctxlen, hd, theta)
        q_last = q[P - 1].cpu().numpy().copy()
        k_dummy = np.zeros(kvd, np.float32)
        oracle.rope_neox(q_last, k_dummy, nh, nkv, hd, P - 1, cr, ci)
        ref = oracle.decode_f16(q_last, k16, v16, nh, nkv, hd, P)
        _close(out[P - 1].cpu().numpy(), ref, TOL_F16, "ingested last row")
        # the reference task over the library cache at position P - 1
        ph = torch.tensor([P - 1], dtype=torch.int32, device="cuda")
        xb = torch.empty(nh * hd, device="cuda")
        qd = torch.from_numpy(q_last).cuda()
        gla_ctx.process_heads_flash_attention(qd, kp, vp, xb, nh, hd, kvd, nh // nkv, ph, layer,
                                              ctxlen, f16_cache=True)
        assert gla_ctx.device_status() == 0
        _close(xb.cpu().numpy(), ref, TOL_F16, "task over the ingested cache")
    finally:
        gla_ctx.kv_cache_free(kp, vp)
