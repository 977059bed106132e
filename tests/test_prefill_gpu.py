"""Causal prefill (tcgen05/TMEM) through the C ABI against the oracle.

The oracle is the reference's prompt ingestion: decode attention at every
position p over rows 0..p (InferenceEngine.java:88-99), in FP32 on the
FP16-rounded q/k/v.  Tolerance 5e-3 (max |err| and max |err| / max |ref|),
the FP16 bound of the north star.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 5e-3


def _case(seed, L, nh, nkv, hd):
    rng = np.random.Generator(np.random.PCG64(seed))
    q = rng.standard_normal((L, nh * hd), dtype=np.float32).astype(np.float16)
    k = rng.standard_normal((L, nkv * hd), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((L, nkv * hd), dtype=np.float32).astype(np.float16)
    return q, k, v


def _run(ctx, q, k, v, L, nh, nkv, hd):
    import torch

    qd = torch.from_numpy(q.view(np.int16)).cuda()
    kd = torch.from_numpy(k.view(np.int16)).cuda()
    vd = torch.from_numpy(v.view(np.int16)).cuda()
    out = torch.full((L, nh * hd), float("nan"), device="cuda")
    ctx.prefill_causal(qd, kd, vd, out, L, nh, nkv, hd)
    assert ctx.device_status() == 0
    return out.cpu().numpy()


def _check(got, ref, what):
    err = np.abs(got.astype(np.float64) - ref).max()
    scale = np.abs(ref).max()
    assert err <= TOL and err / scale <= TOL, f"{what}: max abs err {err:.3e} rel {err / scale:.3e}"


@pytest.mark.parametrize("L,nh,nkv,hd", [
    (1, 2, 2, 96), (7, 2, 1, 64), (128, 2, 2, 96), (129, 2, 2, 96), (300, 4, 2, 128),
    (512, 2, 2, 64), (256, 3, 3, 96),
])
def test_prefill_matches_oracle(gla_ctx, oracle, L, nh, nkv, hd):
    q, k, v = _case(L + hd + nh, L, nh, nkv, hd)
    got = _run(gla_ctx, q, k, v, L, nh, nkv, hd)
    ref = oracle.prefill_causal_f32(q.astype(np.float32), k.astype(np.float32),
                                    v.astype(np.float32), L, nh, nkv, hd)
    assert np.isfinite(got).all()
    _check(got, ref, f"L={L} nh={nh} nkv={nkv} hd={hd}")


def test_prefill_c5_phi3_shape_sampled_rows(gla_ctx, oracle):
    # MHA 32 heads, hd 96, prompt 4096; rows checked
    # against the per-position oracle (every row would take minutes on CPU)
    L, nh, nkv, hd = 4096, 32, 32, 96
    q, k, v = _case(5, L, nh, nkv, hd)
    got = _run(gla_ctx, q, k, v, L, nh, nkv, hd)
    assert np.isfinite(got).all()
    kf, vf = k.astype(np.float32), v.astype(np.float32)
    for p in (0, 1, 127, 128, 129, 1000, 2047, 4095):
        ref = oracle.decode_f32(q[p].astype(np.float32), kf, vf, nh, nkv, hd, p + 1)
        _check(got[p], ref, f"row {p}")


def test_prefill_row_equals_decode_kernel(gla_ctx):
    """Property: prefill row p equals decode attention at position p (FP16 cache)."""
    import torch

    L, nh, nkv, hd = 640, 4, 2, 128
    q, k, v = _case(17, L, nh, nkv, hd)
    got = _run(gla_ctx, q, k, v, L, nh, nkv, hd)
    kd = torch.from_numpy(k.view(np.int16)).cuda()
    vd = torch.from_numpy(v.view(np.int16)).cuda()
    xb = torch.empty(nh * hd, device="cuda")
    for p in (0, 63, 64, 255, 639):
        qp = torch.from_numpy(q[p].astype(np.float32)).cuda()
        gla_ctx.decode(qp, kd, vd, xb, nh, nkv, hd, p + 1, f16_cache=True)
        _check(got[p], xb.cpu().numpy().astype(np.float64), f"row {p}")
