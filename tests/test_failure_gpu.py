"""Failure detection on one GPU, without a GPU fault: the peer exchange's
bounded wait for another rank's records runs out and latches
GLA_ERR_TIMEOUT in the device status; the context stays usable.

The other rank is simulated in one process (gla_debug_xch_loopback): this
context plays rank 0 of a 2-rank exchange whose rank-1 buffer nobody writes,
so the wait has a flag that nothing sets.  The kernel gives up after its 1 s
bound (decode_kernel.cuh, publish_merge)."""
import time

import numpy as np
import pytest

import inputs

pytestmark = pytest.mark.gpu


def test_peer_wait_times_out_and_the_context_recovers(gla_ctx, oracle):
    import torch

    import gpullama_attn as gla

    nh, nkv, hd, n = 28, 4, 128, 3000
    q, k, v = inputs.decode_case(81, nh, nkv, hd, n)
    k16, v16 = inputs.to_f16_bits(k), inputs.to_f16_bits(v)
    qd = torch.from_numpy(q).cuda()
    kd = torch.from_numpy(k16.view(np.int16)).cuda()
    vd = torch.from_numpy(v16.view(np.int16)).cuda()
    xb = torch.empty(nh * hd, device="cuda")
    assert gla_ctx.device_status() == 0
    gla_ctx.debug_xch_loopback(2)
    try:
        assert gla_ctx.peer_exchange
        t0 = time.perf_counter()
        gla_ctx.decode_sharded(qd, kd, vd, xb, nh, nkv, hd, n, f16_cache=True)
        st = gla_ctx.device_status()  # synchronises: the bounded wait has ended
        dt = time.perf_counter() - t0
    finally:
        gla_ctx.debug_xch_loopback(0)
    assert st == -5, gla.STATUS_NAMES.get(st, st)  # GLA_ERR_TIMEOUT
    assert 0.9 < dt < 10.0, dt  # the 1 s bound, not a hang
    # the status was read (and cleared); the same context decodes correctly
    xb2 = torch.empty(nh * hd, device="cuda")
    gla_ctx.decode(qd, kd, vd, xb2, nh, nkv, hd, n, f16_cache=True)
    assert gla_ctx.device_status() == 0
    ref = oracle.decode_f16(q, k16, v16, nh, nkv, hd, n)
    err = float(np.abs(xb2.cpu().numpy() - ref).max())
    assert err <= 5e-3, err
