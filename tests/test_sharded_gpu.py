"""KV-sequence-sharded decode over NCCL (gla_decode_sharded_*), one process
per GPU.  Needs >= 2 GPUs; skipped otherwise (the shard/merge math itself is
covered on one GPU by test_decode_gpu.py::test_partial_records_and_combine and
on CPU by test_multirank_host.py)."""
import os
import socket

import numpy as np
import pytest

import inputs

pytestmark = pytest.mark.gpu


def _n_gpus():
    try:
        import torch

        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:
        return 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, f16, out_dir):
    import datetime

    import torch
    import torch.distributed as dist

    import gpullama_attn as gla
    from gpullama_attn import sharding

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        ctx = gla.Context(rank, torch.cuda.current_stream().cuda_stream)
        uid = [gla.Context.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        ctx.comm_init(world, rank, uid[0])
        nh, nkv, hd, T = 28, 4, 128, 20000
        q, k, v = inputs.decode_case(91, nh, nkv, hd, T)
        lo, hi = sharding.kv_shard_bounds(T, world, rank)
        if f16:
            kk = inputs.to_f16_bits(k[lo:hi]).view(np.int16)
            vv = inputs.to_f16_bits(v[lo:hi]).view(np.int16)
        else:
            kk, vv = np.ascontiguousarray(k[lo:hi]), np.ascontiguousarray(v[lo:hi])
        qd = torch.from_numpy(q).cuda()
        kd, vd = torch.from_numpy(kk).cuda(), torch.from_numpy(vv).cuda()
        xb = torch.empty(nh * hd, device="cuda")
        for _ in range(2):  # twice: the record buffers are reused
            ctx.decode_sharded(qd, kd, vd, xb, nh, nkv, hd, hi - lo, f16_cache=f16)
        torch.cuda.synchronize()
        assert ctx.device_status() == 0
        np.save(os.path.join(out_dir, f"xb{rank}.npy"), xb.cpu().numpy())
        dist.barrier()
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("f16", [True, False], ids=["f16kv", "f32kv"])
def test_sharded_decode_two_gpus(tmp_path, oracle, f16):
    if _n_gpus() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, f16, str(tmp_path)))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    nh, nkv, hd, T = 28, 4, 128, 20000
    q, k, v = inputs.decode_case(91, nh, nkv, hd, T)
    if f16:
        ref = oracle.decode_f16(q, inputs.to_f16_bits(k), inputs.to_f16_bits(v), nh, nkv, hd, T)
        tol = 5e-3
    else:
        ref = oracle.decode_f32(q, k, v, nh, nkv, hd, T)
        tol = 1e-3
    for r in range(world):
        got = np.load(tmp_path / f"xb{r}.npy")
        err = np.abs(got - ref).max()
        assert err <= tol and err / np.abs(ref).max() <= tol, (r, err)
