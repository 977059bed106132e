"""KV-sequence-sharded decode (gla_decode_sharded_*), one process per GPU:
the peer exchange (records stored into every rank's buffer over NVLink and
merged inside the decode kernel) and the NCCL all-gather path.  Needs >= 2
GPUs; skipped otherwise (the shard/merge math itself is covered on one GPU by
test_decode_gpu.py::test_partial_records_and_combine and on CPU by
test_multirank_host.py)."""
import os
import socket

import numpy as np
import pytest

import inputs

pytestmark = pytest.mark.gpu

NH, NKV, HD, T = 28, 4, 128, 20000
N_CALLS = 4  # consecutive calls: both exchange parities, epochs advancing
SCALES = [1.0 + 0.25 * i for i in range(N_CALLS)]  # q of call i = q * SCALES[i]


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


def _shard(x, lo, hi, f16):
    import torch

    if f16:
        return torch.from_numpy(inputs.to_f16_bits(x[lo:hi]).view(np.int16)).cuda()
    return torch.from_numpy(np.ascontiguousarray(x[lo:hi])).cuda()


def _rank_main(rank, world, port, f16, mode, out_dir):
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
        if mode == "nccl":
            ctx.set_option(gla.OPT_SHARD_EXCHANGE, 0)
        uid = [gla.Context.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        ctx.comm_init(world, rank, uid[0])
        np.save(os.path.join(out_dir, f"peer{rank}.npy"), np.array([int(ctx.peer_exchange)]))
        q, k, v = inputs.decode_case(91, NH, NKV, HD, T)
        lo, hi = sharding.kv_shard_bounds(T, world, rank)
        kd, vd = _shard(k, lo, hi, f16), _shard(v, lo, hi, f16)
        outs = []
        for i in range(N_CALLS):  # back to back on the stream, read at the end
            qd = torch.from_numpy(q * np.float32(SCALES[i])).cuda()
            xb = torch.empty(NH * HD, device="cuda")
            ctx.decode_sharded(qd, kd, vd, xb, NH, NKV, HD, hi - lo, f16_cache=f16)
            outs.append(xb)
        # one row in all: every other rank holds an empty shard
        lo1, hi1 = sharding.kv_shard_bounds(1, world, rank)
        k1, v1 = _shard(k, 0, 1, f16), _shard(v, 0, 1, f16)
        xb1 = torch.empty(NH * HD, device="cuda")
        ctx.decode_sharded(torch.from_numpy(q).cuda(), k1, v1, xb1, NH, NKV, HD, hi1 - lo1,
                           f16_cache=f16)
        torch.cuda.synchronize()
        assert ctx.device_status() == 0
        np.save(os.path.join(out_dir, f"xb{rank}.npy"), torch.stack(outs).cpu().numpy())
        np.save(os.path.join(out_dir, f"one{rank}.npy"), xb1.cpu().numpy())
        dist.barrier()
        ctx.close()
    finally:
        dist.destroy_process_group()


def _run_world(tmp_path, oracle, f16, mode, world):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, f16, mode, str(tmp_path)))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(world):
        used_peer = bool(np.load(tmp_path / f"peer{r}.npy")[0])
        assert used_peer == (mode == "peer"), (r, used_peer)
    q, k, v = inputs.decode_case(91, NH, NKV, HD, T)
    tol = 5e-3 if f16 else 1e-3
    kk = inputs.to_f16_bits(k) if f16 else k
    vv = inputs.to_f16_bits(v) if f16 else v
    dec = oracle.decode_f16 if f16 else oracle.decode_f32
    refs = [dec(q * np.float32(s), kk, vv, NH, NKV, HD, T) for s in SCALES]
    ref1 = dec(q, kk, vv, NH, NKV, HD, 1)
    for r in range(world):
        got = np.load(tmp_path / f"xb{r}.npy")
        for i, ref in enumerate(refs):
            err = np.abs(got[i] - ref).max()
            assert err <= tol and err / np.abs(ref).max() <= tol, (r, i, err)
        one = np.load(tmp_path / f"one{r}.npy")
        err = np.abs(one - ref1).max()
        assert err <= tol and err / np.abs(ref1).max() <= tol, (r, "one row", err)


@pytest.mark.parametrize("mode", ["peer", "nccl"])
@pytest.mark.parametrize("f16", [True, False], ids=["f16kv", "f32kv"])
def test_sharded_decode_two_gpus(tmp_path, oracle, f16, mode):
    if _n_gpus() < 2:
        pytest.skip("needs 2 GPUs")
    _run_world(tmp_path, oracle, f16, mode, 2)


@pytest.mark.parametrize("world", [4, 8])
def test_sharded_decode_peer_exchange_wider(tmp_path, oracle, world):
    if _n_gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    _run_world(tmp_path, oracle, True, "peer", world)


def _drop_main(rank, world, port, mode, out_dir):
    """Rank 1 skips one sharded call.  Peer exchange: rank 0's bounded wait
    for rank 1's records runs out (GLA_ERR_TIMEOUT in the device status);
    both ranks then resynchronise the exchange (gla_comm_resync) and the
    next call is right again.  NCCL path: rank 0's all-gather waits for rank
    1 until the host watchdog (gla_comm_wait, 3 s) aborts the communicator;
    both ranks then join a new one and the next call is right again.  No rank
    leaves while its kernels or collectives are in flight; NVLS is off."""
    import datetime
    import time

    import torch
    import torch.distributed as dist

    import gpullama_attn as gla
    from gpullama_attn import sharding

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        ctx = gla.Context(rank, torch.cuda.current_stream().cuda_stream)
        ctx.set_option(gla.OPT_COMM_TIMEOUT_MS, 3000)
        if mode == "nccl":
            ctx.set_option(gla.OPT_SHARD_EXCHANGE, 0)

        def join():
            uid = [gla.Context.comm_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(uid, src=0)
            ctx.comm_init(world, rank, uid[0])

        join()
        q, k, v = inputs.decode_case(91, NH, NKV, HD, T)
        lo, hi = sharding.kv_shard_bounds(T, world, rank)
        kd, vd = _shard(k, lo, hi, True), _shard(v, lo, hi, True)
        qd = torch.from_numpy(q).cuda()
        xb = torch.empty(NH * HD, device="cuda")
        ctx.decode_sharded(qd, kd, vd, xb, NH, NKV, HD, hi - lo)  # call 1: everybody
        assert ctx.device_status() == 0
        dist.barrier()
        result = {}
        if rank == 0:  # call 2: rank 1 skips it
            t0 = time.perf_counter()
            ctx.decode_sharded(qd, kd, vd, xb, NH, NKV, HD, hi - lo)
            if mode == "peer":
                result["status"] = ctx.device_status()
            else:
                try:
                    ctx.comm_wait()
                    result["status"] = 0
                except gla.GlaError as e:
                    result["status"] = e.status
            result["seconds"] = time.perf_counter() - t0
        dist.barrier()  # the others learn of it on the host
        if mode == "peer":
            ctx.comm_resync()
        else:
            join()  # a new communicator (rank 1's old one ends at its watchdog)
        xb3 = torch.empty(NH * HD, device="cuda")
        ctx.decode_sharded(qd, kd, vd, xb3, NH, NKV, HD, hi - lo)  # call 3: everybody
        assert ctx.device_status() == 0
        np.save(os.path.join(out_dir, f"after{rank}.npy"), xb3.cpu().numpy())
        if rank == 0:
            np.save(os.path.join(out_dir, "drop.npy"),
                    np.array([result["status"], result["seconds"]], dtype=np.float64))
        dist.barrier()
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["peer", "nccl"])
def test_rank_skips_a_call_then_recovers(tmp_path, oracle, mode):
    if _n_gpus() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_drop_main, args=(r, 2, port, mode, str(tmp_path)))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    status, seconds = np.load(tmp_path / "drop.npy")
    assert int(status) == -5, status  # GLA_ERR_TIMEOUT
    assert seconds < (5.0 if mode == "peer" else 10.0), seconds
    q, k, v = inputs.decode_case(91, NH, NKV, HD, T)
    ref = oracle.decode_f16(q, inputs.to_f16_bits(k), inputs.to_f16_bits(v), NH, NKV, HD, T)
    for r in range(2):
        got = np.load(tmp_path / f"after{r}.npy")
        err = np.abs(got - ref).max()
        assert err <= 5e-3 and err / np.abs(ref).max() <= 5e-3, (r, err)
