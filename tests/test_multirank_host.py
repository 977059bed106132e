"""Multi-rank host logic on CPU (gloo, world_size 2): KV-sequence sharding
with an all-gather of shard records and the log-sum-exp merge, and the
sequence split of batched decode."""
import os
import socket

import numpy as np
import pytest

import inputs
import reference64
from gpullama_attn import sharding


def test_kv_shard_bounds_cover_rows():
    for T in (1, 2, 7, 4096, 131072):
        for world in (1, 2, 3, 4, 8):
            spans = [sharding.kv_shard_bounds(T, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == T
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1


def test_lpt_assign_balances_c3_lengths():
    rng = np.random.Generator(np.random.PCG64(3))
    lengths = [int(x) for x in rng.integers(1024, 32768, size=16, endpoint=True)]
    for world in (1, 2, 4, 8):
        parts = sharding.lpt_assign(lengths, world)
        assert sorted(i for p in parts for i in p) == list(range(16))
        loads = [sum(lengths[i] for i in p) for p in parts]
        assert max(loads) <= sum(lengths) / world + max(lengths)


def test_merge_of_shard_records_equals_unsharded(oracle):
    nh, nkv, hd, T = 28, 4, 128, 3001
    q, k, v = inputs.decode_case(77, nh, nkv, hd, T)
    full = oracle.decode_f32(q, k, v, nh, nkv, hd, T)
    for world in (1, 2, 3, 8):
        recs = [reference64.records64(q, k, v, nh, nkv, hd,
                                      slice(*sharding.kv_shard_bounds(T, world, r)))
                for r in range(world)]
        merged = reference64.lse_combine64(np.stack(recs), hd)
        np.testing.assert_allclose(merged, full, atol=2e-5)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_path):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        nh, nkv, hd, T = 16, 4, 64, 1000
        q, k, v = inputs.decode_case(5, nh, nkv, hd, T)  # every rank builds the same inputs
        lo, hi = sharding.kv_shard_bounds(T, world, rank)
        rec = torch.from_numpy(reference64.records64(q, k[lo:hi], v[lo:hi], nh, nkv, hd,
                                                     slice(0, hi - lo)))
        gathered = [torch.zeros_like(rec) for _ in range(world)]
        dist.all_gather(gathered, rec)
        merged = reference64.lse_combine64(torch.stack(gathered).numpy(), hd)
        if rank == 0:
            np.save(result_path, merged)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_all_gather_and_merge(tmp_path, oracle):
    import torch.multiprocessing as mp

    world = 2
    out = str(tmp_path / "merged.npy")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    nh, nkv, hd, T = 16, 4, 64, 1000
    q, k, v = inputs.decode_case(5, nh, nkv, hd, T)
    full = oracle.decode_f32(q, k, v, nh, nkv, hd, T)
    np.testing.assert_allclose(np.load(out), full, atol=2e-5)


def _drop_rank_main(rank, world, port, result_path):
    """Rank 1 leaves after step 0 (between steps: nothing of it in flight).
    Rank 0 learns of it on the host, from the store, before its next launch
    (StepBarrier.enter raises RankLost within the timeout), and a collective
    with the departed rank ends with an error within the process group's
    short timeout instead of waiting for good."""
    import datetime
    import time

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    store = dist.distributed_c10d._get_default_store()
    guard = sharding.StepBarrier(store, world, rank, timeout_s=1.0)
    guard.enter(0)
    t = torch.ones(4)
    dist.all_reduce(t)  # step 0's collective: everybody
    if rank == 1:
        os._exit(0)  # leaves between steps, without a goodbye
    out = {}
    t0 = time.monotonic()
    try:
        guard.enter(1)
        out["lost"] = []
    except sharding.RankLost as e:
        out["lost"] = e.missing
    out["detect_s"] = time.monotonic() - t0
    t0 = time.monotonic()
    try:
        dist.all_reduce(t)
        out["collective"] = "completed"
    except Exception as e:  # noqa: BLE001 - any error is the expected outcome
        out["collective"] = type(e).__name__
    out["collective_s"] = time.monotonic() - t0
    np.save(result_path, np.array([out["lost"] == [1], out["detect_s"],
                                   out["collective"] != "completed", out["collective_s"]],
                                  dtype=np.float64))
    os._exit(0)


def test_gloo_rank_drop_is_detected_on_the_host(tmp_path):
    import torch.multiprocessing as mp

    out = str(tmp_path / "drop.npy")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_drop_rank_main, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    lost_ok, detect_s, coll_failed, coll_s = np.load(out)
    assert lost_ok == 1.0
    assert 0.9 < detect_s < 5.0, detect_s
    assert coll_failed == 1.0
    assert coll_s < 30.0, coll_s


def test_step_barrier_passes_when_every_rank_arrives():
    class Store(dict):
        def set(self, k, v):
            self[k] = v

        def check(self, keys):
            return all(k in self for k in keys)

    s = Store()
    a = sharding.StepBarrier(s, 2, 0, timeout_s=0.2)
    b = sharding.StepBarrier(s, 2, 1, timeout_s=0.2)
    s.set(b._key(7, 1), "1")
    a.enter(7)  # rank 1 already there
    with pytest.raises(sharding.RankLost) as e:
        a.enter(8)
    assert e.value.missing == [1] and e.value.step == 8
