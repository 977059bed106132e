#!/usr/bin/env python3
"""Benchmark of libgpullama_attn decode attention on B200.

Default workload: Qwen2.5-7B-shape long-context decode
attention, nHeads 28, nKVHeads 4, headDim 128, context 131072, FP16 KV.  One
step = the attention of one new token through 28 layer caches of that shape
(the model's 28 layers; 28 kernel launches replayed from a CUDA graph), so
successive launches stream 268 MB each from HBM (7.5 GB a step, far above the
126 MB L2; no flush needed).  On N GPUs the KV sequence of every layer is
split evenly (rank r holds rows [r*T/N, (r+1)*T/N)); each launch computes its
shard's (m, l, o) records, exchanges them with every rank over peer memory
(NVLink) and merges them in the same kernel (NCCL all-gather + combine kernel
when the peer mapping is unavailable): strong scaling.

Before timing, every rank's output of layer 0 is compared with the CPU
oracle (the C restatement of the reference's Java attention) on the same
seeded data; a mismatch above the FP16-cache tolerance (5e-3) exits non-zero.

On one GPU the line also carries the C2 config (Llama-3.2-3B, 28 layers,
FP32 KV, context 4096, RoPE'd; device and end-to-end numbers) under "c2" and
the C5 causal prefill (Phi-3-mini, L 4096) under "prefill".

Metric: decode-attn KV-read GB/s (algorithmic bytes / device time), reported
with µs per layer-step, the fraction of the measured HBM peak and the CPU
baseline (the oracle timed on the host cores).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload c1|c2|c3|c4|c5|c4q8]

Multi-GPU (launched by torch.distributed.run, one rank per GPU):
  c4:    KV sequence sharded as above (strong scaling).
  c3:    the 16 sequences are dealt to the ranks (longest-first); strong.
  c2/c1: every rank decodes its own sequence (replicas, weak scaling).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(REPO, "gpullama3.java_b200")]

import numpy as np  # noqa: E402

# ---------------------------------------------------------------------------
# Workloads
# ---------------------------------------------------------------------------
WORKLOADS = {
    "c1": dict(name="llama3.2-1b-decode-attn", layers=1, n_heads=32, n_kv=8, hd=64, T=512,
               f16=False, theta=None, batch=1),
    "c2": dict(name="llama3.2-3b-decode-attn-28L", layers=28, n_heads=24, n_kv=8, hd=128, T=4096,
               f16=False, theta=500000.0, batch=1),
    "c3": dict(name="llama3.1-8b-batched-decode-attn-32L", layers=32, n_heads=32, n_kv=8, hd=128,
               T=None, f16=True, theta=None, batch=16),
    # config 4 is one layer; a step runs 28 layer caches of that shape (the
    # model's layer count) so that successive launches stream from HBM
    "c4": dict(name="qwen2.5-7b-longctx-decode-attn", layers=28, n_heads=28, n_kv=4, hd=128,
               T=131072, f16=True, theta=None, batch=1),
    "c5": dict(name="phi3-mini-causal-prefill-attn", layers=1, n_heads=32, n_kv=32, hd=96,
               T=4096, f16=True, theta=None, batch=1),
    # not a BASELINE config: config 4's shape over a Q8 cache (int8 values, an
    # FP16 scale per 32), one replica per GPU
    "c4q8": dict(name="qwen2.5-7b-longctx-decode-attn-q8kv", layers=1, n_heads=28, n_kv=4, hd=128,
                 T=131072, f16=False, theta=None, batch=1),
}

FALLBACK_HBM_GBS = 6650.0
L2_BYTES = 126e6
F16_TOL = 5e-3  # FP16 KV cache: max abs error and max abs error / max |ref|


def c3_lengths():
    rng = np.random.Generator(np.random.PCG64(3))
    return [int(x) for x in rng.integers(1024, 32768, size=16, endpoint=True)]


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def traffic_from_profiles(workload, kernel="decode_kernel"):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary."""
    path = os.path.join(REPO, "profiles", f"{kernel}_{workload}.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


def kv_bytes_per_layer(key):
    """Algorithmic KV bytes of one layer of the whole job (all ranks)."""
    wl = WORKLOADS[key]
    esize = 2 if wl["f16"] else 4
    rows = sum(c3_lengths()) if key == "c3" else wl["T"]
    return 2 * rows * wl["n_kv"] * wl["hd"] * esize


def workload_config(key, world):
    """The config dict of a workload at `world` ranks; both arms print it."""
    wl = WORKLOADS[key]
    per_rank_launch = kv_bytes_per_layer(key) / (world if key in ("c3", "c4") else 1)
    per_rank_step = per_rank_launch * wl["layers"]
    if per_rank_launch > L2_BYTES:
        l2 = "inputs exceed L2 (KV bytes per launch > 126 MB L2)"
    elif per_rank_step > L2_BYTES:
        l2 = "inputs exceed L2 (KV bytes per step > 126 MB; layer caches rotate)"
    else:
        l2 = "KV set fits in L2 between steps (latency-bound config, no flush)"
    if world == 1:
        par = "single"
    elif key == "c4":
        par = f"kv-shard{world}"
    else:
        par = f"seq-shard{world}"
    cfg = {"workload": wl["name"], "baseline_config": key, "layers": wl["layers"],
           "n_heads": wl["n_heads"], "n_kv_heads": wl["n_kv"], "head_dim": wl["hd"],
           "context": wl["T"] if wl["T"] else "U[1024,32768] x16",
           "kv_dtype": "f16" if wl["f16"] else "f32",
           "rope_theta": wl["theta"],
           "global_batch": wl["batch"] * (world if key in ("c1", "c2") else 1),
           "parallelism": par, "l2": l2}
    if key == "c4":
        cfg["step"] = "28 layer caches of the config-4 single-layer shape (one launch each)"
    return cfg


# ---------------------------------------------------------------------------
# Clock sampling during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# Inputs
# ---------------------------------------------------------------------------
def rope_tables(T, hd, theta, torch, device):
    """RoPE.precomputeFreqsCis (RoPE.java:6-37): float freq, float angle, double cos/sin."""
    i = torch.arange(0, hd, 2, dtype=torch.float64)
    freq = (1.0 / torch.pow(torch.tensor(theta, dtype=torch.float64), i / hd)).float()
    pos = torch.arange(T, dtype=torch.float32)
    ang = pos[:, None] * freq[None, :]
    return (torch.cos(ang.double()).float().to(device), torch.sin(ang.double()).float().to(device))


def rope_interleaved_rows(x, cos, sin):
    """Rotates rows x[t] ([T][n*hd], pairs (2i, 2i+1)) at their own positions t."""
    T, D = x.shape
    hd2 = cos.shape[1]
    xv = x.view(T, D // (2 * hd2), hd2, 2)
    a, b = xv[..., 0].clone(), xv[..., 1].clone()
    c, s = cos[:T, None, :], sin[:T, None, :]
    xv[..., 0] = a * c - b * s
    xv[..., 1] = a * s + b * c


def rope_interleaved_rows_at(x, cos, sin, pos):
    hd2 = cos.shape[1]
    xv = x.view(-1, hd2, 2)
    a, b = xv[..., 0].clone(), xv[..., 1].clone()
    c, s = cos[pos], sin[pos]
    xv[..., 0] = a * c - b * s
    xv[..., 1] = a * s + b * c


def make_decode_inputs(wl, torch, device, seed, lengths=None):
    """KV caches per layer (and sequence), q per layer: ~N(0,1) from a seeded torch generator."""
    g = torch.Generator(device=device).manual_seed(seed)
    dt = torch.float16 if wl["f16"] else torch.float32
    L, nh, nkv, hd = wl["layers"], wl["n_heads"], wl["n_kv"], wl["hd"]
    kv = nkv * hd
    if lengths is None:
        T = wl["T"]
        K = torch.empty(L, T, kv, device=device, dtype=dt)
        V = torch.empty_like(K)
        for l in range(L):
            K[l].normal_(generator=g)
            V[l].normal_(generator=g)
        q = torch.randn(L, nh * hd, device=device, generator=g)
        if wl["theta"]:
            cos, sin = rope_tables(T, hd, wl["theta"], torch, device)
            for l in range(L):
                kl = K[l].float()
                rope_interleaved_rows(kl, cos, sin)
                K[l].copy_(kl)
                ql = q[l].view(1, -1)
                rope_interleaved_rows_at(ql, cos, sin, T - 1)
        return dict(K=K, V=V, q=q, rows=T)
    # batched: one cache per (layer, sequence)
    Ks, Vs = [], []
    for l in range(L):
        Ks.append([torch.randn(n, kv, device=device, dtype=dt, generator=g) for n in lengths])
        Vs.append([torch.randn(n, kv, device=device, dtype=dt, generator=g) for n in lengths])
    q = torch.randn(L, len(lengths), nh * hd, device=device, generator=g)
    kp = torch.tensor([[t.data_ptr() for t in Ks[l]] for l in range(L)], dtype=torch.int64,
                      device=device)
    vp = torch.tensor([[t.data_ptr() for t in Vs[l]] for l in range(L)], dtype=torch.int64,
                      device=device)
    npos = torch.tensor(lengths, dtype=torch.int32, device=device)
    return dict(Ks=Ks, Vs=Vs, q=q, kp=kp, vp=vp, npos=npos)


def c4_full_layer(torch, device, wl, layer, out_k, out_v):
    """Layer `layer` of the config-4 caches, all T rows, FP16 ~N(0,1): the same
    values on every rank (a torch generator seeded by the layer)."""
    g = torch.Generator(device=device).manual_seed(7000 + layer)
    out_k.normal_(generator=g)
    out_v.normal_(generator=g)


def make_sharded_inputs(wl, torch, device, world, rank):
    """Config 4 sharded by KV rows: rank `rank` keeps rows [lo, hi) of every
    layer; q (replicated) from seed 9000."""
    from gpullama_attn import sharding

    L, nh, nkv, hd, T = wl["layers"], wl["n_heads"], wl["n_kv"], wl["hd"], wl["T"]
    kv = nkv * hd
    lo, hi = sharding.kv_shard_bounds(T, world, rank)
    n = hi - lo
    K = torch.empty(L, max(n, 1), kv, device=device, dtype=torch.float16)
    V = torch.empty_like(K)
    fk = torch.empty(T, kv, device=device, dtype=torch.float16)
    fv = torch.empty_like(fk)
    for l in range(L):
        c4_full_layer(torch, device, wl, l, fk, fv)
        K[l, :n].copy_(fk[lo:hi])
        V[l, :n].copy_(fv[lo:hi])
    del fk, fv
    g = torch.Generator(device=device).manual_seed(9000)
    q = torch.randn(L, nh * hd, device=device, generator=g)
    return dict(K=K, V=V, q=q, rows=n, lo=lo, hi=hi)


# ---------------------------------------------------------------------------
# In-run parity check (the oracle as the checker, outside the timed region)
# ---------------------------------------------------------------------------
def check_c4(wl, inp, xb, torch, device, rank, dist):
    """Every rank's layer-0 output against the oracle on the same seeded data.
    Rank 0 runs the oracle (the C restatement of InferenceCore.java:105-144 on
    the decoded FP16 cache) and broadcasts the reference; every rank compares
    its own merged xb.  Returns (max abs error, max abs error / max |ref|)
    over all ranks."""
    nh, nkv, hd, T = wl["n_heads"], wl["n_kv"], wl["hd"], wl["T"]
    ref = torch.zeros(nh * hd, device=device)
    if rank == 0:
        sys.path.insert(0, os.path.join(REPO, "oracle"))
        import oracle  # test infrastructure: the parity checker

        oracle.build()
        fk = torch.empty(T, nkv * hd, device=device, dtype=torch.float16)
        fv = torch.empty_like(fk)
        c4_full_layer(torch, device, wl, 0, fk, fv)
        k16 = fk.view(torch.int16).cpu().numpy().view(np.uint16)
        v16 = fv.view(torch.int16).cpu().numpy().view(np.uint16)
        del fk, fv
        q0 = inp["q"][0].cpu().numpy()
        r = oracle.decode_f16(q0, k16, v16, nh, nkv, hd, T,
                              n_threads=min(nh, oracle.max_threads()))
        ref.copy_(torch.from_numpy(r))
    if dist is not None:
        dist.broadcast(ref, src=0)
    err = (xb[0].reshape(-1) - ref).abs().max()
    rel = err / ref.abs().max().clamp_min(1e-30)
    t = torch.stack([err, rel]).float()
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t[0]), float(t[1])


# ---------------------------------------------------------------------------
# CPU baseline (oracle = C restatement of InferenceCore.java:105-144)
# ---------------------------------------------------------------------------
def cpu_baseline(wl_key, wl, budget_s=8.0):
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle  # test infrastructure: timed CPU baseline only

    oracle.build()
    nh, nkv, hd = wl["n_heads"], wl["n_kv"], wl["hd"]
    threads = min(nh, oracle.max_threads())
    rng = np.random.Generator(np.random.PCG64(0))
    lengths = c3_lengths() if wl_key == "c3" else [wl["T"]]
    # sample: one layer when a layer is large (config 4: 268 MB), else up to 4
    n_layers = 1 if kv_bytes_per_layer(wl_key) > 64e6 else min(wl["layers"], 4)
    cases = []
    for _ in range(n_layers):
        for n in lengths:
            q = rng.standard_normal(nh * hd, dtype=np.float32)
            k = rng.standard_normal((n, nkv * hd), dtype=np.float32)
            v = rng.standard_normal((n, nkv * hd), dtype=np.float32)
            if wl["f16"]:
                k, v = k.astype(np.float16).view(np.uint16), v.astype(np.float16).view(np.uint16)
            cases.append((q, k, v, n))
    esize = 2 if wl["f16"] else 4

    def run_once():
        nbytes = 0
        for q, k, v, n in cases:
            if wl["f16"]:
                oracle.decode_f16(q, k, v, nh, nkv, hd, n, n_threads=threads)
            else:
                oracle.decode_f32(q, k, v, nh, nkv, hd, n, n_threads=threads)
            nbytes += 2 * n * nkv * hd * esize
        return nbytes

    run_once()  # warm-up
    times, nbytes = [], 0
    t_end = time.perf_counter() + budget_s
    while True:
        t0 = time.perf_counter()
        nbytes = run_once()
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end and len(times) >= 3:
            break
    med = statistics.median(times)
    return dict(value=round(nbytes / med / 1e9, 4), unit="GB/s", cores=threads, kind="port",
                sample=f"{len(cases)} decode call(s) ({len(lengths)} seq x {n_layers} "
                       f"layer) of the {wl_key} shape, median of {len(times)} reps",
                seconds_per_sample=med, bytes_per_sample=nbytes)


def ms_est(fn, stream, torch, device):
    """Milliseconds of one call of fn (one untimed replay, events)."""
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        fn()
        e1.record(stream)
    torch.cuda.synchronize(device)
    return e0.elapsed_time(e1)


def all_max(x, torch, device, dist):
    if dist is None:
        return x
    t = torch.tensor([x], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# Our arm: decode workloads
# ---------------------------------------------------------------------------
def run_decode(args, key, rank, world, local_rank, dist, cpu_budget=8.0):
    import torch
    import gpullama_attn as gla
    from gpullama_attn import sharding

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    wl = dict(WORKLOADS[key])
    L, nh, nkv, hd = wl["layers"], wl["n_heads"], wl["n_kv"], wl["hd"]
    esize = 2 if wl["f16"] else 4
    stream = torch.cuda.Stream(device)
    ctx = gla.Context(local_rank, stream.cuda_stream)
    if args.trace:  # before any launch is captured: the stamps are launch arguments
        ctx.set_option(gla.OPT_TRACE, 1)
    sharded = key == "c4" and world > 1

    # ---- per-rank work -----------------------------------------------------
    lengths = None
    if key == "c3":
        all_len = c3_lengths()
        lengths = [all_len[i] for i in sharding.lpt_assign(all_len, world)[rank]]
        scaling = "strong"
        rows_step = sum(all_len)
    elif key == "c4":
        scaling = "strong"
        rows_step = wl["T"]
    else:
        scaling = "weak"
        rows_step = wl["T"] * world  # one sequence per rank
    bytes_step = 2 * L * rows_step * nkv * hd * esize  # whole job, all ranks

    with torch.cuda.stream(stream):
        if key == "c4":
            inp = make_sharded_inputs(wl, torch, device, world, rank)
        else:
            inp = make_decode_inputs(wl, torch, device, seed=1000 + rank, lengths=lengths)
        xb = torch.empty(L, max(1, len(lengths or [1])), nh * hd, device=device)
        if sharded:
            uid = [gla.Context.comm_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(uid, src=0)
            ctx.comm_init(world, rank, uid[0])
        ctx.reserve(16, nkv, nh, hd)
    torch.cuda.synchronize(device)
    peer = sharded and ctx.peer_exchange
    n_local = inp.get("rows", 0)

    launches_per_step = 0

    def step():
        nonlocal launches_per_step
        n = 0
        for l in range(L):
            if key == "c3":
                if lengths:
                    ctx.decode_batched(inp["q"][l], inp["kp"][l], inp["vp"][l], inp["npos"],
                                       max(lengths), xb[l], len(lengths), nh, nkv, hd,
                                       f16_cache=True)
                    n += 1
            elif sharded:
                ctx.decode_sharded(inp["q"][l], inp["K"][l], inp["V"][l], xb[l], nh, nkv, hd,
                                   n_local, f16_cache=True)
                n += 1 if peer else 2
            else:
                ctx.decode(inp["q"][l], inp["K"][l], inp["V"][l], xb[l], nh, nkv, hd,
                           n_local, f16_cache=wl["f16"])
                n += 1
        launches_per_step = n

    # warm-up (also grows the workspace outside capture)
    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup)):
            step()
    torch.cuda.synchronize(device)
    st = ctx.device_status()
    if st != 0:
        raise RuntimeError(f"device status {st} after warm-up")

    # in-run parity: every rank's merged output against the oracle
    parity = None
    if key == "c4" and not args.quick:
        err, rel = check_c4(wl, inp, xb, torch, device, rank, dist)
        parity = {"max_abs_err": err, "max_rel_err": rel, "tol": F16_TOL,
                  "checked": "layer 0 xb of every rank vs the oracle (C restatement of "
                             "InferenceCore.java:105-144 on the decoded FP16 cache)"}
        if not (err <= F16_TOL and rel <= F16_TOL):
            raise SystemExit(f"parity check failed on config 4: max abs err {err:.3e}, "
                             f"rel {rel:.3e} > {F16_TOL}")

    graph = None
    # the NCCL path stays eager; the peer exchange is one kernel and is captured
    use_graph = not sharded or peer
    if use_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        torch.cuda.synchronize(device)

    def replay():
        if graph is not None:
            graph.replay()
        else:
            step()

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            replay()
    torch.cuda.synchronize(device)

    # clocks: nvidia-smi samples every 100 ms from a ~1 s soak of the same
    # replay loop straight into the timed region, so the samples see this load
    sampler = ClockSampler(local_rank) if rank == 0 else None
    if sampler:
        sampler.start()
    t_soak = time.perf_counter()
    per_iter = max(ms_est(replay, stream, torch, device), 1e-3)
    soak_iters = 0 if args.quick else int(min(5000, max(1, 1000.0 / per_iter)))
    if dist is not None:  # every rank must issue the same collectives
        t = torch.tensor([soak_iters], device=device, dtype=torch.int64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        soak_iters = int(t.item())
    with torch.cuda.stream(stream):
        for _ in range(soak_iters):
            replay()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(device)
    soak_s = time.perf_counter() - t_soak
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            replay()
        e1.record(stream)
    torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1) / args.steps
    clocks = sampler.stop() if sampler else None
    ms = all_max(ms, torch, device, dist)
    if dist is not None:
        dist.barrier()
    st = ctx.device_status()
    if st != 0:
        raise RuntimeError(f"device status {st} after the timed region")
    trace = None
    if args.trace:  # phase timeline of the last timed launch, every rank
        from gpullama_attn import phase_trace
        mine = phase_trace.summarize_ctx(ctx, f"rank {rank}")
        trace = [mine]
        if dist is not None:
            trace = [None] * world
            dist.all_gather_object(trace, mine)

    # ---- e2e through the reference-facing calls with host buffers -----------
    e2e = None
    if not args.quick:
        if key in ("c1", "c2"):
            e2e = run_e2e_rope(args, ctx, wl, inp, torch, device, stream, dist)
        elif key == "c4":
            e2e = run_e2e_c4(args, ctx, wl, inp, xb, step, graph, torch, device, stream, dist,
                             bytes_step)

    # dominant kernel's average duration: the timed region holds only decode
    # launches except for sharded c4 over NCCL, whose partial kernel is timed
    # on its own (on the peer exchange the step is one fused kernel a layer)
    per_launch_ms = ms / max(1, launches_per_step if not sharded or peer else L)
    if sharded and not peer:
        part = torch.empty(nh, hd + 2, device=device)
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                ctx.decode_partial(inp["q"][0], inp["K"][0], inp["V"][0], part, nh, nkv, hd,
                                   n_local, f16_cache=True)
        k0 = torch.cuda.Event(enable_timing=True)
        k1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            k0.record(stream)
            for _ in range(args.steps):
                ctx.decode_partial(inp["q"][0], inp["K"][0], inp["V"][0], part, nh, nkv, hd,
                                   n_local, f16_cache=True)
            k1.record(stream)
        torch.cuda.synchronize(device)
        per_launch_ms = all_max(k0.elapsed_time(k1) / args.steps, torch, device, dist)
    del graph
    value = bytes_step / (ms * 1e-3) / 1e9
    hbm, hbm_kind = peaks()
    if key == "c4":
        bytes_launch = 2 * n_local * nkv * hd * esize  # this rank's shard
    else:
        bytes_launch = bytes_step / world / max(1, L)
    achieved = bytes_launch / (per_launch_ms * 1e-3) / 1e9 if key != "c3" or lengths else 0
    traffic = traffic_from_profiles(key)
    traffic_note = "ncu dram bytes of one launch (profiles/)"
    if key == "c4" and traffic is not None and world > 1:
        traffic = round(traffic * n_local / wl["T"])
        traffic_note = "1-GPU ncu capture scaled by the shard's rows"
    config = workload_config(key, world)
    result = {
        "metric": "decode-attn KV-read GB/s",
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 5),
        "us_per_layer_step": round(ms * 1e3 / L, 3),
        "tokens_per_s_equiv": round(1e3 / ms, 2),
        "hbm_frac": round(value / world / hbm, 4),
        "higher_is_better": True,
        "scaling": scaling,
        "vs_baseline": None,
        "dtype": "f16kv-f32acc" if wl["f16"] else "f32",
        "data": "synthetic ~N(0,1), seeded torch generator; RoPE'd q/K where the config says so",
        "config": config,
        "graph": use_graph,
        "gpu_launches": launches_per_step * args.steps,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm,
                     "unit": "GB/s", "frac": round(achieved / hbm, 4),
                     "traffic": traffic, "traffic_source": traffic_note,
                     "peak_source": f"{hbm_kind} copy bandwidth (MEASURED_PEAKS.json hbm_gbs)"
                     if hbm_kind == "measured" else "fallback 6.65 TB/s",
                     "kernel": "gla::decode_kernel", "bytes_per_launch": bytes_launch,
                     "launch_us": round(per_launch_ms * 1e3, 3)},
        "clocks": dict(clocks, soak_s=round(soak_s, 2)) if clocks else None,
    }
    if sharded:
        result["exchange"] = "peer-exchange (records over NVLink, merged in-kernel)" if peer \
            else "nccl-allgather + combine kernel"
    if parity is not None:
        result["parity"] = parity
    if trace is not None:
        result["trace"] = trace
    if e2e is not None:
        result["e2e"] = e2e
    if rank == 0 and world == 1 and not (args.no_cpu_baseline or args.quick):
        result["cpu_baseline"] = cpu_baseline(key, wl, budget_s=cpu_budget)
    ctx.close()
    return result


def timed_loop(args, fn, torch, device, stream, dist, soak_s=1.0):
    """Warm-up, a soak of about soak_s seconds of the same calls (so the
    timed steps run at the clocks of a sustained load, like the device-side
    number measured after its own soak), then device time per call (ms, CUDA
    events on the stream), bounded below by the host wall time, max over
    ranks."""
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            fn()
    torch.cuda.synchronize(device)
    if not args.quick and soak_s > 0:
        per_iter = max(ms_est(fn, stream, torch, device), 1e-3)
        n = int(min(5000, max(1, soak_s * 1000.0 / per_iter)))
        if dist is not None:  # every rank issues the same calls
            t = torch.tensor([n], device=device, dtype=torch.int64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            n = int(t.item())
        with torch.cuda.stream(stream):
            for _ in range(n):
                fn()
        torch.cuda.synchronize(device)
    if dist is not None:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            fn()
        e1.record(stream)
    torch.cuda.synchronize(device)
    wall = (time.perf_counter() - w0) / args.steps * 1e3
    ms = max(e0.elapsed_time(e1) / args.steps, wall)
    return all_max(ms, torch, device, dist)


def run_e2e_c4(args, ctx, wl, inp, xb, step, graph, torch, device, stream, dist, bytes_step):
    """Per step: q of every layer from pinned host memory, the 28 per-layer
    calls (gla_decode_f16kv on one GPU, gla_decode_sharded_f16kv on N: shard
    attention, exchange and merge), every layer's xb back to pinned memory.
    The calls replay from the CUDA graph they were captured into (a layer plan
    replays its tasks every token); the same calls issued eagerly are
    reported beside it."""
    L = wl["layers"]
    host_q = inp["q"].cpu().pin_memory()
    host_x = torch.empty(xb.shape, dtype=xb.dtype).pin_memory()

    def step_graph():
        inp["q"].copy_(host_q, non_blocking=True)
        graph.replay()
        host_x.copy_(xb, non_blocking=True)

    def step_eager():
        inp["q"].copy_(host_q, non_blocking=True)
        step()
        host_x.copy_(xb, non_blocking=True)

    out = {}
    if graph is not None:
        ms = timed_loop(args, step_graph, torch, device, stream, dist)
        ms_eager = timed_loop(args, step_eager, torch, device, stream, dist)
        out = {"value": round(bytes_step / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
               "ms_per_step": round(ms, 5),
               "path": "per step: pinned H2D of every layer's q, one CUDA-graph replay of "
                       "the per-layer calls, pinned D2H of every layer's xb",
               "eager": {"value": round(bytes_step / (ms_eager * 1e-3) / 1e9, 2),
                         "ms_per_step": round(ms_eager, 5),
                         "path": "the same calls issued eagerly from Python every step"}}
    else:
        ms = timed_loop(args, step_eager, torch, device, stream, dist)
        out = {"value": round(bytes_step / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
               "ms_per_step": round(ms, 5),
               "path": "per step: pinned H2D of every layer's q, the per-layer calls issued "
                       "eagerly, pinned D2H of every layer's xb"}
    out["h2d_bytes_per_step"] = int(host_q.numel() * 4)
    out["d2h_bytes_per_step"] = int(host_x.numel() * 4)
    out["gpu_launches_per_step"] = L
    st = ctx.device_status()
    if st != 0:
        raise RuntimeError(f"device status {st} in the e2e loop")
    return out


def run_e2e_rope(args, ctx, wl, inp, torch, device, stream, dist):
    """Per step: one H2D of the token's q (all layers) and new k/v rows from pinned
    memory, then per layer RoPE + KV append + attention through the
    reference-mirror entry point (position read on the device), then one D2H
    of every layer's xb."""
    L, nh, nkv, hd = wl["layers"], wl["n_heads"], wl["n_kv"], wl["hd"]
    T = wl["T"]
    K, V = inp["K"], inp["V"]
    kvd = nkv * hd
    # flat [layer][ctx][kvDim] caches as the reference allocates them
    per = nh * hd + 2 * kvd
    host_in = torch.randn(L, per, generator=torch.Generator().manual_seed(5)).pin_memory()
    host_out = torch.empty(L, nh * hd).pin_memory()
    dev_in = torch.empty(L, per, device=device)
    xb = torch.empty(L, nh * hd, device=device)
    pos = torch.tensor([T - 1], dtype=torch.int32, device=device)
    theta = wl["theta"] or 10000.0

    def layers():
        for l in range(L):
            q = dev_in[l, : nh * hd]
            k = dev_in[l, nh * hd: nh * hd + kvd]
            v = dev_in[l, nh * hd + kvd:]
            # RoPE on q and the new key, KV append and attention: one launch
            ctx.rope_append_attention(q, k, v, K, V, xb[l], nh, hd, kvd, nh // nkv, pos, l, T,
                                      theta)

    # The per-token layer loop as a host plan replays it: captured once into a
    # CUDA graph (the position is read on the device, so the same graph serves
    # every token).  Each timed step still copies the token's inputs in from
    # pinned host memory and every layer's xb back out.
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            dev_in.copy_(host_in, non_blocking=True)
            layers()
            host_out.copy_(xb, non_blocking=True)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        layers()
    torch.cuda.synchronize(device)

    def step_graph():
        dev_in.copy_(host_in, non_blocking=True)
        graph.replay()
        host_out.copy_(xb, non_blocking=True)

    def step_eager():
        dev_in.copy_(host_in, non_blocking=True)
        layers()
        host_out.copy_(xb, non_blocking=True)

    world = dist.get_world_size() if dist is not None else 1
    bytes_step = 2 * L * T * kvd * 4 * world
    ms = timed_loop(args, step_graph, torch, device, stream, dist)
    ms_eager = timed_loop(args, step_eager, torch, device, stream, dist)

    # the step after attention too: each layer's wo projection (FP16 [dim][dim],
    # its own matrix per layer) with the residual add, gla_wo_residual_f16
    # launched right behind the attention call (programmatic dependent launch)
    dim = nh * hd
    g16 = torch.Generator(device=device).manual_seed(6)
    wo = [(torch.randn(dim, dim, device=device, generator=g16) * 0.02).half() for _ in range(L)]
    x_res = torch.zeros(dim, device=device)

    def layers_wo():
        for l in range(L):
            q = dev_in[l, : nh * hd]
            k = dev_in[l, nh * hd: nh * hd + kvd]
            v = dev_in[l, nh * hd + kvd:]
            ctx.rope_append_attention(q, k, v, K, V, xb[l], nh, hd, kvd, nh // nkv, pos, l, T,
                                      theta)
            ctx.wo_residual(xb[l], x_res, wo[l], dim, dim)

    with torch.cuda.stream(stream):
        layers_wo()
    torch.cuda.synchronize(device)
    graph_wo = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_wo, stream=stream):
        layers_wo()
    torch.cuda.synchronize(device)

    def step_graph_wo():
        dev_in.copy_(host_in, non_blocking=True)
        graph_wo.replay()
        host_out.copy_(xb, non_blocking=True)

    ms_wo = timed_loop(args, step_graph_wo, torch, device, stream, dist)
    st = ctx.device_status()
    if st != 0:
        raise RuntimeError(f"device status {st} in the e2e loop")
    del graph, graph_wo
    wo_bytes = L * dim * dim * 2 * world
    return {"value": round(bytes_step / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "ms_per_step": round(ms, 5),
            "h2d_bytes_per_step": int(host_in.numel() * 4),
            "d2h_bytes_per_step": int(host_out.numel() * 4),
            "path": "per step: pinned H2D of q/k/v rows, one CUDA-graph replay of "
                    "gla_rope_append_attention_f32 (RoPE + KV append + attention) for every "
                    "layer (captured once), pinned D2H of every xb",
            "eager": {"value": round(bytes_step / (ms_eager * 1e-3) / 1e9, 2),
                      "ms_per_step": round(ms_eager, 5),
                      "path": "the same calls issued eagerly from Python every step"},
            "with_wo": {"ms_per_step": round(ms_wo, 5),
                        "us_per_layer": round(ms_wo * 1e3 / L, 3),
                        "kv_plus_wo_GBps": round((bytes_step + wo_bytes) / (ms_wo * 1e-3) / 1e9,
                                                 2),
                        "path": "the graph above plus gla_wo_residual_f16 (FP16 wo, "
                                f"{dim}x{dim}, residual add) after every layer's attention"},
            "gpu_launches_per_step": L}


# ---------------------------------------------------------------------------
# Our arm: causal prefill (config 5)
# ---------------------------------------------------------------------------
def cpu_prefill_sample(wl, budget_s=8.0):
    """CPU prefill baseline.  The reference ingests a prompt one position at a
    time (InferenceEngine.java:88-99: decode attention over rows 0..p for every
    p), in FP32.  A spread of 16 positions is timed with the oracle (its C
    restatement) on the FP16-rounded inputs and the time is scaled by row
    count to the whole causal triangle."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle  # test infrastructure: timed CPU baseline only

    oracle.build()
    L, nh, nkv, hd = wl["T"], wl["n_heads"], wl["n_kv"], wl["hd"]
    threads = min(nh, oracle.max_threads())
    rng = np.random.Generator(np.random.PCG64(0))
    q = rng.standard_normal((L, nh * hd), dtype=np.float32).astype(np.float16).astype(np.float32)
    k = rng.standard_normal((L, nkv * hd), dtype=np.float32).astype(np.float16).astype(np.float32)
    v = rng.standard_normal((L, nkv * hd), dtype=np.float32).astype(np.float16).astype(np.float32)
    positions = [int(x) for x in np.linspace(0, L - 1, 16)]
    visits = sum(p + 1 for p in positions)

    def sweep():
        for p in positions:
            oracle.decode_f32(q[p], k, v, nh, nkv, hd, p + 1, n_threads=threads)

    sweep()  # warm-up
    times = []
    t_end = time.perf_counter() + budget_s
    while True:
        t0 = time.perf_counter()
        sweep()
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end and len(times) >= 3:
            break
    full_s = statistics.median(times) / visits * (L * (L + 1) / 2)
    flops = 4.0 * nh * hd * L * (L + 1) / 2
    return dict(value=round(flops / full_s / 1e12, 6), unit="TFLOP/s", cores=threads,
                kind="port",
                sample=f"{len(positions)} prompt positions spread over 0..{L - 1}, "
                       f"median of {len(times)} sweeps, scaled by row count to all "
                       f"{L} positions ({full_s:.1f} s per prompt)")


def prefill_config(world):
    wl = WORKLOADS["c5"]
    return {"workload": wl["name"], "baseline_config": "c5", "L": wl["T"],
            "n_heads": wl["n_heads"], "n_kv_heads": wl["n_kv"], "head_dim": wl["hd"],
            "causal": True,
            "l2": "3 rotating Q/K/V copies (75 MB each set, 226 MB total > 126 MB L2)",
            "parallelism": f"replicas{world}" if world > 1 else "single"}


def run_prefill(args, rank, world, local_rank, dist, cpu_budget=8.0):
    """causal prefill, L 4096, 32 heads, hd 96, FP16 in, FP32
    softmax/accumulation/out. Metric: causal TFLOP/s = 4*nH*hd*L(L+1)/2 / time."""
    import torch
    import gpullama_attn as gla

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    wl = WORKLOADS["c5"]
    L, nh, nkv, hd = wl["T"], wl["n_heads"], wl["n_kv"], wl["hd"]
    stream = torch.cuda.Stream(device)
    ctx = gla.Context(local_rank, stream.cuda_stream)
    g = torch.Generator(device=device).manual_seed(1000 + rank)
    with torch.cuda.stream(stream):
        q = torch.randn(L, nh * hd, device=device, generator=g).half()
        k = torch.randn(L, nkv * hd, device=device, generator=g).half()
        v = torch.randn(L, nkv * hd, device=device, generator=g).half()
        out = torch.empty(L, nh * hd, device=device)
        # rotate inputs through copies larger than L2 so successive launches
        # read from HBM (Q/K/V are 25 MB each)
        n_rot = 3
        qs = [q.clone() for _ in range(n_rot)]
        ks = [k.clone() for _ in range(n_rot)]
        vs = [v.clone() for _ in range(n_rot)]
    torch.cuda.synchronize(device)

    def step(i):
        r = i % n_rot
        ctx.prefill_causal(qs[r], ks[r], vs[r], out, L, nh, nkv, hd)

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i)
    torch.cuda.synchronize(device)
    if ctx.device_status() != 0:
        raise RuntimeError("device status after warm-up")
    sampler = ClockSampler(local_rank) if rank == 0 else None
    if sampler:
        sampler.start()
    t_soak = time.perf_counter()
    if not args.quick:
        per = max(ms_est(lambda: step(0), stream, torch, device), 1e-3)
        with torch.cuda.stream(stream):
            for i in range(int(min(20000, 1000.0 / per))):
                step(i)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(device)
    soak_s = time.perf_counter() - t_soak
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for i in range(args.steps):
            step(i)
        e1.record(stream)
    torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1) / args.steps
    clocks = sampler.stop() if sampler else None
    ms = all_max(ms, torch, device, dist)
    if ctx.device_status() != 0:
        raise RuntimeError("device status after the timed region")
    tflops = 4.0 * nh * hd * L * (L + 1) / 2 / (ms * 1e-3) / 1e12 * world
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        peak, peak_kind = float(pk["bf16_tflops"]), "measured cuBLAS bf16 burst (MEASURED_PEAKS.json)"
    except Exception:
        peak, peak_kind = 1590.0, "fallback 1.59 PFLOP/s"
    flops = 4.0 * nh * hd * L * (L + 1) / 2

    # e2e through the reference-facing call: the prompt's FP32 q/k/v rows (a
    # batched QKV projection's output, before RoPE) from pinned host memory,
    # gla_ingest_prompt_f32 (RoPE, append to an FP32 [ctx][kv_dim] layer cache,
    # causal attention), xb back to pinned host memory
    g32 = torch.Generator(device="cpu").manual_seed(2000 + rank)
    hq = torch.randn(L, nh * hd, generator=g32).pin_memory()
    hk = torch.randn(L, nkv * hd, generator=g32).pin_memory()
    hv = torch.randn(L, nkv * hd, generator=g32).pin_memory()
    hout = torch.empty(L, nh * hd).pin_memory()
    with torch.cuda.stream(stream):
        dq, dk, dv = (torch.empty(x.shape, device=device) for x in (hq, hk, hv))
        kc32 = torch.zeros(L, nkv * hd, device=device)
        vc32 = torch.zeros_like(kc32)
        kc16 = torch.zeros(L, nkv * hd, device=device, dtype=torch.float16)
        vc16 = torch.zeros_like(kc16)
    theta = 10000.0

    def e2e_step():
        dq.copy_(hq, non_blocking=True)
        dk.copy_(hk, non_blocking=True)
        dv.copy_(hv, non_blocking=True)
        ctx.ingest_prompt(dq, dk, dv, kc32, vc32, out, 0, L, nh, nkv, hd, L, theta,
                          gla.ROPE_NEOX)
        hout.copy_(out, non_blocking=True)

    e2e_ms = timed_loop(args, e2e_step, torch, device, stream, dist)

    # the same prompt ingestion with device-resident inputs, both cache types
    def ingest(kc, vc, f16):
        return lambda: ctx.ingest_prompt(dq, dk, dv, kc, vc, out, 0, L, nh, nkv, hd, L, theta,
                                         gla.ROPE_NEOX, f16_cache=f16)

    ing32_ms = timed_loop(args, ingest(kc32, vc32, False), torch, device, stream, dist)
    ing16_ms = timed_loop(args, ingest(kc16, vc16, True), torch, device, stream, dist)
    if ctx.device_status() != 0:
        raise RuntimeError("device status after the ingestion runs")
    res = {
        "metric": "prefill-attn TFLOP/s (causal)", "value": round(tflops, 2), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16-in f32-softmax/acc f32-out",
        "data": "synthetic ~N(0,1), seeded torch generator",
        "config": prefill_config(world),
        "gpu_launches": args.steps,
        "roofline": {"bound": "tensor", "achieved": round(tflops / world, 2), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(tflops / world / peak, 4),
                     "traffic": traffic_from_profiles("c5", "prefill_kernel"),
                     "peak_source": peak_kind, "kernel": "gla::prefill_kernel<96>",
                     "flops_per_launch": flops, "launch_us": round(ms * 1e3, 3)},
        "clocks": dict(clocks, soak_s=round(soak_s, 2)) if clocks else None,
        "e2e": {"value": round(flops / (e2e_ms * 1e-3) / 1e12 * world, 2), "unit": "TFLOP/s",
                "ms_per_step": round(e2e_ms, 4),
                "call": "gla_ingest_prompt_f32 (RoPE + FP32 KV append + causal attention)",
                "h2d_bytes_per_step": int((hq.numel() + hk.numel() + hv.numel()) * 4),
                "d2h_bytes_per_step": int(hout.numel() * 4)},
        "ingest": {"unit": "TFLOP/s", "note": "device-resident FP32 q/k/v, RoPE + append + "
                   "attention of the whole prompt in one call",
                   "f32_cache": round(flops / (ing32_ms * 1e-3) / 1e12, 2),
                   "f16_cache": round(flops / (ing16_ms * 1e-3) / 1e12, 2),
                   "f32_cache_ms": round(ing32_ms, 4), "f16_cache_ms": round(ing16_ms, 4)},
    }
    if rank == 0 and world == 1 and not (args.no_cpu_baseline or args.quick):
        res["cpu_baseline"] = cpu_prefill_sample(wl, budget_s=cpu_budget)
    ctx.close()
    return res


# ---------------------------------------------------------------------------
# Our arm: config 4's shape over a Q8 cache (extra workload)
# ---------------------------------------------------------------------------
def run_q8(args, rank, world, local_rank, dist):
    """Config 4's shape (Qwen2.5-7B: 28 heads, 4 kv heads, hd 128, 131072
    positions) over a Q8 cache: int8 K/V values and FP16 block scales
    (gla_kv_quantize_q8 fills it from seeded FP32 rows), one gla_decode_q8kv a
    step, one replica per GPU.  KV bytes a step: 2*T*kv_dim + T*n_kv*16
    (142.6 MB, above the 126 MB L2, so the cache streams from HBM)."""
    import torch
    import gpullama_attn as gla

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    wl = WORKLOADS["c4q8"]
    nh, nkv, hd, T = wl["n_heads"], wl["n_kv"], wl["hd"], wl["T"]
    kvd = nkv * hd
    stream = torch.cuda.Stream(device)
    ctx = gla.Context(local_rank, stream.cuda_stream)
    g = torch.Generator(device=device).manual_seed(1000 + rank)
    with torch.cuda.stream(stream):
        kq = torch.empty(T, kvd, dtype=torch.int8, device=device)
        vq = torch.empty_like(kq)
        sc = torch.empty(T, nkv, 8, dtype=torch.int16, device=device)
        chunk = 16384
        for r0 in range(0, T, chunk):
            n = min(chunk, T - r0)
            kf = torch.randn(n, kvd, device=device, generator=g)
            vf = torch.randn(n, kvd, device=device, generator=g)
            ctx.quantize_q8(kf, vf, n, nkv, hd, kq[r0:], vq[r0:], sc[r0:])
        q = torch.randn(nh * hd, device=device, generator=g)
        xb = torch.empty(nh * hd, device=device)
    torch.cuda.synchronize(device)
    del kf, vf

    def step():
        ctx.decode_q8(q, kq, vq, sc, xb, nh, nkv, hd, T)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    torch.cuda.synchronize(device)
    sampler = ClockSampler(local_rank) if rank == 0 else None
    if sampler:
        sampler.start()
    t_soak = time.perf_counter()
    per = max(ms_est(graph.replay, stream, torch, device), 1e-3)
    soak = 0 if args.quick else int(min(20000, 1000.0 / per))
    if dist is not None:
        t = torch.tensor([soak], device=device, dtype=torch.int64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        soak = int(t.item())
    with torch.cuda.stream(stream):
        for _ in range(soak):
            graph.replay()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(device)
    soak_s = time.perf_counter() - t_soak
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1) / args.steps
    clocks = sampler.stop() if sampler else None
    ms = all_max(ms, torch, device, dist)
    if ctx.device_status() != 0:
        raise RuntimeError("device status after the timed region")
    # e2e: q from pinned host memory, the call, xb back (the cache stays resident)
    hq = q.cpu().pin_memory()
    hx = torch.empty(nh * hd).pin_memory()

    def e2e_step():
        q.copy_(hq, non_blocking=True)
        step()
        hx.copy_(xb, non_blocking=True)

    e2e_ms = timed_loop(args, e2e_step, torch, device, stream, dist)
    del graph
    kv_bytes = 2 * T * kvd + T * nkv * 16
    peak, peak_kind = peaks()
    gbs = kv_bytes * world / (ms * 1e-3) / 1e9
    res = {
        "metric": "decode-attn KV-read GB/s", "value": round(gbs, 2), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 5), "us_per_layer_step": round(ms * 1e3, 3),
        "tokens_per_s_equiv": round(1e3 / ms, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "q8 (int8 + f16 block scales), f32 acc",
        "data": "synthetic ~N(0,1) rows quantised on the device, seeded torch generator",
        "config": {"workload": wl["name"], "baseline_config": "c4 shape, Q8 cache (extra)",
                   "n_heads": nh, "n_kv_heads": nkv, "head_dim": hd, "context": T,
                   "kv_dtype": "q8", "kv_bytes_per_step_per_gpu": kv_bytes,
                   "l2": "142.6 MB cache > 126 MB L2, no flush",
                   "parallelism": f"replicas{world}" if world > 1 else "single"},
        "gpu_launches": args.steps,
        "roofline": {"bound": "hbm", "achieved": round(kv_bytes / (ms * 1e-3) / 1e9, 1),
                     "peak": peak, "unit": "GB/s",
                     "frac": round(kv_bytes / (ms * 1e-3) / 1e9 / peak, 4),
                     "traffic": traffic_from_profiles("c4q8"),
                     "peak_source": peak_kind, "kernel": "gla::decode_kernel<Q8Consumer<128>>",
                     "bytes_per_launch": kv_bytes},
        "clocks": dict(clocks, soak_s=round(soak_s, 2)) if clocks else None,
        "e2e": {"value": round(kv_bytes * world / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 5), "h2d_bytes_per_step": int(hq.numel() * 4),
                "d2h_bytes_per_step": int(hx.numel() * 4)},
    }
    ctx.close()
    return res


def summary_of(res):
    """The keys of a secondary workload kept in the headline line."""
    keep = ("metric", "value", "unit", "ms_per_step", "us_per_layer_step", "tokens_per_s_equiv",
            "config", "dtype", "gpu_launches", "roofline", "clocks", "e2e", "cpu_baseline",
            "ingest", "parity")
    return {k: res[k] for k in keep if k in res}


# ---------------------------------------------------------------------------
# Reference arm: the reference's CPU attention (C restatement) on host cores
# ---------------------------------------------------------------------------
def run_reference_prefill(args, world):
    wl = WORKLOADS["c5"]
    L, nh, hd = wl["T"], wl["n_heads"], wl["hd"]
    flops = 4.0 * nh * hd * L * (L + 1) / 2
    values = []
    base = None
    for i in range(max(0, args.warmup) + args.steps):
        base = cpu_prefill_sample(wl, budget_s=2.0)
        if i >= args.warmup:
            values.append(base["value"])
    value = statistics.mean(values)
    ms = flops / (value * 1e12) * 1e3
    return {
        "metric": "prefill-attn TFLOP/s (causal)", "value": round(value, 6), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic ~N(0,1), numpy PCG64 seed 0",
        "config": prefill_config(world),
        "impl": "reference",
        "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": base["cores"],
                         "kind": "port", "sample": base["sample"]},
        "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the reference ingests prompts position by position in Java "
                "(InferenceEngine.java:88-99); no JDK exists on this box, so its C "
                "restatement (oracle/) is timed on a sample of positions",
    }


def run_reference(args, rank, world):
    key = args.workload
    wl = WORKLOADS[key]
    if key == "c5":
        return run_reference_prefill(args, world)
    if key == "c4q8":
        return {"impl": "reference",
                "unavailable": "the reference keeps FP32 KV caches: it has no Q8 cache path"}
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle  # the reference's CPU path, restated

    oracle.build()
    nh, nkv, hd, L = wl["n_heads"], wl["n_kv"], wl["hd"], wl["layers"]
    threads = min(nh, oracle.max_threads())
    lengths = c3_lengths() if key == "c3" else [wl["T"]]
    esize = 2 if wl["f16"] else 4
    rng = np.random.Generator(np.random.PCG64(0))
    # per layer its own q and caches, RoPE'd as the config says (the layers of
    # a step are visited in turn; host memory bounds how many distinct layer
    # caches are kept: layers beyond that reuse them in rotation)
    layer_bytes = 2 * sum(lengths) * nkv * hd * esize
    n_distinct = max(1, min(L, int(1.2e9 // layer_bytes)))
    cos = sin = None
    if wl["theta"]:
        T = wl["T"]
        cr, ci = oracle.rope_freqs(T, hd, wl["theta"])
        cos = cr.reshape(T, hd // 2)
        sin = ci.reshape(T, hd // 2)
    layers = []
    for _ in range(n_distinct):
        cases = []
        for n in lengths:
            q = rng.standard_normal(nh * hd, dtype=np.float32)
            k = rng.standard_normal((n, nkv * hd), dtype=np.float32)
            v = rng.standard_normal((n, nkv * hd), dtype=np.float32)
            if cos is not None:  # interleaved pairs at each row's own position
                kv_ = k.reshape(n, nkv, hd // 2, 2)
                a, b = kv_[..., 0].copy(), kv_[..., 1].copy()
                c, s = cos[:n, None, :], sin[:n, None, :]
                kv_[..., 0] = a * c - b * s
                kv_[..., 1] = a * s + b * c
                qv = q.reshape(nh, hd // 2, 2)
                a, b = qv[..., 0].copy(), qv[..., 1].copy()
                qv[..., 0] = a * cos[n - 1] - b * sin[n - 1]
                qv[..., 1] = a * sin[n - 1] + b * cos[n - 1]
            if wl["f16"]:
                k, v = k.astype(np.float16).view(np.uint16), v.astype(np.float16).view(np.uint16)
            cases.append((q, k, v, n))
        layers.append(cases)

    def one_layer(l):
        for q, k, v, n in layers[l % n_distinct]:
            if wl["f16"]:
                oracle.decode_f16(q, k, v, nh, nkv, hd, n, n_threads=threads)
            else:
                oracle.decode_f32(q, k, v, nh, nkv, hd, n, n_threads=threads)

    # bound a step to ~2 s of CPU work: run a subset of the layers and scale
    t0 = time.perf_counter()
    one_layer(0)
    t_layer = time.perf_counter() - t0
    layers_per_step = max(1, min(L, int(2.0 / max(t_layer, 1e-6))))
    nxt = 0
    for _ in range(max(0, args.warmup)):
        for _ in range(layers_per_step):
            one_layer(nxt)
            nxt += 1
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        for _ in range(layers_per_step):
            one_layer(nxt)
            nxt += 1
        times.append((time.perf_counter() - t0) * L / layers_per_step)
    ms = statistics.mean(times) * 1e3
    bytes_step = 2 * L * sum(lengths) * nkv * hd * esize
    value = bytes_step / (ms * 1e-3) / 1e9
    sample = (f"{layers_per_step} of {L} layers per step (time scaled to {L}; "
              f"{n_distinct} distinct layer caches), {len(lengths)} sequence(s), "
              f"{threads} threads over heads")
    return {
        "metric": "decode-attn KV-read GB/s", "value": round(value, 4), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "us_per_layer_step": round(ms * 1e3 / L, 2),
        "higher_is_better": True, "scaling": "strong" if key in ("c3", "c4") else "weak",
        "vs_baseline": None,
        "dtype": "f16kv-f32acc" if wl["f16"] else "f32",
        "data": "synthetic ~N(0,1), numpy PCG64 seed 0; RoPE'd q/K where the config says so",
        "config": workload_config(key, world),
        "impl": "reference",
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the reference's attention is Java (InferenceCore.java:105-144); no JDK or "
                "TornadoVM exists on this box, so its C restatement (oracle/) is timed on "
                "the host cores; the whole job's bytes at any N are the same",
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="c4")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="default workload on one GPU: skip the c2 and prefill entries")
    ap.add_argument("--quick", action="store_true",
                    help="profiling runs: no clock soak, no e2e loop, no CPU baseline, no "
                         "parity check, no extras")
    ap.add_argument("--trace", action="store_true",
                    help="decode workloads: add every rank's per-CTA phase timeline of the "
                         "last timed launch (stamps in every launch: a diagnostic run, not "
                         "the headline number)")
    ap.add_argument("--layers", type=int, default=None,
                    help="profiling runs: fewer layers than the workload's (same per-layer "
                         "launch), to keep an ncu capture small")
    args = ap.parse_args()
    if args.layers is not None:
        for wl in WORKLOADS.values():
            wl["layers"] = max(1, min(wl["layers"], args.layers))
    if args.warmup < 3:
        args.warmup = 3  # timing rule: at least 3 warm-up steps

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return 0
        print(json.dumps(run_reference(args, rank, world)), flush=True)
        return 0

    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as tdist

        torch.cuda.set_device(local_rank)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                 device_id=torch.device("cuda", local_rank))
        dist = tdist
    try:
        if args.workload == "c5":
            res = run_prefill(args, rank, world, local_rank, dist)
        elif args.workload == "c4q8":
            res = run_q8(args, rank, world, local_rank, dist)
        else:
            extras = args.workload == "c4" and world == 1 and not (args.quick or args.no_extras)
            res = run_decode(args, args.workload, rank, world, local_rank, dist,
                             cpu_budget=6.0 if extras else 8.0)
            if extras:
                res["c2"] = summary_of(run_decode(args, "c2", rank, world, local_rank, dist,
                                                  cpu_budget=4.0))
                res["prefill"] = summary_of(run_prefill(args, rank, world, local_rank, dist,
                                                        cpu_budget=6.0))
        if rank == 0:
            print(json.dumps(res), flush=True)
    finally:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
