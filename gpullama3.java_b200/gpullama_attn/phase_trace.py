"""Per-phase timeline of decode launches (the context's phase trace).

With option OPT_TRACE set when a decode call is launched (or captured into a
CUDA graph), every CTA stamps %globaltimer at fixed points of its life; this
module turns the stamps of the last traced launch into a per-phase summary:
for each phase the earliest, median and latest CTA, in microseconds after the
first CTA entered the kernel, plus the merge statistics of the merging CTAs.

Phases (slots of a CTA's 16-word record, csrc/decode_kernel.cuh kTr*):
entry, wait (dependency wait returned), q (q in shared memory), first / last
(first tile ready / last tile consumed), counted (piece stored and counted),
merged (merger wrote the segment), published (sharded: every rank's records
merged), pfirst / plast (producer's first copy after the wait / last copy),
exit, gather / folded (merger: pieces copied in / folded).

Run as a script to trace the single-GPU launch shapes of the benchmark
configurations (a config-2 layer, a config-4 layer and the config-4 shard
shapes of 4 and 8 ranks, launched without the exchange):

    python gpullama3.java_b200/gpullama_attn/phase_trace.py
"""
import json
import os
import sys

import numpy as np

PHASES = {0: "entry", 1: "wait", 2: "q", 3: "first", 4: "last", 5: "counted", 6: "merged",
          7: "published", 8: "pfirst", 9: "plast", 11: "exit", 12: "gather", 13: "folded"}
_MERGER_ONLY = ("merged", "published", "gather", "folded")
TRACE_WORDS = 16  # words a CTA


def summarize(words, n_ctas, tag=""):
    """Summary dict of a launch's trace (`words`: the uint64 words read back
    with Context.debug_trace(), `n_ctas` the launch's grid)."""
    tr = np.asarray(words, dtype=np.uint64)[: n_ctas * TRACE_WORDS]
    tr = tr.reshape(-1, TRACE_WORDS).astype(np.int64)
    info = tr[:, 10]
    merger = ((info >> 24) & 0xFF) == 1
    stamped = tr[:, 0] > 0
    if not stamped.any():
        return {"tag": tag, "ctas": 0}
    t0 = tr[stamped, 0].min()
    out = {"tag": tag, "ctas": int(stamped.sum()), "tiles": int((info & 0xFFFF).sum()),
           "early_tiles": int(((info >> 16) & 0xFF).sum()), "mergers": int(merger.sum()),
           "us_after_first_entry": {}}
    for c, name in PHASES.items():
        ok = tr[:, c] > 0
        if name in _MERGER_ONLY:
            ok = ok & merger
        if ok.any():
            v = (tr[ok, c] - t0) / 1000.0
            out["us_after_first_entry"][name] = [round(float(v.min()), 2),
                                                 round(float(np.median(v)), 2),
                                                 round(float(v.max()), 2)]
    idx = np.nonzero(merger & (tr[:, 5] > 0))[0]
    if idx.size:
        last = idx[np.argmax(tr[idx, 5])]  # the merger that counted last
        c = int(tr[last, 14])
        out["last_merger"] = {
            "cta": int(last),
            "cycles_copy_weights_sums_rest": [c & 0xFFFF, (c >> 16) & 0xFFFF, (c >> 32) & 0xFFFF,
                                              (c >> 48) & 0xFFFF],
            "copy_rounds": int(tr[last, 15]),
            "counted_to_merged_us": round((tr[last, 6] - tr[last, 5]) / 1e3, 3)}
    return out


def summarize_ctx(ctx, tag=""):
    """Summary of the last traced launch of a Context."""
    tr = ctx.debug_trace()
    return summarize(tr.reshape(-1), tr.shape[0], tag)


def _trace_shape(gla, torch, ctx, stream, tag, layers, nh, nkv, hd, rows, f16):
    """Graph of `layers` decode launches of one shape; traced replays; the
    summary of the last launch."""
    dt = torch.float16 if f16 else torch.float32
    with torch.cuda.stream(stream):
        K = torch.randn(layers, rows, nkv * hd, device="cuda").to(dt)
        V = torch.randn(layers, rows, nkv * hd, device="cuda").to(dt)
        q = torch.randn(layers, nh * hd, device="cuda")
        xb = torch.empty(layers, nh * hd, device="cuda")
    torch.cuda.synchronize()

    def step():
        for layer in range(layers):
            ctx.decode(q[layer], K[layer], V[layer], xb[layer], nh, nkv, hd, rows, f16_cache=f16)

    with torch.cuda.stream(stream):
        step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        step()
    for _ in range(5):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(20):
            g.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    s = summarize(ctx.debug_trace(), torch.cuda.get_device_properties(0).multi_processor_count, tag)
    s["shape"] = {"layers": layers, "n_heads": nh, "n_kv_heads": nkv, "head_dim": hd,
                  "rows": rows, "kv": "f16" if f16 else "f32"}
    s["us_per_launch_traced"] = round(e0.elapsed_time(e1) / 20 * 1e3 / layers, 3)
    if ctx.device_status() != 0:
        raise RuntimeError(f"device status {ctx.device_status()} after tracing {tag}")
    del g
    return s


def main():
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch
    import gpullama_attn as gla

    torch.cuda.set_device(0)
    stream = torch.cuda.Stream()
    ctx = gla.Context(0, stream.cuda_stream)
    ctx.set_option(gla.OPT_TRACE, 1)
    try:
        for args in (("c2_layer", 28, 24, 8, 128, 4096, False),
                     ("c4_layer", 4, 28, 4, 128, 131072, True),
                     ("c4_shard_of_4", 28, 28, 4, 128, 32768, True),
                     ("c4_shard_of_8", 28, 28, 4, 128, 16384, True)):
            print(json.dumps(_trace_shape(gla, torch, ctx, stream, *args)))
    finally:
        ctx.set_option(gla.OPT_TRACE, 0)
        ctx.close()


if __name__ == "__main__":
    main()
