"""Host logic of the phase-trace summary (gpullama_attn/phase_trace.py) on a
synthetic trace: no GPU."""
import numpy as np

from gpullama_attn import phase_trace


def _trace(n_ctas):
    tr = np.zeros((n_ctas, phase_trace.TRACE_WORDS), dtype=np.uint64)
    for c in range(n_ctas):
        base = 1_000_000 + 100 * c                  # entry, ns
        tr[c, 0] = base
        tr[c, 1] = base + 2_000                     # wait
        tr[c, 2] = base + 3_000                     # q
        tr[c, 3] = base + 3_500                     # first tile
        tr[c, 4] = base + 9_000                     # last tile
        tr[c, 5] = base + 9_500                     # counted
        tr[c, 10] = 4 | (2 << 16)                   # 4 tiles, 2 early
    # CTA 3 is the merger that counted last
    tr[3, 5] = 1_000_000 + 20_000
    tr[3, 6] = 1_000_000 + 22_500
    tr[3, 10] = 4 | (2 << 16) | (1 << 24)
    tr[3, 12] = 1_000_000 + 21_000
    tr[3, 13] = 1_000_000 + 22_000
    tr[3, 14] = 100 | (200 << 16) | (300 << 32) | (400 << 48)
    tr[3, 15] = 1
    return tr.reshape(-1)


def test_summary_phases_and_merger():
    s = phase_trace.summarize(_trace(8), 8, "synthetic")
    assert s["ctas"] == 8 and s["tiles"] == 32 and s["early_tiles"] == 16 and s["mergers"] == 1
    ph = s["us_after_first_entry"]
    assert ph["entry"] == [0.0, 0.35, 0.7]
    assert ph["wait"][0] == 2.0 and ph["last"][2] == 9.7
    # merger-only phases come from the merging CTA alone
    assert ph["merged"] == [22.5, 22.5, 22.5] and ph["gather"] == [21.0, 21.0, 21.0]
    lm = s["last_merger"]
    assert lm["cta"] == 3 and lm["cycles_copy_weights_sums_rest"] == [100, 200, 300, 400]
    assert lm["copy_rounds"] == 1 and lm["counted_to_merged_us"] == 2.5


def test_summary_of_an_untraced_launch():
    assert phase_trace.summarize(np.zeros(16 * 4, dtype=np.uint64), 4)["ctas"] == 0
