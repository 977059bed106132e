"""The decode work partition (host run of the kernels' own functions)."""
import numpy as np
import pytest

import gpullama_attn as gla


def check(n_pos, n_kv, tile, n_ctas):
    r = gla.debug_partition(n_pos, n_kv, tile, n_ctas)
    n_pos = [max(0, int(x)) for x in n_pos]
    # expected tile list in (sequence, kv head, tile) order
    exp = [(b, g, j * tile) for b, n in enumerate(n_pos) for g in range(n_kv)
           for j in range((n + tile - 1) // tile)]
    got = list(zip(r["seq"].tolist(), r["kv_head"].tolist(), r["row0"].tolist()))
    assert got == exp
    W = len(exp)
    if W == 0:
        return r
    cta = r["cta"]
    # contiguous, non-decreasing ownership with near-equal counts
    assert np.all(np.diff(cta) >= 0)
    counts = np.bincount(cta, minlength=n_ctas)
    assert counts.max() - counts.min() <= 1 or W < n_ctas
    assert counts.max() == -(-W // n_ctas)
    # one slot per (cta, segment) piece, unique across pieces, within bounds
    pieces = {}
    for c, b, g, s in zip(cta, r["seq"], r["kv_head"], r["slot"]):
        pieces.setdefault((int(c), int(b) * n_kv + int(g)), set()).add(int(s))
    slots = []
    for (c, seg), ss in pieces.items():
        assert ss == {c + seg}
        slots.append(c + seg)
    assert len(slots) == len(set(slots))
    assert max(slots) < n_ctas + len(n_pos) * n_kv
    return r


@pytest.mark.parametrize("n_pos,n_kv,tile,n_ctas", [
    ([4096], 8, 32, 148),          # C2 per layer
    ([512], 8, 16, 148),           # C1
    ([131072], 4, 64, 148),        # C4
    ([1], 8, 16, 148),             # one row
    ([100, 0, 37, 1, 4096], 8, 64, 148),   # ragged, with an empty sequence
    ([0, 0, 5], 2, 16, 3),         # leading empty sequences
    ([5, 0, 0], 2, 16, 7),         # trailing empty sequences
    ([33] * 16, 8, 16, 148),
])
def test_partition_cases(n_pos, n_kv, tile, n_ctas):
    check(n_pos, n_kv, tile, n_ctas)


def test_partition_c3_lengths():
    rng = np.random.Generator(np.random.PCG64(3))
    n_pos = rng.integers(1024, 32768, size=16, endpoint=True)
    r = check(n_pos, 8, 64, 148)
    counts = np.bincount(r["cta"], minlength=148)
    assert counts.max() - counts.min() <= 1


def test_partition_random():
    rng = np.random.Generator(np.random.PCG64(11))
    for _ in range(200):
        B = int(rng.integers(1, 12))
        n_pos = rng.integers(0, 300, size=B)
        n_pos[rng.integers(0, B)] = max(1, n_pos[0])
        check(n_pos, int(rng.integers(1, 9)), int(rng.choice([16, 32, 64])),
              int(rng.integers(1, 160)))
