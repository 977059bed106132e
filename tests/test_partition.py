"""The decode work partition, run on the host through the same functions the
kernel uses (gla_debug_partition): 16-row units dealt to CTAs in contiguous,
near-equal ranges, walked in tiles that never cross a (sequence, kv head)
segment."""
import numpy as np
import pytest

import gpullama_attn as gla


def check(n_pos, n_kv, tile, n_ctas, unit=16):
    r = gla.debug_partition(n_pos, n_kv, tile, n_ctas, unit)
    n_pos = [max(0, int(x)) for x in n_pos]
    # every row of every segment is covered exactly once, in order
    covered = {}
    for s, g, r0, nr in zip(r["seq"], r["kv_head"], r["row0"], r["rows"]):
        assert 0 < nr <= tile and r0 % unit == 0
        covered.setdefault((int(s), int(g)), []).append((int(r0), int(nr)))
    for b, n in enumerate(n_pos):
        for g in range(n_kv):
            spans = covered.get((b, g), [])
            if n == 0:
                assert not spans
                continue
            pos = 0
            for r0, nr in spans:
                assert r0 == pos
                pos += nr
            assert pos == n, (b, g, spans)
    if len(r["cta"]) == 0:
        return r
    cta = r["cta"]
    assert np.all(np.diff(cta) >= 0)  # contiguous ranges in CTA order
    units = np.zeros(n_ctas, dtype=np.int64)
    for c, nr in zip(cta, r["rows"]):
        units[c] += -(-int(nr) // unit)
    total = units.sum()
    assert units.max() - units.min() <= 1 or total < n_ctas
    assert units.max() == -(-total // n_ctas)
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
    ([4096], 8, 64, 148),          # C2 per layer
    ([512], 8, 64, 148),           # C1
    ([131072], 4, 64, 148),        # C4
    ([1], 8, 64, 148),             # one row
    ([100, 0, 37, 1, 4096], 8, 64, 148),   # ragged, with an empty sequence
    ([0, 0, 5], 2, 16, 3),         # leading empty sequences
    ([5, 0, 0], 2, 32, 7),         # trailing empty sequences
    ([33] * 16, 8, 64, 148),
])
def test_partition_cases(n_pos, n_kv, tile, n_ctas):
    check(n_pos, n_kv, tile, n_ctas)


def test_partition_c2_balance_is_one_unit():
    r = check([4096], 8, 64, 148)
    rows = np.bincount(r["cta"], weights=r["rows"], minlength=148)
    assert rows.max() - rows.min() <= 16


def test_partition_c3_lengths():
    rng = np.random.Generator(np.random.PCG64(3))
    n_pos = rng.integers(1024, 32768, size=16, endpoint=True)
    check(n_pos, 8, 64, 148)


def test_partition_random():
    rng = np.random.Generator(np.random.PCG64(11))
    for _ in range(200):
        B = int(rng.integers(1, 12))
        n_pos = rng.integers(0, 300, size=B)
        n_pos[rng.integers(0, B)] = max(1, n_pos[0])
        tile = int(rng.choice([16, 32, 64]))
        unit = int(rng.choice([u for u in (16, 32, 64) if tile % u == 0]))
        check(n_pos, int(rng.integers(1, 9)), tile, int(rng.integers(1, 160)), unit)


def test_partition_whole_tile_units():
    check([4096], 8, 64, 148, 64)
    check([100, 0, 37, 1, 4096], 8, 64, 148, 64)
