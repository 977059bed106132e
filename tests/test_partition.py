"""The decode work partition, run on the host through the same functions the
kernel uses (gla_debug_partition): units of `unit` rows dealt to CTAs --
contiguous near-equal ranges over the (sequence, kv head, unit) order for
batches, whole CTA groups per kv head for one sequence -- and walked in tiles
that never cross a (sequence, kv head) segment."""
import numpy as np
import pytest

import gpullama_attn as gla


def check(n_pos, n_kv, tile, n_ctas, unit=64):
    r = gla.debug_partition(n_pos, n_kv, tile, n_ctas, unit)
    n_pos = [max(0, int(x)) for x in n_pos]
    per_segment = len(n_pos) == 1 and n_kv <= n_ctas and n_pos[0] > 0
    # every row of every segment is covered exactly once (one sequence with
    # n_kv <= CTAs: CTA j of a kv head's group of S takes tiles j, j+S, ...;
    # otherwise contiguous ranges walked in order)
    covered = {}
    for c, s, g, r0, nr in zip(r["cta"], r["seq"], r["kv_head"], r["row0"], r["rows"]):
        assert 0 < nr <= tile and r0 % unit == 0
        covered.setdefault((int(s), int(g)), []).append((int(r0), int(nr)))
    for b, n in enumerate(n_pos):
        for g in range(n_kv):
            spans = covered.get((b, g), [])
            if n == 0:
                assert not spans
                continue
            if not per_segment:  # contiguous deal: the walk order is the row order
                assert [r0 for r0, _ in spans] == sorted(r0 for r0, _ in spans)
            pos = 0
            for r0, nr in sorted(spans):
                assert r0 == pos
                pos += nr
            assert pos == n, (b, g, spans)
    if per_segment:
        # round robin: a CTA's tiles are S tiles apart, and which tiles a CTA
        # owns does not depend on the length (a prefix of its infinite list)
        by_cta = {}
        for c, g, r0 in zip(r["cta"], r["kv_head"], r["row0"]):
            by_cta.setdefault(int(c), []).append((int(g), int(r0) // unit))
        groups = {}
        for c, lst in by_cta.items():
            assert len({g for g, _ in lst}) == 1
            groups.setdefault(lst[0][0], []).append(c)
        for g, cs in groups.items():
            cs = sorted(cs)
            lo, S = cs[0], n_ctas // n_kv + (1 if g < n_ctas % n_kv else 0)
            for c in cs:
                j = c - lo
                assert [t for _, t in by_cta[c]] == list(range(j, j + S * len(by_cta[c]), S))
    if len(r["cta"]) == 0:
        return r
    cta = r["cta"]
    assert np.all(np.diff(cta) >= 0)  # each CTA's tiles in walk order
    units = np.zeros(n_ctas, dtype=np.int64)
    for c, nr in zip(cta, r["rows"]):
        units[c] += -(-int(nr) // unit)
    total = units.sum()
    # pieces: one slot per (cta, segment), unique, within bounds; the merge's
    # (first CTA, count) view equals the CTAs that really hold a piece
    pieces, holders, view = {}, {}, {}
    for c, b, g, s, c0, npc in zip(cta, r["seq"], r["kv_head"], r["slot"], r["first_cta"],
                                   r["npieces"]):
        seg = int(b) * n_kv + int(g)
        pieces.setdefault((int(c), seg), set()).add(int(s))
        holders.setdefault(seg, set()).add(int(c))
        view.setdefault(seg, set()).add((int(c0), int(npc)))
    slots = []
    for (c, seg), ss in pieces.items():
        assert ss == {c + seg}
        slots.append(c + seg)
    assert len(slots) == len(set(slots))
    assert max(slots) < n_ctas + len(n_pos) * n_kv
    for seg, cs in holders.items():
        assert len(view[seg]) == 1
        c0, npc = view[seg].pop()
        assert cs == set(range(c0, c0 + npc)), (seg, sorted(cs), c0, npc)
    if per_segment:
        # one piece per CTA; shares within a kv head differ by at most a unit
        per_cta = {}
        for (c, seg) in pieces:
            per_cta.setdefault(c, set()).add(seg)
        assert all(len(v) == 1 for v in per_cta.values())
        nu = -(-n_pos[0] // unit)
        for seg, cs in holders.items():
            u = [units[c] for c in cs]
            assert max(u) - min(u) <= 1
        assert units.max() <= -(-nu // (n_ctas // n_kv))
    else:
        assert units.max() - units.min() <= 1 or total < n_ctas
        assert units.max() == -(-total // n_ctas)
    return r


@pytest.mark.parametrize("n_pos,n_kv,tile,n_ctas", [
    ([4096], 8, 64, 148),          # C2 per layer
    ([512], 8, 64, 148),           # C1
    ([131072], 4, 64, 148),        # C4
    ([1], 8, 64, 148),             # one row
    ([4096], 32, 64, 148),         # MHA, n_kv does not divide the CTAs
    ([4096], 8, 64, 5),            # fewer CTAs than kv heads: contiguous deal
    ([100, 0, 37, 1, 4096], 8, 64, 148),   # ragged, with an empty sequence
    ([0, 0, 5], 2, 16, 3),         # leading empty sequences
    ([5, 0, 0], 2, 32, 7),         # trailing empty sequences
    ([33] * 16, 8, 64, 148),
])
def test_partition_cases(n_pos, n_kv, tile, n_ctas):
    check(n_pos, n_kv, tile, n_ctas, min(tile, 64))


def test_partition_c2_one_piece_per_cta():
    r = check([4096], 8, 64, 148)
    rows = np.bincount(r["cta"], weights=r["rows"], minlength=148)
    assert rows.max() == 4 * 64 and rows.min() == 3 * 64


def test_partition_c3_lengths():
    rng = np.random.Generator(np.random.PCG64(3))
    n_pos = rng.integers(1024, 32768, size=16, endpoint=True)
    check(n_pos, 8, 64, 148)


def test_partition_random():
    rng = np.random.Generator(np.random.PCG64(11))
    for _ in range(300):
        B = int(rng.integers(1, 12))
        n_pos = rng.integers(0, 300, size=B)
        n_pos[rng.integers(0, B)] = max(1, n_pos[0])
        tile = int(rng.choice([16, 32, 64]))
        unit = int(rng.choice([u for u in (16, 32, 64) if tile % u == 0]))
        check(n_pos, int(rng.integers(1, 9)), tile, int(rng.integers(1, 160)), unit)
