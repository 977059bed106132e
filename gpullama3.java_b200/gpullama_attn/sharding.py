"""Host-side work split across GPUs (one process per GPU).

* KV-sequence sharding (long-context decode): rank r of N holds the cache rows
  [r*T//N, (r+1)*T//N) of one sequence; the ranks' shard records are
  all-gathered and merged with the log-sum-exp rule of gla_lse_combine.
* Sequence sharding (batched decode): sequences are dealt to ranks
  longest-first onto the least-loaded rank, so per-rank KV bytes stay even.
"""
from __future__ import annotations


def kv_shard_bounds(n_rows: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous row range [lo, hi) of `rank` (sizes differ by at most one row)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    return rank * n_rows // world, (rank + 1) * n_rows // world


def lpt_assign(lengths, world: int) -> list[list[int]]:
    """Sequence indices per rank: longest first onto the least-loaded rank."""
    if world < 1:
        raise ValueError("world must be >= 1")
    loads = [0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i)):
        r = min(range(world), key=lambda j: (loads[j], j))
        loads[r] += int(lengths[i])
        out[r].append(i)
    return out
