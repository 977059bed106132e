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


class RankLost(RuntimeError):
    """A rank did not reach a sharded step within the host timeout."""

    def __init__(self, missing, step):
        self.missing = list(missing)
        self.step = step
        super().__init__(f"ranks {self.missing} did not reach sharded step {step}")


class StepBarrier:
    """Host-side liveness check before every sharded decode step.

    Every rank announces step `s` in the process group's key-value store and
    waits, at most `timeout_s`, until every other rank has announced it too.
    A rank that left (or hangs on the host) is detected here, before this
    rank launches a kernel whose exchange would wait for it on the device:
    enter() raises RankLost naming the missing ranks.  The peer exchange's
    device-side wait (1 s bound, GLA_ERR_TIMEOUT) and the NCCL watchdog
    (gla_comm_wait) remain the last line behind it.
    """

    def __init__(self, store, world: int, rank: int, timeout_s: float = 5.0,
                 poll_s: float = 0.002, prefix: str = "gla/step"):
        if world < 1 or not 0 <= rank < world:
            raise ValueError("bad world/rank")
        self.store, self.world, self.rank = store, world, rank
        self.timeout_s, self.poll_s, self.prefix = timeout_s, poll_s, prefix

    def _key(self, step, r):
        return f"{self.prefix}/{step}/{r}"

    def enter(self, step: int):
        import time

        self.store.set(self._key(step, self.rank), "1")
        missing = [r for r in range(self.world) if r != self.rank]
        deadline = time.monotonic() + self.timeout_s
        while True:
            missing = [r for r in missing if not self.store.check([self._key(step, r)])]
            if not missing:
                return
            if time.monotonic() > deadline:
                raise RankLost(missing, step)
            time.sleep(self.poll_s)
