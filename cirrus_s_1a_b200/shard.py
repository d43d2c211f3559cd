"""Sequence sharding over the GPUs of one box: one process per GPU, no
collective on the data path.

The decode path partitions by independent sequences: a global batch of
``n_seq`` sequences is cut into ``world`` contiguous shards, rank r decodes
shard r on its own GPU with its own weight copy and caches, and the host adds
up the tokens.  Nothing crosses NVLink while sequences decode.

Coordination goes through the process group's key-value store (the
``TCPStore`` that ``torch.distributed`` rendezvous creates), not through
collectives, so a rank that fails cannot leave the others blocked inside one:

* ``heartbeat(step)`` after every step publishes the rank's progress;
* ``failed_peers()`` between steps (before the next launch) lists the ranks
  that reported a failure, so a caller can stop or carry on with its own shard;
* ``report(tokens)`` / ``fail(exc)`` publish the rank's result exactly once;
* ``gather()`` (rank 0) collects every rank's result, waiting at most
  ``timeout_s`` for each; a rank that never reports (it exited or hung) is
  listed as lost instead of blocking the job.

``run_shard`` wraps one rank's work with these steps.
"""

from __future__ import annotations

import json
import time
import traceback
from dataclasses import dataclass, field


def shard_bounds(n_seq: int, world: int, rank: int) -> tuple:
    """[start, stop) of rank's contiguous shard: the first ``n_seq % world``
    ranks take one sequence more than the others."""
    if world < 1 or not 0 <= rank < world or n_seq < 0:
        raise ValueError(f"bad shard request: n_seq={n_seq} world={world} rank={rank}")
    base, extra = divmod(n_seq, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


@dataclass
class ShardResult:
    """What rank 0 collects: the tokens and seconds of every rank that reported."""
    tokens: int = 0
    seconds: float = 0.0            # the slowest reporting rank's device time
    ranks: dict = field(default_factory=dict)   # rank -> its report
    failed: list = field(default_factory=list)  # ranks that reported a failure
    lost: list = field(default_factory=list)    # ranks that never reported

    @property
    def ok(self) -> bool:
        return not self.failed and not self.lost

    @property
    def tokens_per_s(self) -> float:
        return self.tokens / self.seconds if self.seconds > 0 else 0.0


class ShardCoordinator:
    """Host-side coordination of one rank through a ``torch.distributed`` store."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 60.0, prefix: str = "cb_shard"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.prefix = timeout_s, prefix
        self._reported = False

    def _key(self, kind: str, rank: int) -> str:
        return f"{self.prefix}/{kind}/{rank}"

    def heartbeat(self, step: int) -> None:
        self.store.set(self._key("hb", self.rank), str(int(step)))

    def progress(self, rank: int) -> int | None:
        """The last step ``rank`` published, or None before its first heartbeat."""
        k = self._key("hb", rank)
        return int(self.store.get(k)) if self.store.check([k]) else None

    def _read_done(self, rank: int):
        k = self._key("done", rank)
        return json.loads(self.store.get(k)) if self.store.check([k]) else None

    def failed_peers(self) -> list:
        """Ranks (other than this one) that have reported a failure so far; does not block."""
        out = []
        for r in range(self.world):
            if r == self.rank:
                continue
            d = self._read_done(r)
            if d is not None and d["status"] != "ok":
                out.append(r)
        return out

    def report(self, tokens: int, seconds: float, status: str = "ok", **extra) -> None:
        if self._reported:
            return
        self._reported = True
        rec = {"status": status, "tokens": int(tokens), "seconds": float(seconds), **extra}
        self.store.set(self._key("done", self.rank), json.dumps(rec))

    def fail(self, exc: BaseException, tokens: int = 0, seconds: float = 0.0) -> None:
        msg = "".join(traceback.format_exception_only(type(exc), exc)).strip()
        self.report(tokens, seconds, status=f"failed: {msg}")

    def gather(self) -> ShardResult:
        """Rank 0: every rank's report (waiting up to ``timeout_s`` in total)."""
        res = ShardResult()
        deadline = time.monotonic() + self.timeout_s
        pending = set(range(self.world))
        while pending and time.monotonic() < deadline:
            for r in sorted(pending):
                d = self._read_done(r)
                if d is not None:
                    res.ranks[r] = d
                    pending.discard(r)
            if pending:
                time.sleep(0.01)
        res.lost = sorted(pending)
        for r, d in sorted(res.ranks.items()):
            if d["status"] != "ok":
                res.failed.append(r)
            res.tokens += d["tokens"]
            res.seconds = max(res.seconds, d["seconds"])
        return res


def run_shard(coord: ShardCoordinator, n_seq: int, work, stop_on_peer_failure: bool = False) -> tuple:
    """Run ``work(start, stop, between_steps)`` on this rank's shard and report.

    ``work`` decodes sequences [start, stop) and returns (tokens, seconds); it
    calls ``between_steps(step)`` after each step, which publishes the heartbeat
    and returns False when the caller should stop (a peer failed and
    ``stop_on_peer_failure`` is set).  An exception in ``work`` is reported as
    this rank's failure and re-raised.  Returns (start, stop, tokens, seconds).
    """
    start, stop = shard_bounds(n_seq, coord.world, coord.rank)

    def between_steps(step: int) -> bool:
        coord.heartbeat(step)
        return not (stop_on_peer_failure and coord.failed_peers())

    try:
        tokens, seconds = work(start, stop, between_steps)
    except BaseException as exc:
        coord.fail(exc)
        raise
    coord.report(tokens, seconds, start=start, stop=stop)
    return start, stop, tokens, seconds
