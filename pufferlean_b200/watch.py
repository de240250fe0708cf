"""Host-side liveness of the ranks of a data-parallel update.

A rank that exits or hangs between two updates would leave its peers blocked inside the next
collective. The ranks therefore meet on the host before each launch: a rank about to enqueue update s
records "ready for s" in a key-value store shared by the ranks (the torch.distributed TCPStore the
launcher already created, or any object with `set`, `check` and `wait` of that class) and waits, with
a deadline, until every peer has recorded the same. A peer that exited, or is still stuck in an earlier
update, raises PeerLost naming it before anything is enqueued; the caller then aborts the communicator
(pl_comm_abort) instead of hanging. Collectives already in flight are the watchdog's (pl_comm_wait).
No GPU is involved.
"""
from __future__ import annotations

import datetime
import time


class PeerLost(RuntimeError):
    """A peer rank did not finish an update within the deadline."""

    def __init__(self, step, missing):
        super().__init__(f"rank(s) {missing} did not finish update {step}")
        self.step = step
        self.missing = missing


class RankWatch:
    def __init__(self, store, rank: int, world: int, prefix: str = "pufferlean_b200"):
        self.store, self.rank, self.world, self.prefix = store, rank, world, prefix

    def _key(self, r, step):
        return f"{self.prefix}/ready/{r}/{step}"

    def ready(self, step: int, timeout_s: float) -> None:
        """Records that this rank is about to launch update `step` and returns once every rank has; raises
        PeerLost naming the missing ranks after `timeout_s` otherwise."""
        self.store.set(self._key(self.rank, step), "1")
        keys = [self._key(r, step) for r in range(self.world)]
        t_end = time.monotonic() + timeout_s
        while True:
            missing = [r for r, k in enumerate(keys) if not self.store.check([k])]
            if not missing:
                return
            left = t_end - time.monotonic()
            if left <= 0:
                raise PeerLost(step, missing)
            try:
                self.store.wait([keys[missing[0]]], datetime.timedelta(seconds=min(left, 0.5)))
            except Exception:  # the store's own timeout: poll again until the deadline
                pass
