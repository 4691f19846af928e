"""Failure detection between ranks, on the host.

The reference has none: when one role dies the other blocks in NCCL until an
operator kills it (its docs say so). Here three mechanisms bound that wait:

1. the process group has a finite timeout (``DistributedConfig.timeout_s``),
   so a collective or a p2p receive whose peer is gone ends with an error;
2. device-side flag waits of the fused transport are bounded and report a
   status word that ``Transport.check()`` turns into ``AFDCommTimeout``;
3. ``PeerMonitor`` -- this file -- lets the ranks learn of a failure *before*
   their next launch: a rank that fails writes the reason under a key of the
   rendezvous store, and every rank publishes a heartbeat. A background
   thread polls both; ``check()`` (called between steps) only reads the
   thread's verdict, so the per-step cost is a Python attribute read.

A rank that exits without reporting is caught by its heartbeat going stale.
"""

from __future__ import annotations

import logging
import threading
import time
from typing import List, Optional

logger = logging.getLogger(__name__)

FAIL_KEY = "afd/failure"


class AFDPeerFailure(RuntimeError):
    """Another rank reported a failure or stopped sending heartbeats."""


class PeerMonitor:
    def __init__(self, store, rank: int, world_size: int, interval_s: float = 0.2,
                 dead_after_s: float = 5.0):
        self.store = store
        self.rank = rank
        self.world = world_size
        self.interval = interval_s
        self.dead_after = dead_after_s
        self.verdict: Optional[str] = None
        self._stop = threading.Event()
        self._last_seen = {r: time.monotonic() for r in range(world_size)}
        self._last_val = {r: None for r in range(world_size)}
        self._beat = 0
        self._thread = threading.Thread(target=self._loop, name="afd-peer-monitor", daemon=True)
        self._thread.start()

    # ------------------------------------------------------------------
    def _hb_key(self, r: int) -> str:
        return f"afd/hb/{r}"

    def _loop(self) -> None:
        while not self._stop.wait(self.interval):
            try:
                self._beat += 1
                self.store.set(self._hb_key(self.rank), str(self._beat))
                if self.store.check([FAIL_KEY]):
                    reason = self.store.get(FAIL_KEY).decode()
                    if not reason.startswith(f"rank {self.rank}:"):
                        self.verdict = f"peer failure reported: {reason}"
                now = time.monotonic()
                for r in range(self.world):
                    if r == self.rank:
                        continue
                    k = self._hb_key(r)
                    if not self.store.check([k]):
                        v = None
                    else:
                        v = self.store.get(k)
                    if v != self._last_val[r]:
                        self._last_val[r] = v
                        self._last_seen[r] = now
                    elif now - self._last_seen[r] > self.dead_after and self.verdict is None:
                        self.verdict = (f"rank {r} sent no heartbeat for "
                                        f"{now - self._last_seen[r]:.1f} s")
            except Exception as e:  # the store itself went away (rank 0 died)
                if self.verdict is None and not self._stop.is_set():
                    self.verdict = f"rendezvous store unreachable: {e}"

    # ------------------------------------------------------------------
    def check(self) -> None:
        if self.verdict is not None:
            raise AFDPeerFailure(self.verdict)

    def report(self, reason: str) -> None:
        """Publish this rank's failure so the others stop before their next
        launch."""
        try:
            self.store.set(FAIL_KEY, f"rank {self.rank}: {reason}")
        except Exception as e:  # pragma: no cover - store gone
            logger.warning(f"could not report failure: {e}")

    def stop(self) -> None:
        self._stop.set()
        self._thread.join(timeout=2 * self.interval + 1.0)


def live_ranks(monitor: PeerMonitor) -> List[int]:
    now = time.monotonic()
    return [r for r in range(monitor.world)
            if r == monitor.rank or now - monitor._last_seen[r] <= monitor.dead_after]
