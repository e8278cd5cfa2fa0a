"""Host-side liveness of the ranks of a tensor-parallel group, through the rendezvous key-value store.

Every rank bumps its own heartbeat key ``<prefix>/<rank>`` every ``interval_s`` from a background thread.  A rank
that exits cleanly also sets ``<prefix>/left/<rank>``.  A peer whose counter has not moved for ``timeout_s`` (or that
left) is reported by :meth:`HeartbeatWatchdog.dead_peers`; :meth:`check` raises :class:`PeerFailure`.  The serving
daemon calls ``check()`` on rank 0 before it broadcasts the next engine call, so a lost rank is noticed on the host
before the next collective is launched instead of by a collective that never completes; followers, which block
inside the broadcast, get the verdict from the watchdog thread (``on_failure``, called for silent peers only: a
clean leave follows an orderly shutdown).

The reference has no such watchdog: its TP processes block in NCCL until the process-group timeout
(``tp/dist_utils.py``, ``hrm_flash/flash_daemon.py``).
"""
from __future__ import annotations

import threading
import time
from typing import Callable, Dict, List, Optional


class PeerFailure(RuntimeError):
    def __init__(self, dead: List[int], left: List[int]):
        self.dead, self.left = dead, left
        super().__init__(f"tensor-parallel peers lost: no heartbeat from {dead}, left: {left}")


class HeartbeatWatchdog:
    def __init__(self, store, rank: int, world: int, interval_s: float = 0.5, timeout_s: float = 5.0,
                 prefix: str = "hrm_hb", clock: Callable[[], float] = time.monotonic,
                 on_failure: Optional[Callable[[PeerFailure], None]] = None):
        self.store, self.rank, self.world = store, int(rank), int(world)
        self.interval_s, self.timeout_s, self.prefix, self.clock = float(interval_s), float(timeout_s), prefix, clock
        self.on_failure = on_failure
        self._count = 0
        self._seen: Dict[int, tuple] = {}      # peer -> (last counter, local time it last changed)
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self._lock = threading.Lock()
        self._t0 = clock()

    # ---------------------------------------------------------------- own heartbeat
    def beat(self) -> None:
        self._count += 1
        self.store.set(f"{self.prefix}/{self.rank}", str(self._count))

    def start(self) -> "HeartbeatWatchdog":
        self.beat()
        self._thread = threading.Thread(target=self._run, name=f"hb-{self.rank}", daemon=True)
        self._thread.start()
        return self

    def _run(self) -> None:
        while not self._stop.wait(self.interval_s):
            try:
                self.beat()
                if self.on_failure is not None:
                    dead, left = self._scan()
                    if dead:   # a clean leave is reported by check() only (it follows an orderly shutdown)
                        self.on_failure(PeerFailure(dead, left))
                        return
            except Exception:   # the store itself is gone (rank 0 hosts it): treat as a failure of rank 0
                if self.on_failure is not None and self.rank != 0:
                    self.on_failure(PeerFailure([0], []))
                return

    def stop(self, clean: bool = True) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5 * self.interval_s + 1)
        if clean:
            try:
                self.store.set(f"{self.prefix}/left/{self.rank}", "1")
            except Exception:
                pass

    # ---------------------------------------------------------------- peers
    def _read(self, key: str) -> Optional[str]:
        if not self.store.check([key]):
            return None
        v = self.store.get(key)
        return v.decode() if isinstance(v, (bytes, bytearray)) else str(v)

    def _scan(self):
        now = self.clock()
        dead, left = [], []
        with self._lock:
            for r in range(self.world):
                if r == self.rank:
                    continue
                if self._read(f"{self.prefix}/left/{r}") is not None:
                    left.append(r)
                    continue
                v = self._read(f"{self.prefix}/{r}")
                last = self._seen.get(r)
                if last is None or last[0] != v:
                    self._seen[r] = (v, now)
                    last = self._seen[r]
                # a peer that never beat is measured from this watchdog's start
                since = last[1] if v is not None else self._t0
                if now - since > self.timeout_s:
                    dead.append(r)
        return dead, left

    def dead_peers(self) -> List[int]:
        dead, left = self._scan()
        return sorted(dead + left)

    def check(self) -> None:
        dead, left = self._scan()
        if dead or left:
            raise PeerFailure(dead, left)
