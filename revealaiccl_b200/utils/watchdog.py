"""Host-side failure detection for multi-rank runs.

The reference's failure handling is timeouts that raise (the event bridge's
``wait_ready`` after 120 s, worker joins with a timeout; extensions/
r2_event_bridge/integrated_event_bridge.cpp:81-97, scripts/run_r4_a0_c0_full_moe.py:
581-583) and no liveness tracking.  Here every rank also runs a heartbeat:

* ``Heartbeat`` — a daemon thread that writes ``<prefix>/<rank>`` = a counter
  into a ``torch.distributed`` store every ``interval`` seconds and, on each
  tick, reads every peer's counter.  A peer whose counter has not moved for
  ``timeout`` seconds is reported dead (``dead_ranks()``), and a rank that
  leaves cleanly marks itself ``left`` so the others can tell an exit from a
  hang.
* ``check_peers`` raises ``PeerFailure`` naming the dead ranks: a runner calls
  it between steps, before its next launch or collective, so no rank enters a
  collective that a dead peer will never join.

Nothing here touches the GPU; device-side waits are bounded separately (their
status record is read with ``ProgressiveMoELayer.check_status``).
"""

from __future__ import annotations

import threading
import time
from typing import Iterable


class PeerFailure(RuntimeError):
    def __init__(self, dead: Iterable[int], left: Iterable[int] = ()):
        self.dead = sorted(dead)
        self.left = sorted(left)
        super().__init__(f"peer ranks unresponsive: {self.dead}" + (f"; left: {self.left}" if self.left else ""))


class Heartbeat:
    def __init__(self, store, rank: int, world: int, *, interval: float = 0.2, timeout: float = 2.0,
                 prefix: str = "raiccl_hb") -> None:
        self.store, self.rank, self.world = store, int(rank), int(world)
        self.interval, self.timeout, self.prefix = float(interval), float(timeout), prefix
        self._stop = threading.Event()
        self._count = 0
        self._seen: dict[int, tuple[str, float]] = {}
        self._lock = threading.Lock()
        self._thread: threading.Thread | None = None

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def _beat(self) -> None:
        self._count += 1
        self.store.set(self._key(self.rank), str(self._count))

    def _poll(self) -> None:
        now = time.monotonic()
        for r in range(self.world):
            if r == self.rank:
                continue
            try:
                val = self.store.get(self._key(r)).decode() if self._has(r) else ""
            except Exception:
                val = ""
            with self._lock:
                prev = self._seen.get(r)
                if prev is None or prev[0] != val:
                    self._seen[r] = (val, now)

    def _has(self, r: int) -> bool:
        try:
            return bool(self.store.check([self._key(r)]))
        except Exception:
            return False

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                self._beat()
                self._poll()
            except Exception:
                pass  # the store itself went away: peers will be reported by age
            self._stop.wait(self.interval)

    def start(self) -> "Heartbeat":
        self._beat()
        start = time.monotonic()
        with self._lock:
            for r in range(self.world):
                if r != self.rank:
                    self._seen[r] = ("", start)
        self._thread = threading.Thread(target=self._run, name=f"raiccl-heartbeat-{self.rank}", daemon=True)
        self._thread.start()
        return self

    def stop(self, *, leaving: bool = True) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5 * self.interval + 1.0)
        if leaving:
            try:
                self.store.set(self._key(self.rank), "left")
            except Exception:
                pass

    def __enter__(self) -> "Heartbeat":
        return self.start()

    def __exit__(self, *exc) -> None:
        self.stop()

    def left_ranks(self) -> list[int]:
        with self._lock:
            return sorted(r for r, (v, _) in self._seen.items() if v == "left")

    def dead_ranks(self) -> list[int]:
        now = time.monotonic()
        with self._lock:
            return sorted(r for r, (v, t) in self._seen.items() if v != "left" and now - t > self.timeout)

    def check_peers(self) -> None:
        dead, left = self.dead_ranks(), self.left_ranks()
        if dead or left:
            raise PeerFailure(dead, left)


__all__ = ["Heartbeat", "PeerFailure"]
