"""Host-side failure detection (the reference has none: no heartbeat, no watchdog).

Every rank runs a ``Heartbeat``: a daemon thread writing ``hb/<rank> = <monotonic
timestamp, step>`` into a ``torch.distributed`` key-value store (the rendezvous
``TCPStore``) every ``interval`` seconds.  ``HeartbeatMonitor.stale()`` lists the ranks
whose last beat is older than ``timeout`` (a crashed, hung or departed rank); a training
loop checks it between steps -- never with kernels or collectives in flight -- and
stops (or re-plans with the survivors) instead of blocking in the next collective.
The clock is the store host's: each beat records the writer's wall time and the
monitor compares against its own, so all ranks of one node agree.
"""

from __future__ import annotations

import threading
import time

import torch.distributed as dist


def _key(prefix: str, rank: int) -> str:
    return f"{prefix}/{rank}"


class Heartbeat:
    def __init__(self, store: dist.Store, rank: int, *, interval: float = 1.0, prefix: str = "hb") -> None:
        self.store, self.rank, self.interval, self.prefix = store, rank, interval, prefix
        self.step = 0
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None

    def beat(self) -> None:
        self.store.set(_key(self.prefix, self.rank), f"{time.time():.6f},{self.step}")

    def start(self) -> Heartbeat:
        self.beat()
        self._thread = threading.Thread(target=self._run, name=f"heartbeat-{self.rank}", daemon=True)
        self._thread.start()
        return self

    def _run(self) -> None:
        while not self._stop.wait(self.interval):
            try:
                self.beat()
            except Exception:  # noqa: BLE001 - the store went away: stop beating
                return

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5 * self.interval)


def stale_ranks(store: dist.Store, world: int, timeout: float, *, prefix: str = "hb",
                now: float | None = None) -> list[int]:
    """Ranks whose last beat is older than ``timeout`` s, or that never beat."""
    now = time.time() if now is None else now
    out = []
    for r in range(world):
        k = _key(prefix, r)
        try:
            if not store.check([k]):
                out.append(r)
                continue
            ts = float(store.get(k).decode().split(",")[0])
        except Exception:  # noqa: BLE001
            out.append(r)
            continue
        if now - ts > timeout:
            out.append(r)
    return out


class HeartbeatMonitor:
    def __init__(self, store: dist.Store, world: int, *, timeout: float = 10.0, prefix: str = "hb") -> None:
        self.store, self.world, self.timeout, self.prefix = store, world, timeout, prefix

    def stale(self) -> list[int]:
        return stale_ranks(self.store, self.world, self.timeout, prefix=self.prefix)

    def raise_if_stale(self) -> None:
        bad = self.stale()
        if bad:
            raise RuntimeError(f"ranks {bad} missed their heartbeat for more than {self.timeout:.1f} s")


__all__ = ["Heartbeat", "HeartbeatMonitor", "stale_ranks"]
