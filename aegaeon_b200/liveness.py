"""Host-side liveness of peer workers, checked before launching peer copies.

A migration pulls (or pushes) through another process's GPU memory, mapped
into this process.  If that process has gone, the copy must not be launched.
The reference has no peer copies (its migration is a stub,
aegaeon/worker.py:2420-2451) and ends the actor when fetching a source event
fails (worker.py:2368-2373).  Here every worker publishes a heartbeat in a
``torch.distributed`` key-value store (TCPStore, FileStore, or the process
group's store), and a worker checks its peer's heartbeat before each launch
that touches the peer's memory.  A peer that has left cleanly sets a
departure key; one that died stops beating and is declared gone after
``max_age`` seconds.  Nothing here touches a GPU.
"""

from __future__ import annotations

import threading
import time


class PeerGone(RuntimeError):
    """A peer worker has left or stopped answering."""


class Heartbeat:
    """Publish this worker's heartbeat and check peers'.

    Args:
        store: a ``torch.distributed.Store`` shared by the workers.
        rank: this worker's id in the store's key space.
        interval: seconds between beats (a daemon thread).
    """

    def __init__(self, store, rank: int, interval: float = 0.2, prefix: str = "kvx"):
        self.store = store
        self.rank = rank
        self.interval = interval
        self.prefix = prefix
        self._stop = threading.Event()
        self._beat()
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()

    def _key(self, kind: str, rank: int) -> str:
        return f"{self.prefix}/{kind}/{rank}"

    def _beat(self) -> None:
        self.store.set(self._key("hb", self.rank), repr(time.time()))

    def _run(self) -> None:
        while not self._stop.wait(self.interval):
            try:
                self._beat()
            except Exception:  # noqa: BLE001 - the store went away: stop beating
                return

    def depart(self) -> None:
        """Leave cleanly: peers see this at their next check."""
        self._stop.set()
        self._thread.join(timeout=5)
        self.store.set(self._key("gone", self.rank), "1")

    def stop(self) -> None:
        self._stop.set()
        self._thread.join(timeout=5)

    def check(self, peer: int, max_age: float = 2.0) -> None:
        """Raise PeerGone unless `peer` has beaten within `max_age` seconds."""
        if self.store.check([self._key("gone", peer)]):
            raise PeerGone(f"worker {peer} has left")
        if not self.store.check([self._key("hb", peer)]):
            raise PeerGone(f"worker {peer} never published a heartbeat")
        last = float(self.store.get(self._key("hb", peer)).decode())
        age = time.time() - last
        if age > max_age:
            raise PeerGone(f"worker {peer} silent for {age:.1f} s (limit {max_age} s)")

    def guard(self, peer: int, max_age: float = 2.0):
        """A callable for ``KVSwapper.migrate_blocks(liveness=...)``."""
        return lambda: self.check(peer, max_age)
