"""Host-side failure detection between steps.

The device side of this library never hangs: every wait is bounded and
reports a timeout (``NumaAwareAllReduce.check``). What it cannot tell is
*why* a peer did not arrive. :class:`PeerMonitor` answers that on the host,
before the next launch: every rank publishes a heartbeat counter in the job's
c10d store (the one ``torch.distributed`` already rendezvoused on), and a rank
whose counter stops moving for ``timeout_s`` is reported dead; a rank that
leaves on purpose says so and is reported as left. A caller checks
:meth:`PeerMonitor.assert_healthy` between steps and falls back (or stops)
instead of launching a collective a peer will never join.

The reference has no failure detection (its barrier spins are unbounded, so
one dead peer hangs every GPU: src/numa_all_reduce.cu:177,202).
"""

from __future__ import annotations

import threading
import time


class PeerLost(RuntimeError):
    """A peer stopped heart-beating or left the job."""

    def __init__(self, dead: list[int], left: list[int]):
        self.dead, self.left = dead, left
        parts = []
        if dead:
            parts.append(f"ranks {dead} stopped responding")
        if left:
            parts.append(f"ranks {left} left the job")
        super().__init__("; ".join(parts))


class PeerMonitor:
    """Heartbeats of the ranks of one job through a c10d ``Store``.

    Args:
        store: any ``torch.distributed.Store`` shared by the ranks (TCPStore,
            FileStore, or ``dist.distributed_c10d._get_default_store()``).
        rank, world_size: this rank and the number of ranks.
        interval_s: period of the background heartbeat (``start``); a caller
            may also :meth:`beat` by hand between steps.
        timeout_s: a peer whose counter has not changed for this long (as seen
            by this rank's clock, so no clock agreement is needed) is dead.
    """

    def __init__(self, store, rank: int, world_size: int, interval_s: float = 0.5, timeout_s: float = 5.0,
                 prefix: str = "nab/health"):
        if timeout_s <= interval_s:
            raise ValueError("timeout_s must exceed interval_s")
        self.store, self.rank, self.world_size = store, rank, world_size
        self.interval_s, self.timeout_s, self.prefix = interval_s, timeout_s, prefix
        self._count = 0
        self._seen: dict[int, tuple[bytes | None, float]] = {}
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None
        self._t0 = time.monotonic()
        self.beat()

    # ------------------------------------------------------------ publish --
    def _key(self, r: int, what: str = "beat") -> str:
        return f"{self.prefix}/{r}/{what}"

    def beat(self) -> None:
        self._count += 1
        self.store.set(self._key(self.rank), str(self._count))

    def start(self) -> "PeerMonitor":
        """Heart-beats every ``interval_s`` from a daemon thread."""
        if self._thread is None:
            self._thread = threading.Thread(target=self._run, name="nab-heartbeat", daemon=True)
            self._thread.start()
        return self

    def _run(self) -> None:
        while not self._stop.wait(self.interval_s):
            try:
                self.beat()
            except Exception:  # the store went away: the job is ending
                return

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5 * self.interval_s)
            self._thread = None

    def leave(self) -> None:
        """Announces a clean exit (call between steps, with nothing in flight)."""
        self.stop()
        self.store.set(self._key(self.rank, "left"), "1")

    # -------------------------------------------------------------- query --
    def _peek(self, key: str) -> bytes | None:
        try:
            if not self.store.check([key]):
                return None
            return self.store.get(key)
        except Exception:
            return None

    def status(self) -> tuple[list[int], list[int]]:
        """(dead ranks, ranks that left), as seen now. A peer is judged from
        this rank's first look at it on (a rank that never beat: from this
        monitor's start), so call it every step, not once at the end."""
        now = time.monotonic()
        dead, left = [], []
        for r in range(self.world_size):
            if r == self.rank:
                continue
            if self._peek(self._key(r, "left")) is not None:
                left.append(r)
                continue
            val = self._peek(self._key(r))
            prev = self._seen.get(r)
            if prev is None:  # first look: a rank that never beat counts from our start
                self._seen[r] = (val, now if val is not None else self._t0)
            elif val != prev[0]:
                self._seen[r] = (val, now)
            since = now - self._seen[r][1]
            if since > self.timeout_s:
                dead.append(r)
        return dead, left

    def dead_ranks(self) -> list[int]:
        return self.status()[0]

    def assert_healthy(self) -> None:
        """Raises :class:`PeerLost` if a peer is dead or left."""
        dead, left = self.status()
        if dead or left:
            raise PeerLost(dead, left)

    def __enter__(self):
        return self.start()

    def __exit__(self, *exc):
        self.stop()
