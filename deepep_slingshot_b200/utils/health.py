"""Host-side failure detection: peer heartbeats over the process group's store and a watcher of
the kernels' host-mapped error page.

The reference's fault story is fail-fast: bounded device waits write a diagnostic code to a host
page that stays readable after the failure, and a watchdog thread polls it
(backend/tests/diagnostic_watch.py:65-90, backend/host/gin_plugin.cc:220-226). Here the kernels never
trap: a wait that expires writes its code into the error page and returns, and the host raises.
`ErrorWatch` polls that page from a thread so a hung *host* path (for example a rank blocked in a
collective) still learns about the device-side failure, and `Heartbeat` lets every rank notice a
peer process that died or stopped between steps before it launches its next collective.
"""
import threading
import time
from typing import Callable, Dict, List, Optional, Tuple

import torch.distributed as dist


class Heartbeat:
    """Publish `time.time()` under `prefix/rank` in `store` every `interval` seconds (a daemon
    thread) and report peers whose last beat is older than `max_age`."""

    def __init__(self, store: dist.Store, rank: int, world: int, interval: float = 0.5, prefix: str = 'deepep_b200_hb'):
        self.store, self.rank, self.world = store, rank, world
        self.interval, self.prefix = interval, prefix
        self._stop = threading.Event()
        self._beat()
        self._thread = threading.Thread(target=self._run, name=f'deepep-heartbeat-{rank}', daemon=True)
        self._thread.start()

    def _key(self, r: int) -> str:
        return f'{self.prefix}/{r}'

    def _beat(self) -> None:
        self.store.set(self._key(self.rank), repr(time.time()))

    def _run(self) -> None:
        while not self._stop.wait(self.interval):
            try:
                self._beat()
            except Exception:  # the store went away: the group is being torn down
                return

    def last_beats(self) -> Dict[int, Optional[float]]:
        out = {}
        for r in range(self.world):
            key = self._key(r)
            out[r] = float(self.store.get(key).decode()) if self.store.check([key]) else None
        return out

    def stale_ranks(self, max_age: float) -> List[int]:
        now = time.time()
        return [r for r, t in self.last_beats().items() if r != self.rank and (t is None or now - t > max_age)]

    def require_alive(self, max_age: float) -> None:
        """Raise before a collective when a peer has stopped beating."""
        stale = self.stale_ranks(max_age)
        if stale:
            raise RuntimeError(f'rank {self.rank}: peers {stale} stopped heart-beating (> {max_age:.1f} s)')

    def stop(self) -> None:
        self._stop.set()
        self._thread.join(timeout=2 * self.interval + 1)


class ErrorWatch:
    """Poll `buffer.get_error_state()` (a host-mapped page, no device sync) every `interval` seconds;
    the first non-zero code is kept with its time and passed to `on_error`."""

    def __init__(self, buffer, interval: float = 0.05, on_error: Optional[Callable[[Tuple[int, int, int, int]], None]] = None):
        self.buffer, self.interval, self.on_error = buffer, interval, on_error
        self.error: Optional[Tuple[int, int, int, int]] = None
        self.error_time: Optional[float] = None
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, name='deepep-error-watch', daemon=True)
        self._thread.start()

    def _run(self) -> None:
        while not self._stop.wait(self.interval):
            state = tuple(self.buffer.get_error_state())
            if state[0] != 0:
                self.error, self.error_time = state, time.time()
                if self.on_error is not None:
                    self.on_error(state)
                return

    def raise_if_error(self) -> None:
        if self.error is not None:
            code, peer, detail, rank = self.error
            raise RuntimeError(f'device error code {code} on rank {rank} (peer {peer}, detail {detail})')

    def stop(self) -> None:
        self._stop.set()
        self._thread.join(timeout=1)
