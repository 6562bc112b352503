"""Failure detection and recovery (host side).

RolloutHealthMonitor: one thread per engine group. After `first_wait`, every `interval` seconds
it calls each engine's health probe with a `timeout`; an engine that fails is shut down via its
kill callback and its slot is marked dead (None). Monitoring pauses around offload / weight
updates. `recover(factory)` restarts dead slots (the next weight update then re-onloads them).

RankHeartbeat: every training rank publishes a heartbeat into the torch.distributed store;
`check()` on any rank raises RankFailure when a peer has been silent longer than `timeout`,
before the next collective is launched (so nobody blocks inside NCCL waiting for a dead peer).

Neither component faults a GPU: failures are detected purely on the host (missed heartbeats,
probes that raise or time out).

Reference: miles/utils/health_monitor.py:10-177, miles/ray/rollout.py recover (:263-300,
:513-534), --use-fault-tolerance / --rollout-health-check-* flags.
"""
from __future__ import annotations

import concurrent.futures as cf
import threading
import time
from typing import Callable


class RolloutHealthMonitor:
    def __init__(self, engines: list, probe: Callable, kill: Callable | None = None,
                 interval: float = 30.0, timeout: float = 30.0, first_wait: float = 0.0):
        self.engines = engines          # list of engine handles; a dead slot becomes None
        self.probe = probe              # probe(engine) -> bool (may raise / hang)
        self.kill = kill                # kill(engine) on failure
        self.interval, self.timeout, self.first_wait = interval, timeout, first_wait
        self._stop = threading.Event()
        self._paused = threading.Event()
        self._thread: threading.Thread | None = None
        self._pool = cf.ThreadPoolExecutor(max_workers=max(1, len(engines)))
        self.failures: list[int] = []

    def start(self):
        if self._thread is None:
            self._thread = threading.Thread(target=self._loop, daemon=True)
            self._thread.start()

    def stop(self):
        self._stop.set()
        if self._thread:
            self._thread.join(timeout=self.interval + self.timeout + 1)

    def pause(self):
        self._paused.set()

    def resume(self):
        self._paused.clear()

    def _loop(self):
        if self._stop.wait(self.first_wait):
            return
        while not self._stop.is_set():
            if not self._paused.is_set():
                self.check_once()
            self._stop.wait(self.interval)

    def check_once(self) -> list[int]:
        dead = []
        futs = {i: self._pool.submit(self.probe, e) for i, e in enumerate(self.engines) if e is not None}
        for i, f in futs.items():
            try:
                ok = bool(f.result(timeout=self.timeout))
            except Exception:
                ok = False
            if not ok:
                dead.append(i)
        for i in dead:
            eng = self.engines[i]
            if self.kill is not None and eng is not None:
                try:
                    self.kill(eng)
                except Exception:
                    pass
            self.engines[i] = None
            self.failures.append(i)
        return dead

    def recover(self, factory: Callable[[int], object]) -> list[int]:
        """Restart every dead slot with factory(slot_index); returns the restarted slots."""
        restarted = []
        for i, e in enumerate(self.engines):
            if e is None:
                self.engines[i] = factory(i)
                restarted.append(i)
        return restarted


class RankFailure(RuntimeError):
    pass


class RankHeartbeat:
    def __init__(self, store, rank: int, world: int, timeout: float = 30.0, prefix: str = "hb"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout, self.prefix = timeout, prefix
        self._stop = threading.Event()
        self._t: threading.Thread | None = None

    def beat(self):
        self.store.set(f"{self.prefix}/{self.rank}", repr(time.time()))

    def start(self, period: float = 1.0):
        def loop():
            while not self._stop.is_set():
                self.beat()
                self._stop.wait(period)

        self.beat()
        self._t = threading.Thread(target=loop, daemon=True)
        self._t.start()

    def stop(self):
        self._stop.set()

    def mark_exiting(self):
        """Announce a clean departure between steps."""
        self.store.set(f"{self.prefix}/{self.rank}", "exit")

    def check(self) -> None:
        now = time.time()
        for r in range(self.world):
            if r == self.rank:
                continue
            try:
                v = self.store.get(f"{self.prefix}/{r}").decode()
            except Exception:
                raise RankFailure(f"rank {r} never published a heartbeat")
            if v == "exit":
                raise RankFailure(f"rank {r} left the job")
            if now - float(v) > self.timeout:
                raise RankFailure(f"rank {r} silent for {now - float(v):.1f}s")
