"""Fault tolerance of the colocated loop (--use-fault-tolerance).

EngineSupervisor runs RolloutHealthMonitor over this rank's rollout engine during rollouts
(probe: `RolloutEngine.health_check`, i.e. not marked dead and no kernel reported a failed
bounded wait; interval / timeout / first wait from --rollout-health-check-*). A failed engine
is marked dead and its memory released; before the next rollout `before_rollout` rebuilds it
with the factory and rebinds the client, like the reference's recover_updatable_engines. Under
--ci-test one host-side crash is injected at rollout 1 (the reference's simulate_crash), so
the recovery path runs in CI without faulting a GPU.

With several training ranks a RankHeartbeat publishes liveness into the process-group store;
`check_ranks` raises RankFailure before a step when a peer went silent, instead of every rank
blocking in its next collective.

Reference: miles/ray/rollout.py (health monitoring :399, recover :263-300 / :513-534,
simulate_crash under --ci-test), miles/utils/health_monitor.py.
"""
from __future__ import annotations

import logging

import torch.distributed as dist

from miles_b200.utils.health_monitor import RankHeartbeat, RolloutHealthMonitor

log = logging.getLogger(__name__)


class EngineSupervisor:
    def __init__(self, args, engine, factory, client=None, rank: int = 0, world: int = 1,
                 store=None):
        self.args = args
        self.factory = factory       # factory() -> a new RolloutEngine for this rank
        self.client = client
        self.engine = engine
        self.enabled = bool(getattr(args, "use_fault_tolerance", False))
        self.recoveries = 0
        self.monitor = None
        self.heartbeat = None
        if not self.enabled:
            return
        self.monitor = RolloutHealthMonitor(
            [engine], probe=lambda e: e.health_check(), kill=self._kill,
            interval=float(getattr(args, "rollout_health_check_interval", 30.0) or 30.0),
            timeout=float(getattr(args, "rollout_health_check_timeout", 30.0) or 30.0),
            first_wait=float(getattr(args, "rollout_health_check_first_wait", 0.0) or 0.0))
        self.monitor.pause()
        self.monitor.start()
        if world > 1 and store is not None:
            self.heartbeat = RankHeartbeat(store, rank, world,
                                           timeout=float(getattr(args, "rollout_health_check_timeout", 30.0) or 30.0))
            self.heartbeat.start(1.0)

    @staticmethod
    def _kill(engine):
        engine.dead = True
        try:
            engine.abort()
            engine.release_memory()
        except Exception:  # noqa: BLE001 - a dead engine may fail to release cleanly
            pass

    def simulate_crash(self):
        """Host-side crash injection: the engine is marked dead as a failed probe would."""
        self._kill(self.engine)
        if self.monitor is not None:
            self.monitor.engines[0] = None
            self.monitor.failures.append(0)

    def before_rollout(self, rollout_id: int):
        """Recover a dead engine (rebuilt by the factory, client rebound), then monitor."""
        if not self.enabled:
            return self.engine
        if getattr(self.args, "ci_test", False) and rollout_id == 1 and self.recoveries == 0:
            self.simulate_crash()
        self.check_ranks()
        if self.engine.dead:
            self.monitor.engines[0] = None
        if self.monitor.engines[0] is None:
            self.monitor.recover(lambda i: self.factory())
            self.engine = self.monitor.engines[0]
            if self.client is not None:
                self.client.engine = self.engine
            self.recoveries += 1
            log.warning("recovered the rollout engine before rollout %d", rollout_id)
        self.monitor.resume()
        return self.engine

    def after_rollout(self):
        if self.monitor is not None:
            self.monitor.pause()

    def check_ranks(self):
        if self.heartbeat is not None:
            self.heartbeat.check()

    def close(self):
        if self.monitor is not None:
            self.monitor.stop()
        if self.heartbeat is not None:
            self.heartbeat.mark_exiting()
            self.heartbeat.stop()


def default_store():
    if dist.is_initialized():
        try:
            return dist.distributed_c10d._get_default_store()
        except Exception:  # noqa: BLE001
            return None
    return None
