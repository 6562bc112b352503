"""Host-side failure detection: engine health monitor with a failing / hanging engine, and rank
heartbeats over a gloo world where one rank leaves between steps. No GPU is involved."""
import os
import subprocess
import sys
import time

import pytest

from tests.conftest import free_port

from miles_b200.utils.health_monitor import RankFailure, RankHeartbeat, RolloutHealthMonitor

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


class FakeEngine:
    def __init__(self, mode="ok"):
        self.mode, self.killed = mode, False

    def health(self):
        if self.mode == "raise":
            raise ConnectionError("dropped")
        if self.mode == "hang":
            time.sleep(5)
        return self.mode == "ok"


def test_monitor_kills_and_recovers():
    engines = [FakeEngine(), FakeEngine("raise"), FakeEngine("hang"), FakeEngine("bad")]
    mon = RolloutHealthMonitor(engines, probe=lambda e: e.health(),
                               kill=lambda e: setattr(e, "killed", True), interval=0.05, timeout=0.3)
    dead = mon.check_once()
    assert sorted(dead) == [1, 2, 3]
    assert engines[0] is not None and all(engines[i] is None for i in (1, 2, 3))
    restarted = mon.recover(lambda i: FakeEngine())
    assert restarted == [1, 2, 3]
    assert mon.check_once() == []


def test_monitor_thread_pause_resume():
    engines = [FakeEngine("raise")]
    mon = RolloutHealthMonitor(engines, probe=lambda e: e.health(), interval=0.02, timeout=0.2)
    mon.pause()
    mon.start()
    time.sleep(0.1)
    assert engines[0] is not None  # paused: no checks
    mon.resume()
    t0 = time.time()
    while engines[0] is not None and time.time() - t0 < 3:
        time.sleep(0.02)
    mon.stop()
    assert engines[0] is None


WORKER = r'''
import os, sys, time, datetime
import torch.distributed as dist
sys.path.insert(0, os.environ["ROOT"])
from miles_b200.utils.health_monitor import RankHeartbeat, RankFailure
dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=20))
rank, world = dist.get_rank(), dist.get_world_size()
store = dist.distributed_c10d._get_default_store()
hb = RankHeartbeat(store, rank, world, timeout=2.0)
hb.start(0.2)
time.sleep(0.5)
hb.check()
import torch
dist.all_reduce(torch.ones(1))
if rank == 1:          # leaves between steps, nothing in flight
    hb.mark_exiting(); hb.stop(); sys.exit(0)
time.sleep(0.5)
try:
    hb.check()
    print("NO_FAILURE_DETECTED", flush=True)
except RankFailure as e:
    print("DETECTED", e, flush=True)
'''


@pytest.mark.timeout(120)
def test_rank_departure_detected(tmp_path):
    p = tmp_path / "w.py"
    p.write_text(WORKER)
    env = dict(os.environ, ROOT=ROOT)
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
                        "--master-addr", "127.0.0.1", "--master-port", str(free_port()), str(p)],
                       env=env, capture_output=True, text=True, timeout=110)
    assert "DETECTED rank 1 left the job" in r.stdout, r.stdout + r.stderr[-2000:]
