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


def test_train_recovers_engine_after_injected_crash(tmp_path, monkeypatch):
    """--use-fault-tolerance with --ci-test: a host-side crash is injected into the rollout
    engine at rollout 1; the supervisor rebuilds it before that rollout and training goes on."""
    monkeypatch.setenv("MILES_B200_FORCE_CPU", "1")
    import json

    import numpy as np

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    rng = np.random.default_rng(0)
    with open(tmp_path / "d.jsonl", "w") as f:
        for _ in range(8):
            f.write(json.dumps({"input": rng.integers(0, 4096, 32).tolist(), "label": "1"}) + "\n")
    sys.path.insert(0, root)
    import train as T
    from miles_b200.rollout.default import GenerateState
    from miles_b200.utils.arguments import parse_args

    GenerateState._inst = None
    args = parse_args(["--model-name", "tiny", "--prompt-data", str(tmp_path / "d.jsonl"),
                       "--label-key", "label", "--rollout-batch-size", "2", "--n-samples-per-prompt", "2",
                       "--rollout-max-response-len", "8", "--rm-type", "random", "--num-rollout", "3",
                       "--actor-num-gpus-per-node", "1", "--ci-test", "--use-fault-tolerance",
                       "--rollout-health-check-interval", "0.2", "--rollout-health-check-timeout", "5"])
    hist = T.train(args)
    assert len(hist) == 3
    assert [h["fault_tolerance/recoveries"] for h in hist] == [0, 1, 1]
