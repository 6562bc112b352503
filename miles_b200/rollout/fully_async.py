"""Fully-asynchronous rollout worker: a background thread keeps prompt groups in flight on this
process's engine across training steps, so generation never waits for the trainer.

  * The worker pulls groups from the data source (its partial-rollout buffer first), runs
    generate + reward on them and queues finished groups tagged with the weight version they
    started under.
  * `pause()` (before a weight refit) aborts the in-flight requests and waits until the worker
    is idle. With --partial-rollout the unfinished samples keep their generated tokens and go
    back to the buffer; they resume under the new weights (tokens from the old policy are
    loss-masked with --mask-offpolicy-in-partial-rollout).
  * `get_batch(n)` returns n finished groups; groups whose starting weight version lags the
    current one by more than --max-weight-staleness are dropped (counted in the metrics).

Reference: examples/fully_async/fully_async_rollout.py:77-338 (background worker, recycling of
aborted groups, staleness filter through the engine's weight version).
"""
from __future__ import annotations

import asyncio
import copy
import queue
import threading
import time

from miles_b200.rollout.default import GenerateState, generate_and_rm_group
from miles_b200.utils.types import Sample


class FullyAsyncRollout:
    def __init__(self, args, data_source, state: GenerateState, weight_version_fn,
                 groups_in_flight: int | None = None):
        self.args = args
        self.data_source = data_source
        self.state = state
        self.weight_version = weight_version_fn
        self.in_flight = groups_in_flight or args.rollout_batch_size
        self.done: queue.Queue = queue.Queue()
        self._run = threading.Event()
        self._run.set()
        self._idle = threading.Event()
        self._stop = False
        self.dropped_stale = 0
        self.recycled = 0
        self._thread = threading.Thread(target=self._worker, name="fully-async-rollout", daemon=True)
        self._thread.start()

    # ------------------------------------------------------------------ worker thread
    def _worker(self):
        loop = asyncio.new_event_loop()
        asyncio.set_event_loop(loop)
        try:
            while not self._stop:
                if not self._run.is_set():
                    self._idle.set()
                    self._run.wait(0.05)
                    continue
                self._idle.clear()
                groups = self.data_source.get_samples(self.in_flight)
                if not groups:
                    self._idle.set()
                    time.sleep(0.01)
                    continue
                ver = self.weight_version()
                for g in groups:
                    for s in g:
                        s.metadata.setdefault("start_weight_version", ver)
                self.state.aborted = False
                sp = copy.deepcopy(self.state.sampling_params)
                results = loop.run_until_complete(asyncio.gather(
                    *[generate_and_rm_group(self.args, g, sp) for g in groups]))
                for g in results:
                    if any(s.status in (Sample.Status.ABORTED, Sample.Status.PENDING) for s in g):
                        self._recycle(g)
                    else:
                        self.done.put(g)
        finally:
            self._idle.set()
            loop.close()

    def _recycle(self, g: list[Sample]):
        if not self.args.partial_rollout:
            for s in g:  # start over from the prompt
                s.tokens = s.tokens[: len(s.tokens) - s.response_length]
                s.response_length = 0
                s.loss_mask = None
                s.rollout_log_probs = None
                s.status = Sample.Status.PENDING
                s.reward = None
        else:
            for s in g:
                if self.args.mask_offpolicy_in_partial_rollout and s.response_length:
                    s.loss_mask = [0] * s.response_length
                if s.status == Sample.Status.ABORTED:
                    s.status = Sample.Status.PENDING
                s.reward = None
        self.recycled += 1
        self.data_source.add_samples([g])

    # ------------------------------------------------------------------ control (main thread)
    def pause(self, timeout: float = 600.0):
        """Abort in-flight generation and wait until the worker is idle (before a refit)."""
        self._run.clear()
        self.state.aborted = True
        client = self.state.client
        if client is not None and hasattr(client, "abort"):
            client.abort()
        if not self._idle.wait(timeout):
            raise TimeoutError("fully-async rollout worker did not stop")

    def resume(self):
        self.state.aborted = False
        client = self.state.client
        if client is not None and hasattr(client, "resume"):
            client.resume()
        self._run.set()

    def get_batch(self, n: int, timeout: float = 3600.0) -> list[list[Sample]]:
        out = []
        cur = self.weight_version()
        limit = self.args.max_weight_staleness
        deadline = time.time() + timeout
        while len(out) < n:
            g = self.done.get(timeout=max(0.0, deadline - time.time()))
            start = min(s.metadata.get("start_weight_version", cur) for s in g)
            if limit is not None and cur - start > limit:
                self.dropped_stale += 1
                continue
            out.append(g)
        out.sort(key=lambda g: g[0].index if g[0].index is not None else 0)
        return out

    def metrics(self) -> dict:
        return {"rollout/fully_async/dropped_stale": self.dropped_stale,
                "rollout/fully_async/recycled_groups": self.recycled,
                "rollout/fully_async/queued_groups": self.done.qsize()}

    def shutdown(self):
        self._stop = True
        self.pause()
