"""Engine clients used by rollout / generate functions.

Rollout code talks to an engine through one async call,

    await client.generate(input_ids, sampling_params, return_logprob=True,
                          return_routed_experts=False) -> dict

whose result mirrors an SGLang /generate response ({"output_ids", "text", "meta_info": {
"finish_reason": {"type": ...}, "output_token_logprobs": [(logp, token_id, None), ...],
"routed_experts", "weight_version"}}), so user generate functions written for the reference
keep working.

  * LocalEngineClient batches concurrent requests from many asyncio tasks into calls of the
    in-process RolloutEngine (running in a worker thread so `abort()` stays responsive).
  * HttpEngineClient posts to an engine server / router URL.

Reference: sglang_rollout.py generate (:131-231, HTTP POST /generate, abort :333-374).
"""
from __future__ import annotations

import asyncio
import threading
import time

import numpy as np

from miles_b200.engine.engine import GenRequest, RolloutEngine


def _result_dict(res, tokenizer=None) -> dict:
    text = tokenizer.decode(res.tokens) if tokenizer is not None else ""
    meta = {
        "finish_reason": {"type": res.finish_reason},
        "output_token_logprobs": [(lp, t, None) for lp, t in zip(res.logprobs, res.tokens)],
        "completion_tokens": len(res.tokens),
        "weight_version": str(res.weight_version),
    }
    if res.routed_experts is not None:
        meta["routed_experts"] = res.routed_experts
    return {"output_ids": res.tokens, "text": text, "meta_info": meta}


def _truncate_at_stop(res, stops: list[str], tokenizer):
    """Stop strings: cut the response after the first token whose decoded prefix contains a stop
    string (tokens, log-probs and routing cut alike; finish reason "stop"). The engine stops on
    token ids on the device; strings are matched here on the text."""
    text = ""
    for i in range(len(res.tokens)):
        text = tokenizer.decode(res.tokens[: i + 1])
        if any(s and s in text for s in stops):
            import dataclasses

            ex = res.routed_experts
            if ex is not None:
                ex = ex[: len(ex) - (len(res.tokens) - (i + 1))]
            return dataclasses.replace(res, tokens=res.tokens[: i + 1], logprobs=res.logprobs[: i + 1],
                                       finish_reason="stop", routed_experts=ex)
    return res


class LocalEngineClient:
    # prefill / decode disaggregation: a miles_b200.rollout.pd.RemotePrefill that prefills the
    # requests on a paired prefill rank (this engine then only decodes); None: prefill here
    remote_prefill = None

    def __init__(self, engine: RolloutEngine, tokenizer=None, max_wait_s: float = 0.002,
                 max_batch: int | None = None):
        self.engine = engine
        self.tokenizer = tokenizer
        self.max_wait_s = max_wait_s
        self.max_batch = max_batch or engine.max_batch * 8
        self._pending: list[tuple[GenRequest, asyncio.Future]] = []
        self._lock = threading.Lock()
        self._runner: asyncio.Task | None = None
        self._serve = None  # executor future of the running engine.generate call
        self._outstanding = 0
        self._rid = 0
        self.num_requests = 0

    async def generate(self, input_ids: list[int], sampling_params: dict,
                       return_logprob: bool = True, return_routed_experts: bool = False) -> dict:
        loop = asyncio.get_running_loop()
        fut = loop.create_future()
        self._rid += 1
        stop = tuple(sampling_params.get("stop_token_ids") or ())
        temp = float(sampling_params.get("temperature", 1.0))
        req = GenRequest(prompt=list(input_ids),
                         max_new_tokens=int(sampling_params.get("max_new_tokens", 128)),
                         temperature=temp, seed=int(sampling_params.get("sampling_seed", self._rid)),
                         stop_token_ids=stop, return_routed_experts=return_routed_experts,
                         rid=self._rid, top_k=int(sampling_params.get("top_k", 0) or 0),
                         top_p=float(sampling_params.get("top_p", 1.0) or 1.0))
        self._pending.append((req, fut))
        self.num_requests += 1
        if self._runner is None or self._runner.done():
            self._runner = asyncio.ensure_future(self._run())
        self._outstanding += 1
        try:
            res = await fut
        finally:
            self._outstanding -= 1
            if (self._outstanding == 0 and not self._pending and self._runner is not None
                    and not self._runner.done() and (self._serve is None or self._serve.done())):
                self._runner.cancel()  # nothing left to feed: stop the feeder task
        if isinstance(res, Exception):
            raise res
        stops = sampling_params.get("stop")
        if stops and self.tokenizer is not None:
            res = _truncate_at_stop(res, [stops] if isinstance(stops, str) else list(stops),
                                    self.tokenizer)
        return _result_dict(res, self.tokenizer)

    async def _run(self):
        """Feed queued requests to the engine: into the running generate() call when there is
        one (they join its batch at its next host visit), else into a new call on a worker
        thread. Results come back per request as each finishes."""
        loop = asyncio.get_running_loop()
        while self._pending or (self._serve is not None and not self._serve.done()):
            await asyncio.sleep(self.max_wait_s)
            batch, self._pending = self._pending, []
            if not batch:
                continue
            items = [(req, self._deliver(loop, fut)) for req, fut in batch]
            if self.remote_prefill is not None:
                # the paired prefill rank computes the prompts; this engine admits the hand-offs
                hs = await loop.run_in_executor(None, self.remote_prefill.prefill, [r for r, _ in items])
                items = [(h, cb) for h, (_, cb) in zip(hs, items)]
            if not self.engine.submit(items):
                self._serve = loop.run_in_executor(None, self._serve_items, items)

    @staticmethod
    def _deliver(loop, fut):
        def cb(res):
            loop.call_soon_threadsafe(lambda: fut.done() or fut.set_result(res))
        return cb

    def _serve_items(self, items):
        futs = {req.rid: cb for req, cb in items}
        try:
            self.engine.generate([r for r, _ in items], callbacks=futs)
        except Exception as e:  # propagate to every waiter of this call
            for req, cb in items:
                cb(e)

    def abort(self):
        """Abort in-flight generations (they finish with finish_reason 'abort')."""
        self.engine.abort()
        for req, f in self._pending:
            if not f.done():
                from miles_b200.engine.engine import GenResult
                f.set_result(GenResult(req.rid, [], [], "abort"))
        self._pending = []

    async def health(self) -> bool:
        return self.engine.health_check()


class HttpEngineClient:
    """Client of an engine server (miles_b200.rollout.server) or of the router."""

    def __init__(self, url: str, timeout: float | None = None):
        self.url = url.rstrip("/")
        self.timeout = timeout

    async def generate(self, input_ids, sampling_params, return_logprob=True,
                       return_routed_experts=False) -> dict:
        from miles_b200.utils.http_utils import post

        out = await post(f"{self.url}/generate", {
            "input_ids": list(input_ids), "sampling_params": sampling_params,
            "return_logprob": return_logprob, "return_routed_experts": return_routed_experts})
        re_ = out.get("meta_info", {}).get("routed_experts")
        if isinstance(re_, list):
            out["meta_info"]["routed_experts"] = np.asarray(re_, dtype=np.int32)
        return out

    def abort(self):
        import requests

        try:
            requests.post(f"{self.url}/abort_request", json={"abort_all": True}, timeout=10)
        except Exception:
            pass

    async def health(self) -> bool:
        from miles_b200.utils.http_utils import get

        try:
            await get(f"{self.url}/health_generate")
            return True
        except Exception:
            return False
