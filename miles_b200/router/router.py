"""Miles-router equivalent: an HTTP load balancer in front of engine servers.

  * least-outstanding-requests worker selection (ties -> lowest index)
  * background health checks; a worker failing `failure_threshold` consecutive checks is
    quarantined (excluded) until it passes again
  * /add_worker?url=..., /list_workers, /remove_worker?url=...
  * pass-through of every other path (POST/GET) to the chosen worker, preserving
    meta_info.routed_experts (needed by Rollout Routing Replay)
  * middleware plugins (--miles-router-middleware-paths): objects with async
    `__call__(request_body, path, forward)` wrapping the forward call

Reference: miles/router/router.py:32-237 (MilesRouter), docs/en/advanced/miles-router.md.
"""
from __future__ import annotations

try:  # module level: FastAPI resolves string annotations against module globals
    from fastapi import Request
except ImportError:  # pragma: no cover
    Request = None

import asyncio
import threading

from miles_b200.utils.misc import load_function


class WorkerPool:
    def __init__(self, failure_threshold: int = 3):
        self.workers: list[str] = []
        self.outstanding: dict[str, int] = {}
        self.failures: dict[str, int] = {}
        self.dead: set[str] = set()
        self.failure_threshold = failure_threshold
        self.lock = threading.Lock()

    def add(self, url: str):
        with self.lock:
            if url not in self.workers:
                self.workers.append(url)
                self.outstanding[url] = 0
                self.failures[url] = 0

    def remove(self, url: str):
        with self.lock:
            if url in self.workers:
                self.workers.remove(url)
                self.outstanding.pop(url, None)
                self.failures.pop(url, None)
                self.dead.discard(url)

    def acquire(self) -> str:
        with self.lock:
            live = [w for w in self.workers if w not in self.dead]
            if not live:
                raise RuntimeError("no healthy workers")
            w = min(live, key=lambda u: (self.outstanding[u], self.workers.index(u)))
            self.outstanding[w] += 1
            return w

    def release(self, url: str):
        with self.lock:
            if url in self.outstanding:
                self.outstanding[url] -= 1

    def report(self, url: str, ok: bool):
        with self.lock:
            if url not in self.failures:
                return
            if ok:
                self.failures[url] = 0
                self.dead.discard(url)
            else:
                self.failures[url] += 1
                if self.failures[url] >= self.failure_threshold:
                    self.dead.add(url)


def build_router_app(args=None, workers: list[str] | None = None, health_interval: float = 10.0):
    import aiohttp
    from fastapi import FastAPI, Request
    from fastapi.responses import JSONResponse, Response

    thr = getattr(args, "miles_router_health_check_failure_threshold", 3) if args else 3
    pool = WorkerPool(thr)
    for w in workers or []:
        pool.add(w)
    middlewares = [load_function(p)(args) for p in (getattr(args, "miles_router_middleware_paths", None) or [])]
    app = FastAPI()
    app.state.pool = pool
    sess: dict = {}

    async def session():
        if "s" not in sess:
            sess["s"] = aiohttp.ClientSession(timeout=aiohttp.ClientTimeout(total=getattr(args, "miles_router_timeout", None) if args else None))
        return sess["s"]

    async def health_loop():
        while True:
            await asyncio.sleep(health_interval)
            s = await session()
            for w in list(pool.workers):
                try:
                    async with s.get(f"{w}/health", timeout=aiohttp.ClientTimeout(total=5)) as r:
                        pool.report(w, r.status == 200)
                except Exception:
                    pool.report(w, False)

    @app.on_event("startup")
    async def _start():
        app.state.health_task = asyncio.create_task(health_loop())

    @app.post("/add_worker")
    async def add_worker(url: str):
        pool.add(url)
        return {"workers": pool.workers}

    @app.post("/remove_worker")
    async def remove_worker(url: str):
        pool.remove(url)
        return {"workers": pool.workers}

    @app.get("/list_workers")
    async def list_workers():
        return {"urls": pool.workers, "dead": sorted(pool.dead)}

    async def forward(path: str, method: str, body: bytes, headers: dict):
        w = pool.acquire()
        try:
            s = await session()
            async with s.request(method, f"{w}/{path}", data=body, headers=headers) as r:
                content = await r.read()
                return r.status, content, r.headers.get("content-type", "application/json")
        except Exception:
            pool.report(w, False)
            raise
        finally:
            pool.release(w)

    @app.api_route("/{path:path}", methods=["GET", "POST"])
    async def proxy(path: str, request: Request):
        body = await request.body()
        hdr = {"content-type": request.headers.get("content-type", "application/json")}

        async def call(b=body):
            return await forward(path, request.method, b, hdr)

        fn = call
        for mw in reversed(middlewares):
            prev = fn

            async def fn(b=body, _mw=mw, _prev=prev):  # noqa: E306
                return await _mw(b, path, _prev)

        status, content, ct = await fn()
        return Response(content=content, status_code=status, media_type=ct)

    return app


def launch_router(args, host: str, port: int, workers: list[str] | None = None, background=True):
    import uvicorn

    app = build_router_app(args, workers)
    server = uvicorn.Server(uvicorn.Config(app, host=host, port=port, log_level="warning"))
    if background:
        t = threading.Thread(target=server.run, daemon=True)
        t.start()
        return app, server, t
    server.run()
    return app, server, None
