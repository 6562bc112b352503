"""Async HTTP helpers with retries (aiohttp) and free-port discovery.

Reference: miles/utils/http_utils.py (post / get with retries :188-315, port helpers).
"""
from __future__ import annotations

import asyncio
import json
import socket

import numpy as np

_SESSION = None


def _default(o):
    if isinstance(o, np.ndarray):
        return o.tolist()
    if isinstance(o, (np.integer,)):
        return int(o)
    if isinstance(o, (np.floating,)):
        return float(o)
    raise TypeError(type(o))


async def _session():
    """One client session per event loop (a session is bound to the loop that created it; each
    asyncio.run() starts a new loop)."""
    import aiohttp

    global _SESSION
    loop = asyncio.get_running_loop()
    if _SESSION is None or _SESSION[1].closed or _SESSION[0] is not loop:
        _SESSION = (loop, aiohttp.ClientSession(timeout=aiohttp.ClientTimeout(total=None),
                                                json_serialize=lambda x: json.dumps(x, default=_default)))
    return _SESSION[1]


async def post(url: str, payload: dict, max_retries: int = 10, retry_wait: float = 1.0):
    last = None
    for attempt in range(max_retries):
        try:
            s = await _session()
            async with s.post(url, json=payload) as resp:
                resp.raise_for_status()
                return await resp.json()
        except Exception as e:  # connection reset / 5xx: retry with backoff
            last = e
            await asyncio.sleep(retry_wait * (1 + attempt))
    raise RuntimeError(f"POST {url} failed after {max_retries} attempts: {last!r}")


async def get(url: str, max_retries: int = 3, retry_wait: float = 0.5):
    last = None
    for attempt in range(max_retries):
        try:
            s = await _session()
            async with s.get(url) as resp:
                resp.raise_for_status()
                ct = resp.headers.get("content-type", "")
                return await (resp.json() if "json" in ct else resp.text())
        except Exception as e:
            last = e
            await asyncio.sleep(retry_wait)
    raise RuntimeError(f"GET {url} failed: {last!r}")


def find_free_port(start: int = 10000, host: str = "127.0.0.1") -> int:
    for port in range(start, start + 10000):
        with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
            try:
                s.bind((host, port))
                return port
            except OSError:
                continue
    raise RuntimeError("no free port")


def is_port_available(port: int, host: str = "127.0.0.1") -> bool:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        try:
            s.bind((host, port))
            return True
        except OSError:
            return False
