"""Router and engine server on CPU (tiny model engines), radix-tree cache."""
import asyncio
import time

import requests
import torch

from miles_b200.router.radix_tree import StringRadixTree
from miles_b200.router.router import WorkerPool, launch_router
from miles_b200.utils.http_utils import find_free_port


def test_worker_pool_policy():
    p = WorkerPool(failure_threshold=2)
    p.add("a"); p.add("b")
    w1 = p.acquire(); w2 = p.acquire()
    assert {w1, w2} == {"a", "b"}
    p.release("a")
    assert p.acquire() == "a"
    p.report("b", False); p.report("b", False)
    assert "b" in p.dead
    p.release("a"); p.release("a")
    assert p.acquire() == "a"
    p.report("b", True)
    assert "b" not in p.dead


def test_radix_tree():
    t = StringRadixTree()
    t.insert("hello world", [1, 2, 3], weight_version=1)
    t.insert("hello there", [1, 4], weight_version=2)
    n, toks, _, wv = t.longest_prefix("hello world, again")
    assert n == len("hello world") and toks == [1, 2, 3] and wv == 1
    assert t.longest_prefix("hello")[1] is None
    assert t.gc(2) == 1
    assert t.longest_prefix("hello world!")[1] is None
    assert t.longest_prefix("hello there!")[1] == [1, 4]


def test_server_and_router_end_to_end():
    from miles_b200.engine.engine import RolloutEngine
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer
    from miles_b200.rollout.server import serve

    urls = []
    for s in range(2):
        m = Transformer(preset("tiny"), device="cpu", dtype=torch.float32, seed=s)
        port = find_free_port(21000 + 37 * s)
        serve(RolloutEngine(m, max_batch=8, num_pages=64, use_cuda_graph=False), "127.0.0.1", port,
              background=True)
        urls.append(f"http://127.0.0.1:{port}")
    rport = find_free_port(22500)
    launch_router(None, "127.0.0.1", rport, workers=urls)
    base = f"http://127.0.0.1:{rport}"
    for _ in range(100):
        try:
            if requests.get(f"{base}/list_workers", timeout=1).ok and all(
                    requests.get(f"{u}/health", timeout=1).ok for u in urls):
                break
        except Exception:
            time.sleep(0.1)
    r = requests.post(f"{base}/generate", json={"input_ids": [1, 2, 3, 4],
                      "sampling_params": {"max_new_tokens": 5, "temperature": 0.0}}, timeout=60).json()
    assert len(r["output_ids"]) == 5
    assert r["meta_info"]["finish_reason"]["type"] == "length"
    assert len(r["meta_info"]["output_token_logprobs"]) == 5
    info = requests.get(f"{base}/list_workers").json()
    assert sorted(info["urls"]) == sorted(urls)
