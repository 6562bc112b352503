"""String radix tree caching (text -> token ids, log-probs, weight version) for multi-turn
rollouts, plus the router middleware that uses it.

When a multi-turn conversation sends its growing transcript as text, the longest cached
prefix's tokens (and the log-probs the engine reported for generated spans) are reused so the
request carries exact token ids: re-tokenising a decoded response can change tokens, which
would silently break the train/rollout log-prob correspondence. Entries whose weight version
is older than `min_weight_version` are garbage-collected.

Reference: miles/router/middleware_hub/radix_tree.py:96-681, radix_tree_middleware.py:59-190.
"""
from __future__ import annotations

import json
import threading
from dataclasses import dataclass, field


@dataclass
class _Node:
    key: str = ""
    children: dict = field(default_factory=dict)  # first char -> node
    tokens: list | None = None                    # token ids of the full prefix ending here
    logprobs: list | None = None
    weight_version: int = 0
    hits: int = 0


class StringRadixTree:
    def __init__(self):
        self.root = _Node()
        self.lock = threading.Lock()
        self.size = 0

    def insert(self, text: str, tokens: list[int], logprobs: list[float] | None = None,
               weight_version: int = 0) -> None:
        with self.lock:
            node, rest = self.root, text
            while rest:
                ch = node.children.get(rest[0])
                if ch is None:
                    new = _Node(rest)
                    node.children[rest[0]] = new
                    node, rest = new, ""
                    self.size += 1
                    break
                k = ch.key
                i = 0
                while i < len(k) and i < len(rest) and k[i] == rest[i]:
                    i += 1
                if i < len(k):  # split the edge
                    mid = _Node(k[:i])
                    ch.key = k[i:]
                    mid.children[ch.key[0]] = ch
                    node.children[rest[0]] = mid
                    self.size += 1
                    ch = mid
                node, rest = ch, rest[i:]
            node.tokens = list(tokens)
            node.logprobs = list(logprobs) if logprobs is not None else None
            node.weight_version = weight_version

    def longest_prefix(self, text: str):
        """(matched_text_len, tokens, logprobs, weight_version) of the longest cached prefix."""
        with self.lock:
            node, rest, matched = self.root, text, 0
            best = (0, None, None, 0)
            while rest:
                ch = node.children.get(rest[0])
                if ch is None or not rest.startswith(ch.key):
                    break
                matched += len(ch.key)
                rest = rest[len(ch.key):]
                node = ch
                if node.tokens is not None:
                    node.hits += 1
                    best = (matched, node.tokens, node.logprobs, node.weight_version)
            return best

    def gc(self, min_weight_version: int) -> int:
        """Drop cached entries older than `min_weight_version`; returns the number removed."""
        removed = 0

        def walk(n: _Node):
            nonlocal removed
            for c in list(n.children.values()):
                walk(c)
                if c.tokens is not None and c.weight_version < min_weight_version:
                    c.tokens, c.logprobs = None, None
                    removed += 1
                if c.tokens is None and not c.children:
                    del n.children[c.key[0]]
                    self.size -= 1

        with self.lock:
            walk(self.root)
        return removed


class RadixTreeMiddleware:
    """Router middleware: for /generate requests that carry `text`, prepend the cached token
    prefix (as input_ids) and insert the completed transcript after the response."""

    def __init__(self, args=None, tokenizer=None):
        self.tree = StringRadixTree()
        self.tokenizer = tokenizer

    async def __call__(self, body: bytes, path: str, forward):
        if path != "generate":
            return await forward(body)
        try:
            req = json.loads(body)
        except Exception:
            return await forward(body)
        text = req.get("text")
        if text is None or self.tokenizer is None:
            return await forward(body)
        n, toks, _, _ = self.tree.longest_prefix(text)
        ids = list(toks or []) + self.tokenizer(text[n:], add_special_tokens=False)["input_ids"]
        req.pop("text")
        req["input_ids"] = ids
        status, content, ct = await forward(json.dumps(req).encode())
        if status == 200:
            out = json.loads(content)
            full = text + out.get("text", "")
            wv = int(out.get("meta_info", {}).get("weight_version", 0) or 0)
            self.tree.insert(full, ids + out.get("output_ids", []), None, wv)
        return status, content, ct
