"""Session server: an OpenAI-chat-compatible endpoint per agent session that records the exact
token trajectory (token-in, token-out) for training.

Agents keep calling `POST /sessions/{id}/v1/chat/completions` with the growing message list.
The server never re-tokenizes what the model generated: it keeps the token ids of the last
checkpoint (prompt + completion as generated) and appends only the tokens of the new messages
(tool results, user turns) plus the generation prompt, obtained as the difference between
chat-template renderings. The engine is called with these `input_ids`. Each completion is
recorded with its log-probs; at the end `to_sample()` yields one linear trajectory whose loss
mask covers exactly the model-generated tokens.

Retries are handled the way agents produce them: a request whose messages stop at an earlier
assistant turn rolls the session back to that turn's checkpoint (at most one step).
A request that rewrites earlier messages is rejected (the trajectory must stay linear).

Endpoints:  POST /sessions -> {session_id};  GET /sessions/{id} -> trajectory;
            DELETE /sessions/{id};  POST /sessions/{id}/v1/chat/completions;  GET /health

Reference: miles/rollout/session/ (sessions.py routes :23-250, linear_trajectory.py
LinearTrajectory / SessionRegistry :38-294, session_server.py :24-105) and the TITO tokenizer
of utils/chat_template_utils.
"""
from __future__ import annotations

try:  # module level: FastAPI resolves string annotations against module globals
    from fastapi import Request
except ImportError:  # pragma: no cover
    Request = None

import asyncio
import itertools
import time
from dataclasses import dataclass, field

from miles_b200.utils.types import Sample


class SessionError(ValueError):
    pass


def _render(tok, messages, add_generation_prompt: bool, tools=None) -> list[int]:
    kw = {"tools": tools} if tools else {}
    out = tok.apply_chat_template(messages, tokenize=True, add_generation_prompt=add_generation_prompt, **kw)
    return list(out["input_ids"] if isinstance(out, dict) else out)


@dataclass
class Checkpoint:
    token_ids: list[int]
    loss_mask: list[int]
    logprobs: list[float]
    num_messages: int  # messages covered (including the assistant reply)


@dataclass
class Session:
    messages: list[dict] = field(default_factory=list)
    checkpoints: list[Checkpoint] = field(default_factory=list)
    records: list[dict] = field(default_factory=list)
    lock: asyncio.Lock = field(default_factory=asyncio.Lock)
    closed: bool = False

    @property
    def head(self) -> Checkpoint | None:
        return self.checkpoints[-1] if self.checkpoints else None

    def prepare(self, tok, request_messages: list[dict], tools=None,
                allowed_roles=None) -> tuple[list[int], list[int], list[float]]:
        """(input_ids, loss mask so far, log-probs so far) for the next completion.
        allowed_roles: roles that may be appended after the last assistant turn
        (--tito-allowed-append-roles; None = any)."""
        # roll back one assistant step if the agent retries from the previous checkpoint
        if len(self.checkpoints) >= 2 and len(request_messages) < len(self.messages) and \
                len(request_messages) >= self.checkpoints[-2].num_messages:
            self.checkpoints.pop()
            self.messages = self.messages[:self.checkpoints[-1].num_messages]
        head = self.head
        if head is None:
            ids = _render(tok, request_messages, True, tools)
            return ids, [0] * len(ids), [0.0] * len(ids)
        n = head.num_messages
        if request_messages[:n] != self.messages[:n]:
            raise SessionError("request rewrites earlier messages; sessions are linear")
        if allowed_roles is not None:
            bad = [m.get("role") for m in request_messages[n:] if m.get("role") not in allowed_roles]
            if bad:
                raise SessionError(f"appending role(s) {bad} is not allowed (allowed: {sorted(allowed_roles)})")
        from miles_b200.rollout.tito import IncrementalTokenizer

        tito = IncrementalTokenizer(tok, tools)
        old = _render(tok, self.messages[:n], False, tools)
        new = _render(tok, request_messages, True, tools)
        try:
            # the generated turn ends where the engine stopped: add what the template renders
            # after an assistant turn that the generation did not emit (e.g. the newline after
            # the end-of-turn token)
            join = tito.junction(head.token_ids)
            if new[:len(old)] == old:
                delta = join + new[len(old):]
            else:
                # not prefix-stable (e.g. a thinking template dropping earlier reasoning):
                # tokenize the appended messages incrementally
                delta = join + tito.suffix(request_messages[n:])
        except ValueError as e:
            raise SessionError(str(e)) from e
        return (head.token_ids + delta, head.loss_mask + [0] * len(delta),
                head.logprobs + [0.0] * len(delta))

    def commit(self, request_messages, reply: dict, input_ids, mask, lps, out_ids, out_lps):
        self.messages = list(request_messages) + [reply]
        self.checkpoints.append(Checkpoint(list(input_ids) + list(out_ids),
                                           list(mask) + [1] * len(out_ids),
                                           list(lps) + list(out_lps), len(self.messages)))

    def to_sample(self, index: int | None = None) -> Sample:
        h = self.head
        if h is None:
            raise SessionError("empty session")
        start = h.loss_mask.index(1) if 1 in h.loss_mask else len(h.token_ids)
        s = Sample(prompt=self.messages, index=index, tokens=list(h.token_ids))
        s.response_length = len(h.token_ids) - start
        s.loss_mask = h.loss_mask[start:]
        s.rollout_log_probs = h.logprobs[start:]
        s.status = Sample.Status.COMPLETED
        return s


class SessionRegistry:
    def __init__(self, tokenizer, client, default_max_tokens: int = 1024, allowed_append_roles=None,
                 model_name: str | None = None):
        self.allowed_roles = set(allowed_append_roles) if allowed_append_roles else None
        self.model_name = model_name
        self.tok = tokenizer
        self.client = client  # .generate(input_ids, sampling_params, return_logprob) -> dict
        self.sessions: dict[str, Session] = {}
        self._ids = itertools.count()
        self.default_max_tokens = default_max_tokens

    def create(self) -> str:
        sid = f"s{next(self._ids)}-{int(time.time() * 1000) % 100000}"
        self.sessions[sid] = Session()
        return sid

    def get(self, sid: str) -> Session:
        s = self.sessions.get(sid)
        if s is None or s.closed:
            raise KeyError(sid)
        return s

    def remove(self, sid: str):
        s = self.sessions.pop(sid, None)
        if s is not None:
            s.closed = True

    async def chat(self, sid: str, body: dict) -> dict:
        sess = self.get(sid)
        msgs = body.get("messages", [])
        tools = body.get("tools")
        async with sess.lock:
            ids, mask, lps = sess.prepare(self.tok, msgs, tools, self.allowed_roles)
            nmsg = len(sess.checkpoints)
        sp = {"temperature": body.get("temperature", 1.0),
              "max_new_tokens": body.get("max_tokens") or body.get("max_completion_tokens")
              or self.default_max_tokens}
        if body.get("seed") is not None:
            sp["sampling_seed"] = int(body["seed"])
        out = await self.client.generate(ids, sp, return_logprob=True)
        out_ids = list(out["output_ids"])
        out_lps = [x[0] for x in out["meta_info"]["output_token_logprobs"]]
        text = out.get("text") or (self.tok.decode(out_ids) if hasattr(self.tok, "decode") else "")
        reply = {"role": "assistant", "content": text}
        async with sess.lock:
            if len(sess.checkpoints) == nmsg:  # no concurrent change while generating
                sess.commit(msgs, reply, ids, mask, lps, out_ids, out_lps)
        finish = out["meta_info"].get("finish_reason", {}).get("type", "stop")
        resp = {
            "id": f"chatcmpl-{sid}-{nmsg}", "object": "chat.completion", "created": int(time.time()),
            "model": body.get("model", self.model_name or "miles-b200"),
            "choices": [{"index": 0, "message": reply,
                         "finish_reason": "length" if finish == "length" else "stop",
                         "prompt_token_ids": ids,
                         "meta_info": {"output_token_logprobs": [[lp, t] for lp, t in zip(out_lps, out_ids)],
                                       "completion_tokens": len(out_ids)}}],
            "usage": {"prompt_tokens": len(ids), "completion_tokens": len(out_ids),
                      "total_tokens": len(ids) + len(out_ids)},
        }
        sess.records.append({"request": body, "response": resp, "time": time.time()})
        return resp


def build_session_app(registry: SessionRegistry):
    from fastapi import FastAPI, HTTPException, Request
    from fastapi.responses import JSONResponse

    app = FastAPI()

    @app.get("/health")
    async def health():
        return {"status": "ok", "sessions": len(registry.sessions)}

    @app.post("/sessions")
    async def create():
        return {"session_id": registry.create()}

    @app.get("/sessions/{sid}")
    async def get(sid: str):
        try:
            s = registry.get(sid)
        except KeyError:
            raise HTTPException(404, f"session not found: {sid}")
        h = s.head
        return {"session_id": sid, "messages": s.messages, "num_turns": len(s.checkpoints),
                "token_ids": h.token_ids if h else [], "loss_mask": h.loss_mask if h else [],
                "logprobs": h.logprobs if h else []}

    @app.delete("/sessions/{sid}")
    async def delete(sid: str):
        registry.remove(sid)
        return {"deleted": sid}

    @app.post("/sessions/{sid}/v1/chat/completions")
    async def chat(sid: str, req: Request):
        try:
            return JSONResponse(await registry.chat(sid, await req.json()))
        except KeyError:
            raise HTTPException(404, f"session not found: {sid}")
        except SessionError as e:
            raise HTTPException(400, str(e))

    return app


def launch_session_server(args, tokenizer, client, background: bool = True):
    """--use-session-server: the OpenAI-style session endpoint on --session-server-ip /
    --session-server-port (a free port when unset), backed by this rank's engine client.
    Returns (registry, url)."""
    import socket
    import threading

    import uvicorn

    host = getattr(args, "session_server_ip", None) or "127.0.0.1"
    port = getattr(args, "session_server_port", None)
    if not port:
        with socket.socket() as sk:
            sk.bind((host, 0))
            port = sk.getsockname()[1]
    reg = SessionRegistry(tokenizer, client,
                          default_max_tokens=getattr(args, "rollout_max_response_len", None) or 1024,
                          allowed_append_roles=getattr(args, "tito_allowed_append_roles", None),
                          model_name=getattr(args, "tito_model", None))
    server = uvicorn.Server(uvicorn.Config(build_session_app(reg), host=host, port=int(port),
                                           log_level="warning"))
    if background:
        threading.Thread(target=server.run, daemon=True).start()
    else:
        server.run()
    url = f"http://{host}:{port}"
    args.session_server_url = url
    return reg, url
