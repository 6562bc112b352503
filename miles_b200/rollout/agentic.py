"""Agentic generate function: a user agent drives the policy through the session server's
OpenAI-style endpoint, and the session's token-in / token-out trajectory becomes the sample.

    --use-session-server \
    --custom-generate-function-path miles_b200.rollout.agentic.generate \
    --custom-agent-function-path my_pkg.agent.run [--max-seq-len N] [--generate-multi-samples]

Agent contract (async):

    async def run(base_url: str, prompt, request_kwargs: dict, metadata: dict, **kw) -> dict | None

`base_url` is an OpenAI-compatible base (POST {base_url}/chat/completions) bound to a fresh
session; the agent calls it as often as it likes (tool calls, environment steps, retries that
roll back one turn). `request_kwargs` are the rollout sampling parameters under OpenAI names
(max_tokens, temperature, top_p, top_k, seed). A returned dict is merged into the sample's
metadata (custom reward functions read it).

After the agent returns, the session's trajectory is read: the tokens of every turn with a loss
mask that is 1 on model-generated tokens and 0 on prompt / tool / environment tokens, and the
engine's log-probs of the generated tokens. With --generate-multi-samples every assistant turn
becomes its own sample (its context as the prompt); otherwise the whole trajectory is one sample.
--max-seq-len truncates a trajectory to that many tokens. A session with no model call returns
the input sample marked ABORTED.

Reference role: miles/rollout/generate_hub/agentic_tool_call.py (OpenAI endpoint tracer,
records -> samples, multi-sample mode, truncation).
"""
from __future__ import annotations

import copy
import logging

from miles_b200.utils.http_utils import get, post
from miles_b200.utils.misc import load_function
from miles_b200.utils.types import Sample

log = logging.getLogger(__name__)

_KEYMAP = {"max_new_tokens": "max_tokens", "min_new_tokens": "min_tokens", "sampling_seed": "seed"}


def request_kwargs(sampling_params: dict) -> dict:
    """Rollout sampling parameters -> OpenAI chat-completion request fields."""
    out = {}
    for k, v in (sampling_params or {}).items():
        out[_KEYMAP.get(k, k)] = v
    return out


def _session_url(args) -> str:
    url = getattr(args, "session_server_url", None)
    if url:
        return url
    ip, port = getattr(args, "session_server_ip", None), getattr(args, "session_server_port", None)
    if not (ip and port):
        raise ValueError("the agentic generate function needs the session server (--use-session-server)")
    return f"http://{ip}:{port}"


def _turn_samples(sample: Sample, traj: dict) -> list[Sample]:
    """One sample per assistant turn: the prefix before the turn is its prompt."""
    toks, mask, lps = traj["token_ids"], traj["loss_mask"], traj["logprobs"]
    out = []
    i = 0
    while i < len(mask):
        if mask[i] != 1:
            i += 1
            continue
        j = i
        while j < len(mask) and mask[j] == 1:
            j += 1
        s = copy.deepcopy(sample)
        s.tokens = list(toks[:j])
        s.response_length = j - i
        s.loss_mask = [1] * (j - i)
        s.rollout_log_probs = list(lps[i:j])
        s.status = Sample.Status.COMPLETED
        out.append(s)
        i = j
    return out


def _trajectory_sample(sample: Sample, traj: dict) -> Sample:
    toks, mask, lps = traj["token_ids"], traj["loss_mask"], traj["logprobs"]
    start = mask.index(1) if 1 in mask else len(toks)
    s = copy.deepcopy(sample)
    s.tokens = list(toks)
    s.response_length = len(toks) - start
    s.loss_mask = list(mask[start:])
    s.rollout_log_probs = list(lps[start:])
    s.status = Sample.Status.COMPLETED
    return s


def _truncate(s: Sample, max_len: int) -> Sample | None:
    if len(s.tokens) <= max_len:
        return s
    cut = len(s.tokens) - max_len
    if cut >= s.response_length:
        return None  # the prompt alone exceeds the budget
    s.tokens = s.tokens[:max_len]
    s.response_length -= cut
    s.loss_mask = s.loss_mask[: s.response_length]
    s.rollout_log_probs = s.rollout_log_probs[: s.response_length]
    s.status = Sample.Status.TRUNCATED
    return s


async def generate(args, sample: Sample, sampling_params: dict):
    agent = load_function(args.custom_agent_function_path)
    url = _session_url(args)
    sid = (await post(f"{url}/sessions", {}))["session_id"]
    meta = dict(sample.metadata or {})
    if getattr(args, "max_seq_len", None):
        meta["max_seq_len"] = args.max_seq_len
    extra = None
    try:
        extra = await agent(base_url=f"{url}/sessions/{sid}/v1", prompt=sample.prompt,
                            request_kwargs=request_kwargs(sampling_params), metadata=meta)
    except Exception as e:  # noqa: BLE001 - a failing agent still yields what it recorded
        log.warning("agent function failed in session %s: %s", sid, e)
    traj = await get(f"{url}/sessions/{sid}")
    try:
        import requests

        requests.delete(f"{url}/sessions/{sid}", timeout=10)
    except Exception:  # noqa: BLE001
        pass
    if not traj.get("token_ids") or 1 not in traj.get("loss_mask", []):
        s = copy.deepcopy(sample)
        s.status = Sample.Status.ABORTED
        return s
    samples = _turn_samples(sample, traj) if getattr(args, "generate_multi_samples", False) \
        else [_trajectory_sample(sample, traj)]
    if getattr(args, "max_seq_len", None):
        samples = [t for t in (_truncate(s, args.max_seq_len) for s in samples) if t is not None]
        if not samples:
            s = copy.deepcopy(sample)
            s.status = Sample.Status.ABORTED
            return s
    for s in samples:
        s.metadata = {**(s.metadata or {}), **(extra or {}), "num_turns": traj.get("num_turns", 1)}
    return samples if getattr(args, "generate_multi_samples", False) else samples[0]


def _add_arguments(parser):
    parser.add_argument("--custom-agent-function-path", type=str, default=None)
    parser.add_argument("--generate-multi-samples", action="store_true", default=False)
    parser.add_argument("--max-seq-len", type=int, default=None, dest="max_seq_len")


generate.add_arguments = _add_arguments
