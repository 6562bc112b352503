"""Generate-function hub: single-turn, multi-turn tool calling with loss-masked observations,
and multi-sample generation.

Each function has the reference signature `async generate(args, sample, sampling_params)` and
can be selected with --custom-generate-function-path.

Multi-turn protocol: after each assistant turn, `parse_tool_calls` looks for
<tool_call>{"name": ..., "arguments": {...}}</tool_call> blocks; every call is executed through
the tool registry and its result is appended as an observation whose tokens carry loss_mask 0
(and rollout log-prob 0.0), then generation continues until no call is made, the turn limit is
hit or the response budget is exhausted.

Reference: miles/rollout/generate_hub/single_turn.py:15-46, multi_turn.py:23-88,
generate_utils/tool_call_utils.py.
"""
from __future__ import annotations

import copy
import json
import re

from miles_b200.rollout.default import GenerateState, generate as single_turn_generate
from miles_b200.utils.types import Sample

TOOLS: dict = {}


def register_tool(name: str):
    def deco(fn):
        TOOLS[name] = fn
        return fn

    return deco


@register_tool("calculator")
def _calculator(expression: str = "", **_) -> str:
    if not re.fullmatch(r"[0-9+\-*/(). eE]+", expression or ""):
        return "error: unsupported expression"
    try:
        return str(eval(expression, {"__builtins__": {}}, {}))  # arithmetic only (checked above)
    except Exception as e:
        return f"error: {e}"


_CALL_RE = re.compile(r"<tool_call>\s*(\{.*?\})\s*</tool_call>", re.S)


def parse_tool_calls(text: str) -> list[dict]:
    calls = []
    for m in _CALL_RE.finditer(text or ""):
        try:
            d = json.loads(m.group(1))
            if isinstance(d, dict) and "name" in d:
                calls.append(d)
        except json.JSONDecodeError:
            continue
    return calls


async def execute_tool(call: dict) -> str:
    fn = TOOLS.get(call.get("name"))
    if fn is None:
        return f"error: unknown tool {call.get('name')}"
    args = call.get("arguments") or {}
    if isinstance(args, str):
        try:
            args = json.loads(args)
        except json.JSONDecodeError:
            args = {}
    res = fn(**args)
    if hasattr(res, "__await__"):
        res = await res
    return str(res)


async def single_turn(args, sample: Sample, sampling_params: dict) -> Sample:
    return await single_turn_generate(args, sample, sampling_params)


def _observation_tokens(state: GenerateState, text: str) -> list[int]:
    tok = state.tokenizer
    if tok is None:  # token-level fallback: a fixed separator + byte tokens modulo vocab
        return [1] + [b % 255 + 2 for b in text.encode()[:64]]
    msg = [{"role": "tool", "content": text}]
    try:
        return tok.apply_chat_template(msg, tokenize=True, add_generation_prompt=True)
    except Exception:
        return tok(f"\n<tool_response>\n{text}\n</tool_response>\n", add_special_tokens=False)["input_ids"]


async def multi_turn(args, sample: Sample, sampling_params: dict) -> Sample:
    state = GenerateState.get(args)
    max_turns = getattr(args, "generate_max_turns", 8)
    budget = sampling_params["max_new_tokens"]
    for _ in range(max_turns):
        sp = dict(sampling_params)
        sp["max_new_tokens"] = budget - sample.response_length
        if sp["max_new_tokens"] <= 0:
            sample.status = Sample.Status.TRUNCATED
            break
        before = sample.response_length
        sample = await single_turn_generate(args, sample, sp)
        if sample.status in (Sample.Status.ABORTED, Sample.Status.FAILED):
            break
        new_text = sample.response[-(sample.response_length - before) * 8:] if state.tokenizer is None else \
            state.tokenizer.decode(sample.tokens[-(sample.response_length - before):])
        calls = parse_tool_calls(new_text)
        if not calls:
            break
        obs_tokens: list[int] = []
        for c in calls:
            obs_tokens += _observation_tokens(state, await execute_tool(c))
        if sample.response_length + len(obs_tokens) >= budget:
            sample.status = Sample.Status.TRUNCATED
            break
        sample.tokens = sample.tokens + obs_tokens
        sample.response_length += len(obs_tokens)
        sample.loss_mask = sample.loss_mask + [0] * len(obs_tokens)
        sample.rollout_log_probs = sample.rollout_log_probs + [0.0] * len(obs_tokens)
        sample.metadata["num_turns"] = sample.metadata.get("num_turns", 1) + 1
    return sample


def _add_multi_turn_arguments(parser):
    parser.add_argument("--generate-max-turns", type=int, default=8)


multi_turn.add_arguments = _add_multi_turn_arguments


async def multi_sample(args, sample: Sample, sampling_params: dict) -> list[Sample]:
    """Generate `args.n_samples_per_prompt` independent responses for one prompt."""
    outs = []
    for k in range(args.n_samples_per_prompt):
        s = copy.deepcopy(sample)
        s.index = (sample.index or 0) * args.n_samples_per_prompt + k
        outs.append(await single_turn_generate(args, s, dict(sampling_params, sampling_seed=s.index)))
    return outs
