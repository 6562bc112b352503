"""Default rollout function: asynchronous over-sampling with dynamic filtering, abort of
stragglers, partial rollout, per-sample reward and evaluation rollouts.

Hook signatures are the reference's:
  generate_rollout(args, rollout_id, data_source, evaluation=False) -> RolloutFnOutput | list
  generate(args, sample, sampling_params) -> Sample            (--custom-generate-function-path)
  custom_rm(args, sample) / batched for --group-rm              (--custom-rm-path)
  dynamic filter(args, samples) -> DynamicFilterOutput | bool   (--dynamic-sampling-filter-path)

Reference: miles/rollout/sglang_rollout.py (GenerateState :60-110, generate :131-231,
generate_and_rm(_group) :234-330, abort :333-374, generate_rollout_async :377-470, eval
:476-590), miles/rollout/base_types.py.
"""
from __future__ import annotations

import asyncio
import copy
import time
from dataclasses import dataclass, field

import numpy as np

from miles_b200.rollout.filter_hub import DropMetrics, as_output
from miles_b200.rollout.rm_hub import async_rm, batched_async_rm
from miles_b200.utils.misc import load_function
from miles_b200.utils.types import Sample


@dataclass
class RolloutFnTrainOutput:
    samples: list[list[Sample]]
    metrics: dict = field(default_factory=dict)


@dataclass
class RolloutFnEvalOutput:
    data: dict
    metrics: dict = field(default_factory=dict)


class GenerateState:
    """Process-wide rollout state: engine client, tokenizer, concurrency semaphore and the
    sampling parameters derived from the CLI (reference GenerateState)."""

    _inst = None

    def __init__(self, args, client=None, tokenizer=None):
        self.args = args
        self.client = client
        self.tokenizer = tokenizer
        conc = getattr(args, "sglang_server_concurrency", 512) * max(
            1, args.rollout_num_gpus // max(1, args.rollout_num_gpus_per_engine))
        self.semaphore = asyncio.Semaphore(conc)
        self.sampling_params = dict(
            temperature=args.rollout_temperature, top_p=args.rollout_top_p,
            top_k=args.rollout_top_k, max_new_tokens=args.rollout_max_response_len,
            stop=args.rollout_stop, stop_token_ids=args.rollout_stop_token_ids,
            skip_special_tokens=args.rollout_skip_special_tokens)
        self.aborted = False
        self.pendings: set = set()
        self.reset()

    @classmethod
    def get(cls, args=None, **kw):
        if cls._inst is None:
            cls._inst = cls(args, **kw)
        return cls._inst

    @classmethod
    def set(cls, state):
        cls._inst = state

    def reset(self):
        self.remaining_batch_size = 0
        self.aborted = False
        self.pendings = set()

    def submit_generate_tasks(self, groups):
        for g in groups:
            self.pendings.add(asyncio.ensure_future(generate_and_rm_group(self.args, g, copy.deepcopy(self.sampling_params))))
        self.remaining_batch_size += len(groups)


def _tokenize_prompt(state: GenerateState, sample: Sample) -> list[int]:
    p = sample.prompt
    if isinstance(p, list) and (not p or isinstance(p[0], int)):
        return list(p)
    tok = state.tokenizer
    if tok is None:
        raise ValueError("a tokenizer is needed for text prompts (--hf-checkpoint)")
    if isinstance(p, list):  # chat messages
        return tok.apply_chat_template(p, tokenize=True, add_generation_prompt=True)
    return tok(p, add_special_tokens=False)["input_ids"]


async def generate(args, sample: Sample, sampling_params: dict) -> Sample:
    """Single-turn generation; continues from `sample.tokens` for partial rollout."""
    state = GenerateState.get(args)
    if not sample.tokens:
        sample.tokens = _tokenize_prompt(state, sample)
    prompt_len = len(sample.tokens) - sample.response_length
    sp = dict(sampling_params)
    if sample.response_length:  # resume a partial response with the remaining budget
        sp["max_new_tokens"] = max(0, sp["max_new_tokens"] - sample.response_length)
    if args.rollout_max_context_len is not None:
        sp["max_new_tokens"] = min(sp["max_new_tokens"], args.rollout_max_context_len - len(sample.tokens))
    if sp["max_new_tokens"] <= 0:
        sample.status = Sample.Status.TRUNCATED
        return sample
    sp.setdefault("sampling_seed", args.rollout_seed * 1_000_003 + (sample.index or 0))
    out = await state.client.generate(sample.tokens, sp, return_logprob=True,
                                      return_routed_experts=args.use_rollout_routing_replay)
    ids = out["output_ids"]
    lps = [x[0] for x in out["meta_info"]["output_token_logprobs"]]
    sample.tokens = sample.tokens + ids
    sample.response_length += len(ids)
    sample.response = (sample.response or "") + out.get("text", "")
    sample.loss_mask = (sample.loss_mask or []) + [1] * len(ids)
    sample.rollout_log_probs = (sample.rollout_log_probs or []) + lps
    rex = out["meta_info"].get("routed_experts")
    if rex is not None:
        sample.rollout_routed_experts = np.asarray(rex, dtype=np.int32)
    sample.update_from_meta_info(out["meta_info"]["finish_reason"]["type"],
                                 out["meta_info"].get("weight_version"))
    del prompt_len
    return sample


async def generate_and_rm(args, sample: Sample, sampling_params: dict, evaluation=False) -> Sample:
    state = GenerateState.get(args)
    if sample.status == Sample.Status.COMPLETED or sample.status == Sample.Status.TRUNCATED:
        return sample
    async with state.semaphore:
        if state.aborted:
            sample.status = Sample.Status.ABORTED
            return sample
        t0 = time.perf_counter()
        gen = load_function(args.custom_generate_function_path) if args.custom_generate_function_path else generate
        sample = await gen(args, sample, sampling_params)
        for s in (sample if isinstance(sample, list) else [sample]):
            s.metadata.setdefault("gen_time", time.perf_counter() - t0)
    if isinstance(sample, list):  # a generate function that returns several samples
        if not args.group_rm:
            for s in sample:
                if s.status != Sample.Status.ABORTED and s.reward is None:
                    s.reward = await async_rm(args, s)
        return sample
    if sample.status == Sample.Status.ABORTED or args.group_rm:
        return sample
    if sample.reward is None:
        sample.reward = await async_rm(args, sample)
    return sample


async def generate_and_rm_group(args, group: list[Sample], sampling_params: dict,
                                evaluation=False) -> list[Sample]:
    state = GenerateState.get(args)
    if state.aborted:
        return group
    out = await asyncio.gather(*[generate_and_rm(args, s, sampling_params, evaluation) for s in group])
    group = [x for o in out for x in (o if isinstance(o, list) else [o])]
    if args.group_rm and not state.aborted and all(s.status != Sample.Status.ABORTED for s in group):
        await batched_async_rm(args, group, inplace_set_reward_field=True)
    return group


async def abort(args, rollout_id: int) -> list[list[Sample]]:
    """Stop outstanding work; with --partial-rollout return unfinished groups for the buffer."""
    state = GenerateState.get(args)
    state.aborted = True
    if state.client is not None and hasattr(state.client, "abort"):
        state.client.abort()
    partial = []
    if state.pendings:
        done, _ = await asyncio.wait(state.pendings)
        for t in done:
            g = t.result()
            if args.partial_rollout:
                for s in g:
                    if args.mask_offpolicy_in_partial_rollout and s.response_length:
                        s.loss_mask = [0] * s.response_length
                    s.status = Sample.Status.PENDING
                    s.reward = None
                    s.metadata["start_rollout_id"] = s.metadata.get("start_rollout_id", rollout_id)
                partial.append(g)
    state.pendings = set()
    return partial


async def generate_rollout_async(args, rollout_id: int, data_source) -> tuple[list[list[Sample]], dict]:
    state = GenerateState.get(args)
    state.reset()
    target = args.rollout_batch_size
    dyn = load_function(args.dynamic_sampling_filter_path) if args.dynamic_sampling_filter_path else None
    drops = DropMetrics()
    data: list[list[Sample]] = []
    t0 = time.perf_counter()
    while len(data) < target:
        while state.remaining_batch_size < target - len(data) + (args.over_sampling_batch_size - target):
            groups = data_source.get_samples(args.over_sampling_batch_size)
            if not groups:
                break
            state.submit_generate_tasks(groups)
        if not state.pendings:
            break
        done, state.pendings = await asyncio.wait(state.pendings, return_when=asyncio.FIRST_COMPLETED)
        for t in done:
            g = t.result()
            state.remaining_batch_size -= 1
            if dyn is not None:
                out = as_output(dyn(args, g))
                if not out.keep:
                    drops.add(out.reason)
                    continue
            if len(data) < target:
                data.append(g)
    partial = await abort(args, rollout_id)
    if partial and hasattr(data_source, "add_samples"):
        data_source.add_samples(partial)
    data.sort(key=lambda g: g[0].index)
    if args.rollout_sample_filter_path:
        filt = load_function(args.rollout_sample_filter_path)
        filt(args, data)
    if args.rollout_all_samples_process_path:
        load_function(args.rollout_all_samples_process_path)(args, data, data_source)
    metrics = drops.to_dict()
    metrics["rollout/time"] = time.perf_counter() - t0
    return data, metrics


def run(coro):
    """Run a coroutine on the rollout event loop (a dedicated loop per process)."""
    try:
        loop = asyncio.get_running_loop()
    except RuntimeError:
        loop = None
    if loop is not None and loop.is_running():
        raise RuntimeError("run() called from inside an event loop")
    if not hasattr(run, "_loop"):
        run._loop = asyncio.new_event_loop()
    return run._loop.run_until_complete(coro)


def generate_rollout(args, rollout_id: int, data_source, evaluation: bool = False):
    if evaluation:
        return run(eval_rollout(args, rollout_id))
    groups, metrics = run(generate_rollout_async(args, rollout_id, data_source))
    return RolloutFnTrainOutput(groups, metrics)


async def eval_rollout(args, rollout_id: int) -> RolloutFnEvalOutput:
    """Evaluate every configured dataset (n samples per prompt, eval sampling params)."""
    from miles_b200.rollout.data import Dataset

    state = GenerateState.get(args)
    out, metrics = {}, {}
    datasets = getattr(args, "eval_datasets", None) or []
    if not datasets and args.eval_prompt_data:
        it = iter(args.eval_prompt_data)
        datasets = [{"name": n, "path": p} for n, p in zip(it, it)]
    for ds in datasets:
        # per-dataset settings (--eval-config) fall back to the eval flags
        opt = lambda key, flag: ds.get(key) if ds.get(key) is not None else getattr(args, flag, None)  # noqa: E731
        d = Dataset(ds["path"], state.tokenizer, prompt_key=opt("input_key", "eval_input_key") or args.input_key,
                    label_key=opt("label_key", "eval_label_key") or args.label_key,
                    tool_key=opt("tool_key", "eval_tool_key") or getattr(args, "tool_key", None))
        sp = dict(state.sampling_params, temperature=opt("temperature", "eval_temperature"),
                  max_new_tokens=opt("max_response_len", "eval_max_response_len"))
        for key, flag in (("top_p", "eval_top_p"), ("top_k", "eval_top_k"),
                          ("min_new_tokens", "eval_min_new_tokens"), ("stop_token_ids", None)):
            v = ds.get(key) if ds.get(key) is not None else (getattr(args, flag, None) if flag else None)
            if v is not None:
                sp[key] = v
        n_per = int(opt("n_samples_per_eval_prompt", "n_samples_per_eval_prompt") or 1)
        dargs = args
        if ds.get("rm_type"):
            dargs = copy.copy(args)
            dargs.rm_type = ds["rm_type"]
        max_prompt = getattr(args, "eval_max_prompt_len", None)
        max_ctx = getattr(args, "eval_max_context_len", None)
        tasks = []
        for s in d.samples:
            if max_prompt and len(s.tokens) > max_prompt:
                continue  # --eval-max-prompt-len drops longer prompts
            spp = sp
            if max_ctx:  # --eval-max-context-len caps prompt + response
                spp = dict(sp, max_new_tokens=max(0, min(sp["max_new_tokens"] or max_ctx,
                                                         max_ctx - len(s.tokens))))
            for k in range(n_per):
                c = copy.deepcopy(s)
                c.index = (s.index or 0) * n_per + k
                tasks.append(generate_and_rm(dargs, c, spp, evaluation=True))
        samples = await asyncio.gather(*tasks)
        key = getattr(args, "eval_reward_key", None)
        rewards = [(s.reward.get(key, 0.0) if key and isinstance(s.reward, dict) else
                    s.get_reward_value(dargs)) if s.reward is not None else 0.0 for s in samples]
        out[ds["name"]] = {"rewards": rewards, "samples": samples,
                           "truncated": [int(s.status == Sample.Status.TRUNCATED) for s in samples]}
        metrics[f"eval/{ds['name']}"] = float(np.mean(rewards)) if rewards else 0.0
        if out[ds["name"]]["truncated"]:
            metrics[f"eval/{ds['name']}-truncated_ratio"] = float(np.mean(out[ds["name"]]["truncated"]))
        if getattr(args, "log_passrate", False):
            from miles_b200.utils.metric_utils import compute_pass_rate

            for k, v in compute_pass_rate(rewards, n_per).items():
                metrics[f"eval/{ds['name']}-{k}"] = v
    return RolloutFnEvalOutput(out, metrics)
