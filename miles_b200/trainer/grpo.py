"""Colocated GRPO/PPO step: generate -> reward -> advantage -> log-probs -> policy update.

The public entry point `ColocatedRL.step(prompt_batches)` is the synchronous loop body of the
reference's train.py (train.py:69-102) executed inside one process per GPU: the rollout engine
and the trainer share the parameter buffer, so the reference's offload / onload / refit
(CUDA-IPC) sequence reduces to releasing the KV cache before training, releasing gradient
memory before rollout, and bumping the weight version.

Reference: train.py, miles/ray/rollout.py (generate :445-455, reward post-process with GRPO
group normalisation :640-665, train-data conversion :667-738), megatron_utils/actor.py.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np
import torch

from miles_b200.engine.engine import GenRequest, RolloutEngine
from miles_b200.ops.rl import grpo_advantages
from miles_b200.trainer.actor import Actor, ActorConfig, TrainItem
from miles_b200.utils.flops import train_tflops
from miles_b200.utils.types import Sample


@dataclass
class RLConfig:
    n_samples_per_prompt: int = 8
    temperature: float = 1.0
    max_new_tokens: int = 1024
    advantage_estimator: str = "grpo"      # grpo | gspo | reinforce_plus_plus(_baseline) | ...
    normalize_std: bool = True
    routing_replay: bool = False
    check_logprob_parity: bool = True
    eos_token_id: int | None = None
    seed: int = 0
    # partial rollout (reference --partial-rollout with --over-sampling-batch-size): the rollout
    # stops once `groups_per_step` groups are complete; unfinished groups keep their tokens,
    # log-probs and routing and continue in the next step's rollout (re-prefilled under the new
    # weights, like the reference's SGLang engines). The caller keeps `groups_per_step *
    # over_sampling` groups in flight by feeding `prompts_needed()` fresh prompts per step.
    partial_rollout: bool = False
    groups_per_step: int | None = None
    over_sampling: int = 1


class ColocatedRL:
    def __init__(self, engine: RolloutEngine, actor: Actor, cfg: RLConfig, reward_fn=None):
        self.engine = engine
        self.actor = actor
        self.cfg = cfg
        self.reward_fn = reward_fn
        self.rollout_id = 0
        self.last_metrics: dict = {}
        self.buffer: list[list[Sample]] = []   # unfinished groups (partial rollout)
        self._next_uid = 0
        self._next_group = 0
        self.generated_tokens = 0

    def prompts_needed(self) -> int:
        """Fresh prompt groups the next step() wants (partial rollout keeps the in-flight count
        at groups_per_step * over_sampling; without it, whatever the caller passes)."""
        if not self.cfg.partial_rollout:
            return self.cfg.groups_per_step or 0
        return self.cfg.groups_per_step * self.cfg.over_sampling - len(self.buffer)

    def _new_groups(self, prompts, max_new, rewards):
        cfg = self.cfg
        groups = []
        for gi, p in enumerate(prompts):
            g = []
            for j in range(cfg.n_samples_per_prompt):
                idx = gi * cfg.n_samples_per_prompt + j
                uid = self._next_uid
                self._next_uid += 1
                s = Sample(group_index=self._next_group, index=uid, tokens=list(p),
                           response_length=0, loss_mask=[], rollout_log_probs=[])
                s.metadata = {"prompt_len": len(p),
                              "max_new": max_new[idx] if max_new is not None else cfg.max_new_tokens,
                              "reward": None if rewards is None else float(rewards[idx]),
                              "seed": cfg.seed * 1_000_003 + self.rollout_id * 65_537 + idx}
                g.append(s)
            self._next_group += 1
            groups.append(g)
        return groups

    def generate(self, prompts: list[list[int]], max_new: list[int] | None = None,
                 rewards: list[float] | None = None) -> list[Sample]:
        """Roll out the fresh prompt groups (and, with partial rollout, the buffered unfinished
        groups first). Returns the samples of the groups to train on this step."""
        cfg = self.cfg
        groups = self.buffer + self._new_groups(prompts, max_new, rewards)
        self.buffer = []
        reqs, owner = [], {}
        for g in groups:
            for s in g:
                md = s.metadata
                md["fresh_from"] = s.response_length  # tokens from here on: current weights
                left = md["max_new"] - s.response_length
                if left <= 0 or md.get("finished"):
                    continue
                if s.response_length:
                    md["resumed"] = md.get("resumed", 0) + 1
                reqs.append(GenRequest(prompt=list(s.tokens), max_new_tokens=left,
                                       temperature=cfg.temperature, seed=md["seed"],
                                       stop_token_ids=(cfg.eos_token_id,) if cfg.eos_token_id is not None else (),
                                       return_routed_experts=cfg.routing_replay, rid=s.index))
                owner[s.index] = s
        by_uid = {s.index: s for g in groups for s in g}
        gid_of = {s.index: gi for gi, g in enumerate(groups) for s in g}
        need = {gi: sum(1 for s in g if not s.metadata.get("finished")) for gi, g in enumerate(groups)}
        target = cfg.groups_per_step if cfg.partial_rollout else None

        def done_enough(results):
            fin: dict[int, int] = {}
            for rid in results:
                gi = gid_of[rid]
                fin[gi] = fin.get(gi, 0) + 1
            return sum(1 for gi, n in fin.items() if n >= need[gi]) >= target

        outs = self.engine.generate(reqs, stop_when=done_enough if target else None)
        self.generated_tokens = 0
        for o in outs:
            s = by_uid[o.rid]
            self.generated_tokens += len(o.tokens)
            plen = s.metadata["prompt_len"]
            s.tokens = s.tokens + o.tokens
            s.response_length += len(o.tokens)
            s.loss_mask = s.loss_mask + [1] * len(o.tokens)
            s.rollout_log_probs = list(s.rollout_log_probs) + list(o.logprobs)
            if o.routed_experts is not None:
                # routing of every token fed so far (prompt and earlier partial response included)
                s.rollout_routed_experts = o.routed_experts[: plen + s.response_length - 1]
            if o.finish_reason != "abort":
                s.metadata["finished"] = True
                s.update_from_meta_info(o.finish_reason, o.weight_version)
        complete = [g for g in groups if all(s.metadata.get("finished") for s in g)]
        if target:
            train, rest = complete[:target], [g for g in groups if g not in complete[:target]]
            self.buffer = rest
        else:
            train = groups
        self.last_groups = train
        return [s for g in train for s in g]

    def step(self, prompts: list[list[int]], max_new: list[int] | None = None,
             rewards: list[float] | None = None) -> dict:
        cfg = self.cfg
        t0 = time.perf_counter()
        self.actor.release_grads()
        if isinstance(prompts, torch.Tensor):  # [groups, prompt_len] token ids (any device)
            prompts = prompts.tolist()
        samples = self.generate(prompts, max_new, rewards)
        t_gen = time.perf_counter()
        self.engine.release_memory()
        rewards = [s.metadata["reward"] if s.metadata.get("reward") is not None
                   else float(self.reward_fn(s)) for s in samples]
        r = torch.tensor(rewards, dtype=torch.float32, device=self.actor.dev)
        adv = grpo_advantages(r, cfg.n_samples_per_prompt, cfg.normalize_std).cpu().numpy()
        items = [TrainItem(tokens=s.tokens, prompt_len=s.prompt_length, advantage=float(a),
                           loss_mask=s.loss_mask, rollout_logp=s.rollout_log_probs,
                           routed_experts=s.rollout_routed_experts,
                           fresh_from=s.metadata.get("fresh_from", 0))
                 for s, a in zip(samples, adv)]
        # old log-probs (forward pass); bitwise equal to the rollout's under colocated weights
        diff = 0.0
        if not self.actor.cfg.use_rollout_logprobs and not self.actor.cfg.old_logp_from_forward:
            olds = self.actor.compute_logprobs(items)
            num = 0
            for it, o in zip(items, olds):
                it.old_logp = o
                d = np.abs(o - np.asarray(it.rollout_logp, np.float32))
                diff += float(d.sum())
                num += len(d)
            diff /= max(num, 1)
        t_lp = time.perf_counter()
        dp = self.actor.dp_group
        world = torch.distributed.get_world_size(dp) if dp is not None else 1
        # loss weights are 1 / (global sample count); gradients are summed over DP ranks
        m = self.actor.train_step(items, global_num_samples=len(items) * world)
        if self.actor.cfg.old_logp_from_forward:
            diff = m.pop("train_rollout_logprob_abs_diff", 0.0)
            m["train/train_rollout_logprob_abs_diff_current_weights"] = m.pop(
                "train_rollout_logprob_abs_diff_current_weights", 0.0)
            m["train/train_rollout_logprob_current_weight_tokens"] = m.pop(
                "train_rollout_logprob_current_weight_tokens", 0.0)
        t_train = time.perf_counter()
        self.rollout_id += 1
        n_resp = sum(s.response_length for s in samples)
        n_tok = sum(len(s.tokens) for s in samples)
        m.update({
            "rollout/response_len_mean": n_resp / len(samples),
            "rollout/raw_reward": float(np.mean(rewards)),
            "train/train_rollout_logprob_abs_diff": diff,
            "perf/rollout_time": t_gen - t0,
            "perf/log_probs_time": t_lp - t_gen,
            "perf/actor_train_time": t_train - t_lp,
            "perf/step_time": t_train - t0,
            "perf/tokens_per_gpu_per_sec": self.generated_tokens / max(t_gen - t0, 1e-9),
            "rollout/generated_tokens": self.generated_tokens,
            "rollout/buffered_groups": len(self.buffer),
            "rollout/decode_steps": self.engine.stats.get("decode_steps", 0),
            "rollout/preemptions": self.engine.stats.get("preemptions", 0),
            # speculative rollout (MTP draft): accepted drafts / drafts of the step's generate
            "rollout/spec_accept_rate": (self.engine.stats.get("spec_accepted", 0)
                                         / max(self.engine.stats.get("spec_drafts", 0), 1)),
            "perf/actor_train_tok_per_s": n_tok / max(t_train - t_lp, 1e-9),
            "perf/actor_train_tflops": train_tflops(self.actor.model.cfg, [len(s.tokens) for s in samples],
                                                    t_train - t_lp),
            "tokens_total": n_tok,
            "response_tokens": n_resp,
        })
        self.last_metrics = m
        return m
