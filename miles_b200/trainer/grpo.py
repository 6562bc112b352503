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


class ColocatedRL:
    def __init__(self, engine: RolloutEngine, actor: Actor, cfg: RLConfig, reward_fn=None):
        self.engine = engine
        self.actor = actor
        self.cfg = cfg
        self.reward_fn = reward_fn
        self.rollout_id = 0
        self.last_metrics: dict = {}

    def generate(self, prompts: list[list[int]], max_new: list[int] | None = None) -> list[Sample]:
        cfg = self.cfg
        reqs = []
        samples = []
        for gi, p in enumerate(prompts):
            for j in range(cfg.n_samples_per_prompt):
                idx = gi * cfg.n_samples_per_prompt + j
                mn = max_new[idx] if max_new is not None else cfg.max_new_tokens
                reqs.append(GenRequest(prompt=list(p), max_new_tokens=mn,
                                       temperature=cfg.temperature,
                                       seed=(cfg.seed * 1_000_003 + self.rollout_id * 65_537 + idx),
                                       stop_token_ids=(cfg.eos_token_id,) if cfg.eos_token_id is not None else (),
                                       return_routed_experts=cfg.routing_replay, rid=idx))
                samples.append(Sample(group_index=gi, index=idx, tokens=list(p)))
        outs = self.engine.generate(reqs)
        for s, o in zip(samples, outs):
            s.tokens = s.tokens + o.tokens
            s.response_length = len(o.tokens)
            s.loss_mask = [1] * len(o.tokens)
            s.rollout_log_probs = o.logprobs
            s.rollout_routed_experts = o.routed_experts
            s.update_from_meta_info(o.finish_reason, o.weight_version)
        return samples

    def step(self, prompts: list[list[int]], max_new: list[int] | None = None,
             rewards: list[float] | None = None) -> dict:
        cfg = self.cfg
        t0 = time.perf_counter()
        self.actor.release_grads()
        samples = self.generate(prompts, max_new)
        t_gen = time.perf_counter()
        self.engine.release_memory()
        if rewards is None:
            rewards = [float(self.reward_fn(s)) for s in samples]
        r = torch.tensor(rewards, dtype=torch.float32, device=self.actor.dev)
        adv = grpo_advantages(r, cfg.n_samples_per_prompt, cfg.normalize_std).cpu().numpy()
        items = [TrainItem(tokens=s.tokens, prompt_len=s.prompt_length, advantage=float(a),
                           loss_mask=s.loss_mask, rollout_logp=s.rollout_log_probs,
                           routed_experts=s.rollout_routed_experts)
                 for s, a in zip(samples, adv)]
        # old log-probs (forward pass); bitwise equal to the rollout's under colocated weights
        diff = 0.0
        if not self.actor.cfg.use_rollout_logprobs:
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
            "perf/tokens_per_gpu_per_sec": n_resp / max(t_gen - t0, 1e-9),
            "perf/actor_train_tok_per_s": n_tok / max(t_train - t_lp, 1e-9),
            "tokens_total": n_tok,
            "response_tokens": n_resp,
        })
        self.last_metrics = m
        return m
