"""Advantage / return estimators and the conversion of rollout data into train items.

  grpo / gspo                 : advantage = normalised group reward, broadcast over tokens
  reinforce_plus_plus         : discounted return of (reward at the last token - kl_coef * KL)
  reinforce_plus_plus_baseline: group-mean-subtracted reward broadcast, then whitened
  ppo                         : GAE over critic values (fused GAE kernel)
  on_policy_distillation      : per-token teacher log-prob - student log-prob
Optional masked whitening over the data-parallel group (--normalize-advantages).

Reference: training_utils/loss.py compute_advantages_and_returns (:279-447),
utils/ppo_utils.py (get_grpo_returns, get_reinforce_plus_plus_returns, GAE :505-645),
utils/distributed_utils.py masked whitening (:131).
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from miles_b200.ops.rl import gae
from miles_b200.trainer.actor import TrainItem


def discounted_returns(token_rewards: np.ndarray, gamma: float) -> np.ndarray:
    out = np.zeros_like(token_rewards)
    run = 0.0
    for t in range(len(token_rewards) - 1, -1, -1):
        run = token_rewards[t] + gamma * run
        out[t] = run
    return out


def masked_whiten(advs: list[np.ndarray], masks: list[np.ndarray], group=None, eps: float = 1e-8):
    """Whiten token advantages with mean/std over all masked tokens of all DP ranks."""
    s = np.array([0.0, 0.0, 0.0])
    for a, m in zip(advs, masks):
        s += [float((a * m).sum()), float((a * a * m).sum()), float(m.sum())]
    if group is not None and dist.is_initialized() and dist.get_world_size(group) > 1:
        t = torch.tensor(s, dtype=torch.float64)
        dist.all_reduce(t, group=group)
        s = t.numpy()
    mean = s[0] / max(s[2], 1)
    var = s[1] / max(s[2], 1) - mean * mean
    inv = 1.0 / np.sqrt(max(var, 0.0) + eps)
    return [(a - mean) * inv * m for a, m in zip(advs, masks)]


def compute_advantages(args, data: dict, log_probs: list[np.ndarray] | None = None,
                       ref_log_probs: list[np.ndarray] | None = None,
                       values: list[np.ndarray] | None = None, dp_group=None):
    """Returns (advantages per sample [token arrays], returns per sample)."""
    est = args.advantage_estimator
    rewards = data["rewards"]
    n = len(rewards)
    resp = data["response_lengths"]
    masks = [np.asarray(m, np.float32) for m in data["loss_masks"]]
    advs, rets = [], []
    kl = None
    if log_probs is not None and ref_log_probs is not None and args.kl_coef:
        kl = [np.asarray(lp) - np.asarray(rl) for lp, rl in zip(log_probs, ref_log_probs)]
    if est in ("grpo", "gspo"):
        for i in range(n):
            a = np.full(resp[i], rewards[i], np.float32)
            advs.append(a)
            rets.append(a)
    elif est == "reinforce_plus_plus":
        for i in range(n):
            r = np.zeros(resp[i], np.float32)
            if kl is not None:
                r -= args.kl_coef * kl[i]
            if resp[i]:
                r[-1] += rewards[i]
            ret = discounted_returns(r * masks[i], args.gamma)
            advs.append(ret.astype(np.float32))
            rets.append(ret.astype(np.float32))
        advs = masked_whiten(advs, masks, dp_group)
    elif est == "reinforce_plus_plus_baseline":
        for i in range(n):
            a = np.full(resp[i], rewards[i], np.float32)
            if kl is not None:
                a = a - args.kl_coef * kl[i]
            advs.append(a)
            rets.append(a)
        advs = masked_whiten(advs, masks, dp_group)
    elif est == "ppo":
        assert values is not None, "PPO needs critic values"
        tok_r, vals, cu = [], [], [0]
        for i in range(n):
            r = np.zeros(resp[i], np.float32)
            if kl is not None:
                r -= args.kl_coef * kl[i]
            if resp[i]:
                r[-1] += rewards[i]
            tok_r.append(r)
            vals.append(np.asarray(values[i], np.float32))
            cu.append(cu[-1] + resp[i])
        R = torch.from_numpy(np.concatenate(tok_r)) if tok_r else torch.zeros(0)
        V = torch.from_numpy(np.concatenate(vals)) if vals else torch.zeros(0)
        dev = torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")
        A, Rt = gae(R.to(dev), V.to(dev), cu, args.gamma, args.lambd)
        A, Rt = A.cpu().numpy(), Rt.cpu().numpy()
        advs = [A[cu[i]:cu[i + 1]] for i in range(n)]
        rets = [Rt[cu[i]:cu[i + 1]] for i in range(n)]
        if args.normalize_advantages:
            advs = masked_whiten(advs, masks, dp_group)
    elif est == "on_policy_distillation":
        teacher = data["teacher_log_probs"]
        for i in range(n):
            a = np.asarray(teacher[i], np.float32) - np.asarray(log_probs[i], np.float32)
            advs.append(a)
            rets.append(a)
    else:
        raise ValueError(f"unknown advantage estimator {est}")
    if args.normalize_advantages and est in ("grpo", "gspo"):
        advs = masked_whiten(advs, masks, dp_group)
    return advs, rets


def data_to_items(data: dict, advantages=None) -> list[TrainItem]:
    items = []
    for i, toks in enumerate(data["tokens"]):
        rl = data["response_lengths"][i]
        items.append(TrainItem(
            tokens=list(toks), prompt_len=len(toks) - rl,
            advantage=advantages[i] if advantages is not None else float(data["rewards"][i]),
            loss_mask=list(data["loss_masks"][i]),
            rollout_logp=data.get("rollout_log_probs", [None] * len(data["tokens"]))[i],
            routed_experts=data.get("rollout_routed_experts", [None] * len(data["tokens"]))[i]))
    return items
