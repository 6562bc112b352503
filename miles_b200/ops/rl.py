"""Fused RL loss kernels: clipped policy loss (+TIS, KL), GAE and GRPO advantages
(csrc/rl_ops.cu), with fp64-checkable PyTorch references used on CPU.

Reference: miles/utils/ppo_utils.py compute_policy_loss (:124-148), compute_approx_kl (:11-51),
get_advantages_and_returns / chunked GAE (:505-645), GRPO group normalisation
(miles/ray/rollout.py:640-665).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from miles_b200.ops._lib import lib, use_native

KL_TYPES = {"none": 0, "k1": 1, "k2": 2, "k3": 3, "low_var_kl": 3}
METRIC_NAMES = ["pg_loss", "pg_clipfrac", "ppo_kl", "kl_loss", "tis", "tis_clipfrac", "weight"]


@dataclass
class PolicyLossCfg:
    eps_clip: float = 0.2
    eps_clip_high: float = 0.2
    eps_clip_c: float | None = None
    use_tis: bool = False
    tis_clip_low: float = 0.0
    tis_clip: float = 2.0
    kl_coef: float = 0.0
    kl_type: str = "none"
    tis_mode: str = "tis"         # "tis": clamp the IS ratio; "icepop": zero it outside [low, high]
    loss_type: str = "policy_loss"  # policy_loss | sft_loss | custom_loss
    custom_loss_path: str | None = None
    custom_tis_path: str | None = None
    use_opsm: bool = False
    opsm_delta: float = 1e-4
    gspo: bool = False
    unbiased_kl: bool = False        # --use-unbiased-kl: KL term weighted by exp(logp - old_logp)
    custom_pg_loss_reducer_path: str | None = None


def kl_terms(logp, ref_logp, kl_type: str):
    """Per-token KL estimator of log(pi / pi_ref) (k1 / k2 / k3 = low_var_kl, clamped)."""
    kt = KL_TYPES[kl_type]
    if not kt:
        return torch.zeros_like(logp)
    lr = logp - ref_logp
    if kt == 1:
        return lr
    if kt == 2:
        return 0.5 * lr * lr
    return ((-lr).exp() + lr - 1).clamp(-10, 10)


def policy_loss_ref(logp, old_logp, adv, weight, cfg: PolicyLossCfg, rollout_logp=None,
                    ref_logp=None, pg_reducer=None):
    """Returns (loss, metrics dict) with autograd through logp. pg_reducer: optional callable
    mapping the per-token policy-gradient loss to its scalar (a custom reducer replaces the
    weighted sum for the pg term)."""
    ppo_kl = old_logp - logp
    ratio = (-ppo_kl).exp()
    pg1 = -adv * ratio
    pg2 = -adv * ratio.clamp(1 - cfg.eps_clip, 1 + cfg.eps_clip_high)
    pg = torch.maximum(pg1, pg2)
    clipfrac = (pg2 > pg1).to(logp.dtype)
    if cfg.eps_clip_c is not None and cfg.eps_clip_c > 1:
        pg3 = -adv * cfg.eps_clip_c
        pg = torch.where(adv < 0, torch.minimum(pg3, pg), pg)
    tis = torch.ones_like(logp)
    tis_clip = torch.zeros_like(logp)
    if cfg.use_tis:
        raw = (old_logp - rollout_logp).exp()
        if cfg.tis_mode == "icepop":
            tis = torch.where((raw >= cfg.tis_clip_low) & (raw <= cfg.tis_clip), raw,
                              torch.zeros_like(raw))
        else:
            tis = raw.clamp(cfg.tis_clip_low, cfg.tis_clip)
        tis_clip = (tis != raw).to(logp.dtype)
        pg = pg * tis.detach()
    kl = kl_terms(logp, ref_logp, cfg.kl_type)
    if cfg.unbiased_kl and KL_TYPES[cfg.kl_type]:
        kl = kl * (logp - old_logp).exp()  # importance ratio pi / pi_old (reference loss.py:669)
    pg_term = pg_reducer(pg) if pg_reducer is not None else (weight * pg).sum()
    loss = pg_term + (weight * cfg.kl_coef * kl).sum()
    w = weight.detach()
    m = {
        "pg_loss": float(pg_term.detach()) if pg_reducer is not None else (w * pg).sum().item(),
        "pg_clipfrac": (w * clipfrac).sum().item(),
        "ppo_kl": (w * ppo_kl).sum().item(),
        "kl_loss": (w * kl).sum().item(),
        "tis": (w * tis).sum().item(),
        "tis_clipfrac": (w * tis_clip).sum().item(),
        "weight": w.sum().item(),
    }
    return loss, m


class _PolicyLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logp, old_logp, adv, weight, rollout_logp, ref_logp, cfg: PolicyLossCfg):
        if cfg.use_tis and rollout_logp is None:
            raise ValueError("policy_loss: TIS / IcePop needs the rollout log-probs")
        if cfg.kl_type != "none" and ref_logp is None:
            raise ValueError("policy_loss: a KL term needs the reference log-probs")
        n = logp.numel()
        dev = logp.device
        dlogp = torch.empty(n, dtype=torch.float32, device=dev)
        part = torch.empty(256 * 7, dtype=torch.float32, device=dev)
        metrics = torch.empty(7, dtype=torch.float32, device=dev)
        eps_c = cfg.eps_clip_c if cfg.eps_clip_c is not None else 0.0
        lib().policy_loss(logp.float().contiguous(), old_logp.float().contiguous(),
                          adv.float().contiguous(), weight.float().contiguous(),
                          None if rollout_logp is None else rollout_logp.float().contiguous(),
                          None if ref_logp is None else ref_logp.float().contiguous(),
                          dlogp, None, part, metrics, cfg.eps_clip, cfg.eps_clip_high, eps_c,
                          cfg.tis_clip_low, cfg.tis_clip, cfg.kl_coef, KL_TYPES[cfg.kl_type],
                          (2 if cfg.tis_mode == "icepop" else 1) if cfg.use_tis else 0)
        ctx.save_for_backward(dlogp)
        loss = metrics[0] + cfg.kl_coef * metrics[3]
        ctx.mark_non_differentiable(metrics)
        return loss, metrics

    @staticmethod
    def backward(ctx, gloss, gmetrics):
        (dlogp,) = ctx.saved_tensors
        return dlogp * gloss, None, None, None, None, None, None


def policy_loss(logp, old_logp, adv, weight, cfg: PolicyLossCfg, rollout_logp=None, ref_logp=None,
                pg_reducer=None):
    """Fused clipped policy loss. `weight` carries mask and reduction normaliser.
    Returns (loss scalar tensor, metrics tensor [7] of weighted sums in METRIC_NAMES order).
    The unbiased KL (KL x pi / pi_old, with its gradient) and a custom pg reducer run as PyTorch
    ops around the fused kernel."""
    if not use_native(logp) or pg_reducer is not None:
        loss, m = policy_loss_ref(logp, old_logp, adv, weight, cfg, rollout_logp, ref_logp, pg_reducer)
        return loss, torch.tensor([m[k] for k in METRIC_NAMES], device=logp.device)
    if cfg.unbiased_kl and KL_TYPES[cfg.kl_type]:
        import dataclasses

        loss, m = _PolicyLoss.apply(logp, old_logp, adv, weight, rollout_logp, None,
                                    dataclasses.replace(cfg, kl_coef=0.0, kl_type="none"))
        kl = kl_terms(logp, ref_logp, cfg.kl_type) * (logp - old_logp).exp()
        loss = loss + cfg.kl_coef * (weight * kl).sum()
        m = m.clone()
        m[METRIC_NAMES.index("kl_loss")] = (weight.detach() * kl.detach()).sum()
        return loss, m
    return _PolicyLoss.apply(logp, old_logp, adv, weight, rollout_logp, ref_logp, cfg)


def gae_ref(rewards, values, cu, gamma, lam):
    adv = torch.zeros_like(rewards)
    for b in range(len(cu) - 1):
        last = 0.0
        nv = 0.0
        for t in range(cu[b + 1] - 1, cu[b] - 1, -1):
            delta = rewards[t] + gamma * nv - values[t]
            last = delta + gamma * lam * last
            adv[t] = last
            nv = values[t]
    return adv, adv + values


def gae(rewards, values, cu: list[int], gamma: float, lam: float):
    """Packed GAE. rewards/values fp32 [N]; cu: sequence boundaries. Returns (adv, returns)."""
    if not use_native(rewards):
        return gae_ref(rewards, values, cu, gamma, lam)
    adv = torch.empty_like(rewards)
    ret = torch.empty_like(rewards)
    cu_t = torch.tensor(cu, dtype=torch.int32, device=rewards.device)
    lib().gae(rewards.float().contiguous(), values.float().contiguous(), cu_t, gamma, lam, adv, ret)
    return adv, ret


def grpo_advantages(rewards: torch.Tensor, group_size: int, normalize_std: bool = True,
                    eps: float = 1e-6) -> torch.Tensor:
    """Group-normalised rewards: (r - mean_g) [/ (std_g + eps)] per group of `group_size`."""
    r = rewards.float().contiguous()
    if not use_native(r):
        g = r.view(-1, group_size)
        a = g - g.mean(-1, keepdim=True)
        if normalize_std:
            std = g.std(-1, keepdim=True) if group_size > 1 else torch.zeros_like(a[:, :1])
            a = a / (std + eps)
        return a.view(-1)
    adv = torch.empty_like(r)
    lib().grpo_adv(r, group_size, normalize_std, eps, adv)
    return adv
