"""Learning-rate schedule counted in consumed samples (warm-up, then constant / linear /
cosine / inverse-square-root decay to --min-lr).

The reference builds Megatron's OptimizerParamScheduler with iteration counts scaled by the
global batch size (miles/backends/megatron_utils/model.py:49-96): train_iters = num_rollout *
rollout_batch_size * n_samples_per_prompt / global_batch_size, lr_decay_iters defaults to it,
warm-up is --lr-warmup-iters iterations or --lr-warmup-fraction of the decay span, and the
scheduler advances by the global batch size after every optimizer step. This module computes the
same curve from its definition:

  warm-up  (s < W):        lr = init + (max - init) * s / W
  decay    (W <= s <= D):  r = (s - W) / (D - W)
                           linear:  lr = min + (max - min) * (1 - r)
                           cosine:  lr = min + (max - min) * (1 + cos(pi r)) / 2
                           inverse-square-root: lr = max * sqrt(max(W, 1)) / sqrt(max(s, 1)),
                                                floored at min
  after    (s > D):        lr = min   (constant: lr = max throughout, after warm-up)
"""
from __future__ import annotations

import math
from dataclasses import dataclass


@dataclass
class LRSchedule:
    max_lr: float
    min_lr: float = 0.0
    init_lr: float = 0.0
    warmup_samples: int = 0
    decay_samples: int = 0
    style: str = "constant"          # constant | linear | cosine | inverse-square-root
    samples: int = 0                 # consumed samples (checkpointed)

    def __post_init__(self):
        if self.style not in ("constant", "linear", "cosine", "inverse-square-root"):
            raise ValueError(f"unknown --lr-decay-style {self.style}")
        if self.style in ("linear", "cosine") and self.decay_samples <= self.warmup_samples:
            if self.decay_samples > 0 or self.warmup_samples > 0:
                raise ValueError("the LR decay span must be longer than the warm-up")

    def lr(self, samples: int | None = None) -> float:
        s = self.samples if samples is None else samples
        W = self.warmup_samples
        if W > 0 and s < W:
            return self.init_lr + (self.max_lr - self.init_lr) * s / W
        if self.style == "constant":
            return self.max_lr
        if self.style == "inverse-square-root":
            return max(self.min_lr, self.max_lr * math.sqrt(max(W, 1)) / math.sqrt(max(s, 1)))
        D = self.decay_samples
        if D <= 0 or s > D:
            return self.min_lr if D > 0 else self.max_lr
        r = (s - W) / (D - W)
        coeff = 1.0 - r if self.style == "linear" else 0.5 * (math.cos(math.pi * r) + 1.0)
        return self.min_lr + (self.max_lr - self.min_lr) * coeff

    def advance(self, n: int) -> None:
        self.samples += int(n)

    def state_dict(self) -> dict:
        return {"samples": self.samples}

    def load_state_dict(self, d: dict) -> None:
        self.samples = int(d.get("samples", 0))


def schedule_from_args(args, lr: float | None = None, warmup_iters: int | None = None) -> LRSchedule:
    """Build the schedule of the reference's CLI (iterations are optimizer steps of
    --global-batch-size samples)."""
    gbs = args.global_batch_size or (args.rollout_batch_size * args.n_samples_per_prompt)
    n_steps = getattr(args, "num_steps_per_rollout", None) or 1
    train_iters = max(1, (args.num_rollout or 1) * n_steps)
    decay_iters = args.lr_decay_iters if args.lr_decay_iters is not None else train_iters
    decay = decay_iters * gbs
    if args.lr_warmup_fraction is not None:
        warm = int(args.lr_warmup_fraction * decay)
    else:
        warm = (args.lr_warmup_iters if warmup_iters is None else warmup_iters) * gbs
    return LRSchedule(max_lr=args.lr if lr is None else lr, min_lr=args.min_lr,
                      init_lr=getattr(args, "lr_warmup_init", 0.0) or 0.0, warmup_samples=warm,
                      decay_samples=decay, style=args.lr_decay_style)


def schedule_state(actor) -> dict:
    """Checkpoint `extra` entry of an actor's LR schedule (empty without one)."""
    sch = getattr(getattr(actor, "cfg", None), "lr_schedule", None)
    return {"lr_schedule": sch.state_dict()} if sch is not None else {}


def restore_schedule(actor, info: dict) -> None:
    """Resume an actor's LR schedule from a checkpoint's `extra` entry."""
    sch = getattr(getattr(actor, "cfg", None), "lr_schedule", None)
    st = info.get("extra", {}).get("lr_schedule")
    if sch is not None and st is not None:
        sch.load_state_dict(st)
