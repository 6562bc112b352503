"""LR schedule in consumed samples: warm-up, linear / cosine / inverse-square-root decay to
--min-lr (the reference's Megatron OptimizerParamScheduler curve), driven by the actor's
optimizer steps and resumed from a checkpoint."""
import math
import os

import pytest

os.environ.setdefault("MILES_B200_FORCE_CPU", "1")


def test_schedule_curves():
    from miles_b200.trainer.lr_scheduler import LRSchedule

    s = LRSchedule(max_lr=1.0, min_lr=0.1, warmup_samples=10, decay_samples=110, style="linear")
    assert s.lr(0) == 0.0 and s.lr(5) == pytest.approx(0.5) and s.lr(10) == pytest.approx(1.0)
    assert s.lr(60) == pytest.approx(0.1 + 0.9 * 0.5)
    assert s.lr(110) == pytest.approx(0.1) and s.lr(500) == pytest.approx(0.1)
    c = LRSchedule(max_lr=1.0, min_lr=0.0, warmup_samples=0, decay_samples=100, style="cosine")
    assert c.lr(50) == pytest.approx(0.5) and c.lr(25) == pytest.approx(0.5 * (1 + math.cos(math.pi / 4)))
    assert LRSchedule(max_lr=2.0, style="constant").lr(10 ** 6) == 2.0
    r = LRSchedule(max_lr=1.0, min_lr=0.0, warmup_samples=4, style="inverse-square-root")
    assert r.lr(16) == pytest.approx(0.5)


def test_schedule_from_cli_args():
    from miles_b200.trainer.lr_scheduler import schedule_from_args
    from miles_b200.utils.arguments import parse_args

    args = parse_args(["--model-name", "tiny", "--lr", "1e-5", "--min-lr", "1e-6",
                       "--lr-decay-style", "cosine", "--lr-warmup-iters", "2",
                       "--rollout-batch-size", "4", "--n-samples-per-prompt", "2",
                       "--global-batch-size", "8", "--num-rollout", "10", "--adam-eps", "1e-6"])
    s = schedule_from_args(args)
    assert s.warmup_samples == 16 and s.decay_samples == 80 and s.style == "cosine"
    assert s.lr(8) == pytest.approx(0.5e-5)


def test_actor_steps_follow_schedule():
    import numpy as np
    import torch

    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer
    from miles_b200.trainer.actor import Actor, ActorConfig, TrainItem
    from miles_b200.trainer.lr_scheduler import LRSchedule

    m = Transformer(preset("tiny"), device="cpu", dtype=torch.float32, seed=0)
    sch = LRSchedule(max_lr=1e-3, min_lr=0.0, warmup_samples=4, decay_samples=12, style="linear")
    a = Actor(m, ActorConfig(grad_dtype=torch.float32, optimizer_placement="device", lr_schedule=sch,
                             adam_eps=1e-6))
    rng = np.random.default_rng(0)
    items = [TrainItem(rng.integers(0, 100, 12).tolist(), 4, advantage=1.0,
                       rollout_logp=(-rng.random(8)).tolist()) for _ in range(2)]
    lrs = [a.train_step(items)["lr"] for _ in range(4)]
    assert lrs == pytest.approx([0.0, 0.5e-3, 1e-3, 0.75e-3])
    assert a.opt.eps == 1e-6
    assert sch.state_dict() == {"samples": 8}
