"""Reference / old-actor weight handling: --ref-load (HF or torch_dist, --ref-ckpt-step),
--ref-update-interval and the --keep-old-actor queue."""
import os

import torch

os.environ.setdefault("MILES_B200_FORCE_CPU", "1")


def _setup(tmp_path, extra):
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer
    from miles_b200.trainer.actor import Actor, ActorConfig
    from miles_b200.trainer.train_actor import TrainActor
    from miles_b200.utils.arguments import parse_args

    args = parse_args(["--model-name", "tiny", "--use-kl-loss", "--kl-loss-coef", "0.1",
                       "--rollout-batch-size", "2", "--n-samples-per-prompt", "2"] + extra)
    m = Transformer(preset("tiny"), device="cpu", dtype=torch.float32, seed=0)
    a = Actor(m, ActorConfig(grad_dtype=torch.float32, optimizer_placement="device"))
    return m, TrainActor(args, a)


def test_ref_load_hf_and_torch_dist(tmp_path):
    from miles_b200.checkpoint.hf import save_hf
    from miles_b200.checkpoint.torch_dist import save_checkpoint
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer

    other = Transformer(preset("tiny"), device="cpu", dtype=torch.float32, seed=7)
    save_hf(other, str(tmp_path / "hf"))
    save_checkpoint(str(tmp_path / "td"), 3, other, None, save_optim=False)
    for path, ex in ((tmp_path / "hf", []), (tmp_path / "td", ["--ref-ckpt-step", "3"])):
        m, ta = _setup(tmp_path, ["--ref-load", str(path)] + ex)
        before = m.flat.clone()
        ta.init_ref()
        assert torch.equal(m.flat, before)                  # the actor keeps its own weights
        assert torch.equal(ta.backuper.backups["ref"], other.flat)


def test_ref_update_interval_and_old_actor_queue(tmp_path):
    m, ta = _setup(tmp_path, ["--ref-update-interval", "2", "--keep-old-actor"])
    ta.init_ref()
    w0 = m.flat.clone()
    m.flat.add_(1.0)                                         # "update" of rollout 0
    ta.after_update(0)
    assert torch.equal(ta.backuper.backups["ref"], w0)       # not due yet
    assert torch.equal(ta.backuper.backups["old_actor"], w0)
    assert torch.equal(ta.backuper.backups["rollout_actor"], m.flat)
    w1 = m.flat.clone()
    m.flat.add_(1.0)                                         # rollout 1
    ta.after_update(1)
    assert torch.equal(ta.backuper.backups["ref"], m.flat)   # refreshed every 2 rollouts
    assert torch.equal(ta.backuper.backups["old_actor"], w1)
