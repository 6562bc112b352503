"""Loss variants of the actor on CPU: SFT, IcePop, OPSM, GSPO, custom TIS hook."""
import os

import numpy as np
import torch

os.environ.setdefault("MILES_B200_FORCE_CPU", "1")

from miles_b200.models.config import preset  # noqa: E402
from miles_b200.models.transformer import Transformer  # noqa: E402
from miles_b200.ops.rl import PolicyLossCfg, policy_loss_ref  # noqa: E402
from miles_b200.trainer.actor import Actor, ActorConfig, TrainItem, _seg_mean  # noqa: E402


def _items(n=4, P=8, R=6, seed=0, vocab=4096):
    rng = np.random.default_rng(seed)
    out = []
    for i in range(n):
        toks = rng.integers(0, vocab, P + R).tolist()
        out.append(TrainItem(toks, P, advantage=float(rng.standard_normal()),
                             rollout_logp=(-rng.random(R) * 3).astype(np.float32).tolist()))
    return out


def _actor(loss: PolicyLossCfg):
    m = Transformer(preset("tiny"), device="cpu", dtype=torch.float32, seed=0)
    return Actor(m, ActorConfig(lr=1e-3, loss=loss, optimizer_placement="device",
                                grad_dtype=torch.float32))


def test_seg_mean():
    x = torch.tensor([1.0, 3.0, 5.0, 7.0, 9.0])
    mask = torch.tensor([1.0, 1.0, 0.0, 1.0, 1.0])
    seg = torch.tensor([0, 0, 0, 1, 1])
    out = _seg_mean(x * mask, mask, seg, 2)
    assert torch.allclose(out, torch.tensor([2.0, 2.0, 2.0, 8.0, 8.0]))


def test_icepop_reference_masks_outside_band():
    lp = torch.zeros(4, requires_grad=True)
    old = torch.zeros(4)
    roll = torch.tensor([0.0, -0.1, -2.0, 3.0])  # ratios 1, 1.105, 7.39, 0.05
    cfg = PolicyLossCfg(use_tis=True, tis_mode="icepop", tis_clip_low=0.5, tis_clip=2.0)
    adv = torch.ones(4)
    w = torch.ones(4)
    loss, m = policy_loss_ref(lp, old, adv, w, cfg, roll)
    loss.backward()
    g = lp.grad
    assert g[2] == 0 and g[3] == 0 and g[0] != 0 and g[1] != 0


def test_loss_variants_train_step():
    for loss in (PolicyLossCfg(loss_type="sft_loss"),
                 PolicyLossCfg(use_tis=True, tis_mode="icepop", tis_clip_low=0.5),
                 PolicyLossCfg(use_opsm=True, opsm_delta=0.0),
                 PolicyLossCfg(gspo=True, eps_clip=3e-4, eps_clip_high=4e-4),
                 PolicyLossCfg(use_tis=True,
                               custom_tis_path="miles_b200.trainer.is_functions.icepop_function")):
        a = _actor(loss)
        before = a.model.flat.clone()
        out = a.train_step(_items())
        assert np.isfinite(out["pg_loss"]), loss
        assert not torch.equal(before, a.model.flat), loss


def test_sft_loss_is_nll():
    a = _actor(PolicyLossCfg(loss_type="sft_loss"))
    items = _items(n=2)
    lps = a.compute_logprobs(items)
    nll = -sum(float(np.sum(x)) for x in lps) / 2  # per-sample mean weights: 1/R each, 1/n
    out = a.train_step(items)
    R = items[0].resp_len
    assert abs(out["pg_loss"] - nll / R) < 1e-3 * abs(nll / R) + 1e-5
