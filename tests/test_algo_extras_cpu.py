"""Algorithm extras on CPU: MIS weights (levels, modes, rejection + veto, batch
normalisation), the unbiased KL term, a custom pg-loss reducer, pass@k, CI model hashes and
grad-norm checks, and the mismatch metrics."""
import math
import os
import types

import numpy as np
import pytest
import torch

os.environ.setdefault("MILES_B200_FORCE_CPU", "1")


def _args(**kw):
    base = dict(use_tis=True, tis_level="token", tis_mode="truncate", tis_upper_bound=2.0,
                tis_lower_bound=None, use_rs=False, rs_level=None, rs_lower_bound=None,
                rs_upper_bound=None, rs_veto_threshold=None, tis_batch_normalize=False)
    base.update(kw)
    return types.SimpleNamespace(**base)


def test_mis_levels_and_modes():
    from miles_b200.trainer.mis import compute_mis_weights

    t = [torch.tensor([0.0, -1.0, -2.0]), torch.tensor([-0.5, -0.5])]
    r = [torch.tensor([-1.0, -1.0, -1.0]), torch.tensor([-0.5, -1.5])]
    m = [torch.ones(3), torch.tensor([1.0, 1.0])]
    pg = torch.ones(5)
    out, masks, _ = compute_mis_weights(_args(), pg_loss=pg, train_log_probs=t,
                                        rollout_log_probs=r, loss_masks=m)
    assert torch.allclose(out, torch.tensor([2.0, 1.0, math.exp(-1), 1.0, 2.0]))  # e^1 truncated at 2
    out, _, _ = compute_mis_weights(_args(tis_level="sequence", tis_upper_bound=10.0), pg_loss=pg,
                                    train_log_probs=t, rollout_log_probs=r, loss_masks=m)
    assert torch.allclose(out[:3], torch.full((3,), 1.0)) and torch.allclose(out[3:], torch.full((2,), math.e))
    out, _, _ = compute_mis_weights(_args(tis_level="geometric", tis_upper_bound=10.0), pg_loss=pg,
                                    train_log_probs=t, rollout_log_probs=r, loss_masks=m)
    assert torch.allclose(out[3:], torch.full((2,), math.exp(0.5)))
    _, masks, _ = compute_mis_weights(_args(tis_mode="mask"), pg_loss=pg, train_log_probs=t,
                                      rollout_log_probs=r, loss_masks=m)
    assert masks[0].tolist() == [0.0, 1.0, 0.0] and masks[1].tolist() == [1.0, 0.0]
    _, masks, _ = compute_mis_weights(_args(use_rs=True, rs_veto_threshold=0.5), pg_loss=pg,
                                      train_log_probs=t, rollout_log_probs=r, loss_masks=m)
    assert masks[0].sum() == 0  # token with ratio e^-1 < 0.5 vetoes the whole sample
    out, _, mt = compute_mis_weights(_args(tis_batch_normalize=True), pg_loss=pg, train_log_probs=t,
                                     rollout_log_probs=r, loss_masks=m)
    assert abs(float(out.mean()) - 1.0) < 1e-6 and "batch_norm_factor" in mt


def test_unbiased_kl_and_custom_reducer():
    from miles_b200.ops.rl import PolicyLossCfg, policy_loss

    g = torch.Generator().manual_seed(0)
    lp = (-torch.rand(6, generator=g)).requires_grad_()
    old, ref = -torch.rand(6, generator=g), -torch.rand(6, generator=g)
    adv, w = torch.randn(6, generator=g), torch.full((6,), 1 / 6)
    cfg = PolicyLossCfg(kl_coef=0.5, kl_type="k1", unbiased_kl=True)
    loss, _ = policy_loss(lp, old, adv, w, cfg, None, ref)
    base, _ = policy_loss(lp, old, adv, w, PolicyLossCfg(), None, ref)
    kl = (lp - ref) * (lp - old).exp()
    assert torch.allclose(loss, base + 0.5 * (w * kl).sum())
    # a custom reducer replaces the weighted sum of the pg term
    red_loss, m = policy_loss(lp, old, adv, w, PolicyLossCfg(), None, None, pg_reducer=lambda x: x.max())
    ratio = (lp - old).exp()
    pg = torch.maximum(-adv * ratio, -adv * ratio.clamp(0.8, 1.2))
    assert torch.allclose(red_loss, pg.max(), atol=1e-6)
    red_loss.backward()
    assert lp.grad is not None


def test_pass_at_k():
    from miles_b200.utils.metric_utils import compute_pass_rate, pass_at_k

    assert pass_at_k(4, 0, 2) == 0.0 and pass_at_k(4, 4, 1) == 1.0
    assert pass_at_k(4, 1, 1) == pytest.approx(0.25) and pass_at_k(4, 1, 2) == pytest.approx(0.5)
    out = compute_pass_rate([1, 0, 0, 0, 1, 1, 0, 0], 4)
    assert out["pass@1"] == pytest.approx((0.25 + 0.5) / 2)
    assert set(out) == {"pass@1", "pass@2", "pass@4"} and out["pass@4"] == 1.0


def test_ci_hashes_and_grad_norm(tmp_path):
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer
    from miles_b200.utils.ci_utils import check_grad_norm, check_model_hashes, save_model_hashes

    m = Transformer(preset("tiny"), device="cpu", dtype=torch.float32, seed=0)
    a = types.SimpleNamespace(ci_test=True, ci_save_model_hash=True, ci_check_model_hash=True,
                              save=str(tmp_path), load=str(tmp_path),
                              ci_save_grad_norm=str(tmp_path / "gn_{role}_{rollout_id}_{step_id}.pt"),
                              ci_load_grad_norm=None)
    save_model_hashes(a, m, 3)
    check_model_hashes(a, m, 3)
    m.flat[0] += 1.0
    with pytest.raises(AssertionError):
        check_model_hashes(a, m, 3)
    check_grad_norm(a, 1.25, 0, 1)
    b = types.SimpleNamespace(ci_save_grad_norm=None, ci_load_grad_norm=a.ci_save_grad_norm)
    check_grad_norm(b, 1.26, 0, 1)
    with pytest.raises(AssertionError):
        check_grad_norm(b, 2.0, 0, 1)


def test_mismatch_metrics():
    from miles_b200.trainer.mis import mismatch_metrics

    out = mismatch_metrics([np.array([0.0, -1.0])], [np.array([0.0, -0.5])], [[1, 1]])
    assert out["train/mismatch_abs_logprob_diff"] == pytest.approx(0.25)
    assert out["train/mismatch_max_abs_logprob_diff"] == pytest.approx(0.5)
