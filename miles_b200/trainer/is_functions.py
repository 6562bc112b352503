"""Train/rollout mismatch importance-sampling corrections with the reference's hook signature
(`--custom-tis-function-path`): fn(args, *, pg_loss, train_log_probs, rollout_log_probs,
loss_masks, **kw) -> (pg_loss, loss_masks, metrics).

The two built-in corrections also run inside the fused policy-loss kernel (csrc/rl_ops.cu):
naming one of them on the command line selects the kernel mode instead of a host-side pass.

Reference: miles/backends/training_utils/loss.py vanilla_tis_function (:450-471) and
icepop_function (:474-497).
"""
from __future__ import annotations

import torch


def _ratio(train_log_probs, rollout_log_probs):
    old = torch.cat(list(train_log_probs), 0)
    roll = torch.cat(list(rollout_log_probs), 0)
    return torch.exp(old - roll)


def vanilla_tis_function(args, *, pg_loss, train_log_probs, rollout_log_probs, loss_masks, **kw):
    """Truncated IS: weight = clamp(exp(old - rollout), tis_clip_low, tis_clip)."""
    r = _ratio(train_log_probs, rollout_log_probs)
    lo = getattr(args, "tis_clip_low", 0.0) if args is not None else 0.0
    hi = getattr(args, "tis_clip", 2.0) if args is not None else 2.0
    w = r.clamp(lo, hi)
    return pg_loss * w, loss_masks, {"tis": r.detach(), "tis_clipfrac": (w != r).float(),
                                     "tis_abs": (r - 1).abs().detach()}


def icepop_function(args, *, pg_loss, train_log_probs, rollout_log_probs, loss_masks, **kw):
    """IcePop: keep the IS ratio inside [tis_clip_low, tis_clip], zero the token otherwise."""
    r = _ratio(train_log_probs, rollout_log_probs)
    lo = getattr(args, "tis_clip_low", 0.0) if args is not None else 0.0
    hi = getattr(args, "tis_clip", 2.0) if args is not None else 2.0
    w = torch.where((r >= lo) & (r <= hi), r, torch.zeros_like(r))
    return pg_loss * w, loss_masks, {"tis": r.detach(), "tis_clipfrac": (w != r).float(),
                                     "tis_abs": (r - 1).abs().detach()}


# fused-kernel modes for the built-in functions (reference module paths and ours)
KERNEL_MODES = {
    "miles.backends.training_utils.loss.vanilla_tis_function": "tis",
    "miles.backends.training_utils.loss.icepop_function": "icepop",
    "miles_b200.trainer.is_functions.vanilla_tis_function": "tis",
    "miles_b200.trainer.is_functions.icepop_function": "icepop",
}
