"""Train / inference mismatch importance sampling (MIS): truncated / clipped / masked IS weights
at token, sequence or geometric level, rejection sampling with a catastrophic-token veto, and
optional batch normalisation of the weights.

Use it as the custom TIS function of the policy loss:

    --use-tis --custom-tis-function-path miles_b200.trainer.mis.compute_mis_weights \
        --custom-config-path mis.yaml      # tis_level, tis_mode, tis_upper_bound, use_rs, ...

Definitions, per sample with response log-probs of the trainer (old policy) t and of the
rollout engine r, and loss mask m (d = t - r per token):

  level   token: l = d;  sequence: l = sum_m(d) on every token;  geometric: l = mean_m(d)
  weight  w = exp(clamp(l, -20, 20))
  tis_mode  truncate: min(w, U);  clip: clamp(w, L, U);  mask: w kept, tokens outside [L, U]
            leave the loss mask
  rs (use_rs): tokens whose rs-level weight is outside [rs_L, rs_U] leave the loss mask; with
            rs_veto_threshold v, a sample with any token of d < log v leaves entirely
  tis_batch_normalize: weights divided by their batch mean (token level: over masked tokens;
            sequence level: mean of per-sample means)

L defaults to 1 / U, the rs bounds to the tis bounds. Returns (pg_loss * w, masks, metrics).

Reference: examples/train_infer_mismatch_helper/mis.py compute_mis_weights (:151-310) and its
mis.yaml; the function signature is the reference's custom-TIS hook.
"""
from __future__ import annotations

import math

import torch

SAFETY = 20.0


def _level(d: torch.Tensor, m: torch.Tensor, level: str) -> torch.Tensor:
    if level == "token":
        return d
    if level == "sequence":
        return (d * m).sum().expand_as(d)
    if level == "geometric":
        return ((d * m).sum() / m.sum().clamp_min(1)).expand_as(d)
    raise ValueError(f"unknown MIS level {level}")


def _get(args, name, default=None):
    v = getattr(args, name, None)
    return default if v is None else v


def _mean_metric(metrics: dict, key: str, x: torch.Tensor, m: torch.Tensor):
    metrics.setdefault(key, []).append(((x.float() * m).sum() / m.sum().clamp_min(1)).detach())


def compute_mis_weights(args, *, pg_loss: torch.Tensor, train_log_probs, rollout_log_probs,
                        loss_masks, **kw):
    """pg_loss: concatenated per-token loss (or ones); train / rollout log-probs and loss masks:
    one 1-D tensor per sample. Returns (pg_loss * weights, per-sample masks, metrics of means)."""
    U = float(_get(args, "tis_upper_bound", _get(args, "tis_clip", 2.0)))
    L = float(_get(args, "tis_lower_bound", 1.0 / U))
    rs_L = float(_get(args, "rs_lower_bound", L))
    rs_U = float(_get(args, "rs_upper_bound", U))
    tis_level = _get(args, "tis_level", "token")
    tis_mode = _get(args, "tis_mode", "truncate")
    if tis_mode == "tis":       # the fused-kernel names of the standard modes
        tis_mode = "clip"
    elif tis_mode == "icepop":
        tis_mode = "mask"
    use_tis = bool(_get(args, "use_tis", True))
    use_rs = bool(_get(args, "use_rs", False))
    rs_level = _get(args, "rs_level", tis_level)
    veto = _get(args, "rs_veto_threshold", None)
    metrics: dict[str, list] = {}
    weights, masks = [], []
    for t, r, m in zip(train_log_probs, rollout_log_probs, loss_masks):
        m = m.float()
        d = (t - r).float()
        # perplexity-style mismatch diagnostics: mean log-ratio and |1 - ratio|
        _mean_metric(metrics, "mismatch_log_ratio", d, m)
        _mean_metric(metrics, "mismatch_abs_ratio_minus_1", (d.exp() - 1).abs(), m)
        mask = m.clone()
        w = torch.ones_like(d)
        if use_tis:
            w = _level(d, m, tis_level).clamp(-SAFETY, SAFETY).exp()
            _mean_metric(metrics, "tis_weight_before_bound", w, m)
            if tis_mode == "truncate":
                _mean_metric(metrics, "tis_truncate_fraction", (w > U), m)
                w = w.clamp(max=U) * m
            elif tis_mode == "clip":
                _mean_metric(metrics, "tis_clip_fraction_low", (w < L), m)
                _mean_metric(metrics, "tis_clip_fraction_high", (w > U), m)
                w = w.clamp(L, U) * m
            elif tis_mode == "mask":
                _mean_metric(metrics, "tis_mask_fraction_low", (w < L), m)
                _mean_metric(metrics, "tis_mask_fraction_high", (w > U), m)
                mask = mask * ((w >= L) & (w <= U)).float()
                w = w * m
            else:
                raise ValueError(f"unknown tis_mode {tis_mode}")
        if use_rs:
            rw = _level(d, m, rs_level).clamp(-SAFETY, SAFETY).exp()
            _mean_metric(metrics, "rs_mask_fraction_low", (rw < rs_L), m)
            _mean_metric(metrics, "rs_mask_fraction_high", (rw > rs_U), m)
            mask = mask * ((rw >= rs_L) & (rw <= rs_U)).float()
            if veto is not None:
                bad = (d < math.log(veto)) & m.bool()
                _mean_metric(metrics, "rs_catastrophic_token_fraction", bad, m)
                if bool(bad.any()):
                    mask = torch.zeros_like(mask)
        weights.append(w.detach())
        masks.append(mask.detach())
    if use_tis and _get(args, "tis_batch_normalize", False) and weights:
        if tis_level == "token":
            tot = sum((w * m.float()).sum() for w, m in zip(weights, loss_masks))
            mean = tot / max(sum(float(m.float().sum()) for m in loss_masks), 1.0)
        else:
            means = [(w * m.float()).sum() / m.float().sum().clamp_min(1) for w, m in zip(weights, loss_masks)]
            mean = sum(means) / len(means)
        if float(mean) > 1e-8:
            weights = [w / mean for w in weights]
        metrics.setdefault("batch_norm_factor", []).append(torch.as_tensor(float(mean)))
    flat_w = torch.cat(weights) if weights else torch.ones(0)
    out = {k: float(torch.stack([v.float().reshape(()) for v in vs]).mean()) for k, vs in metrics.items()}
    return pg_loss * flat_w.to(pg_loss.device), masks, out


def mismatch_metrics(train_log_probs, rollout_log_probs, loss_masks) -> dict[str, float]:
    """--get-mismatch-metrics: train / rollout log-prob mismatch statistics without changing the
    loss (mean |t - r|, mean log-ratio, mean |1 - exp(t - r)|, per-sample max |t - r|)."""
    ds, ms, maxes = [], [], []
    for t, r, m in zip(train_log_probs, rollout_log_probs, loss_masks):
        t = torch.as_tensor(t, dtype=torch.float32)
        r = torch.as_tensor(r, dtype=torch.float32)
        m = torch.as_tensor(m if m is not None else [1] * len(t), dtype=torch.float32)
        d = t - r
        ds.append(d)
        ms.append(m)
        maxes.append(float((d.abs() * m).max()) if len(d) else 0.0)
    if not ds:
        return {}
    d, m = torch.cat(ds), torch.cat(ms)
    n = m.sum().clamp_min(1)
    return {"train/mismatch_abs_logprob_diff": float((d.abs() * m).sum() / n),
            "train/mismatch_log_ratio": float((d * m).sum() / n),
            "train/mismatch_abs_ratio_minus_1": float(((d.exp() - 1).abs() * m).sum() / n),
            "train/mismatch_max_abs_logprob_diff": max(maxes)}
