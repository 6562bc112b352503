"""CI assertion on an eval metric (reference: miles/utils/metric_checker.py:6-28)."""
from __future__ import annotations


def check_metric(args, history: list[dict]) -> None:
    key, thr = args.ci_metric_checker_key, args.ci_metric_checker_threshold
    vals = [h[key] for h in history if key in h]
    if not vals:
        raise AssertionError(f"metric {key} was never logged")
    if vals[-1] < thr:
        raise AssertionError(f"{key} = {vals[-1]} < threshold {thr}")
