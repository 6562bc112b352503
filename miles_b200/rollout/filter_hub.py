"""Dynamic-sampling filters and their drop metrics.

Reference: miles/rollout/filter_hub/ (check_reward_nonzero_std, no-aborted filter,
DynamicFilterOutput with a drop reason recorded per group).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from miles_b200.utils.types import Sample


@dataclass
class DynamicFilterOutput:
    keep: bool
    reason: str | None = None


def _reward(args, s: Sample) -> float:
    return s.get_reward_value(args)


def check_reward_nonzero_std(args, samples: list[Sample], **kwargs) -> DynamicFilterOutput:
    """Keep a group only if its rewards are not all equal (GRPO gives it zero advantage)."""
    r = np.array([_reward(args, s) for s in samples], dtype=np.float64)
    keep = bool(r.std() > 0.0)
    return DynamicFilterOutput(keep, None if keep else f"zero_std_{r.mean():.1f}")


def check_no_aborted(args, samples: list[Sample], **kwargs) -> DynamicFilterOutput:
    keep = all(s.status != Sample.Status.ABORTED for s in samples)
    return DynamicFilterOutput(keep, None if keep else "aborted")


def as_output(x) -> DynamicFilterOutput:
    """Filters may also return a bare bool."""
    return x if isinstance(x, DynamicFilterOutput) else DynamicFilterOutput(bool(x))


class DropMetrics:
    def __init__(self):
        self.counts: dict[str, int] = {}

    def add(self, reason: str | None):
        if reason:
            self.counts[reason] = self.counts.get(reason, 0) + 1

    def to_dict(self, prefix="rollout/dynamic_filter/drop_") -> dict:
        return {prefix + k: v for k, v in self.counts.items()}
