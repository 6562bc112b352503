"""Evaluation metrics: pass@k over groups of samples of one prompt (--log-passrate).

pass@k of a prompt with n samples of which c are correct is the probability that at least one
of k samples drawn without replacement is correct: 1 - C(n - c, k) / C(n, k) (the unbiased
estimator of Chen et al., 2021, "Evaluating Large Language Models Trained on Code"), computed
here as 1 - prod_{i=n-c+1}^{n} (1 - k / i). It is averaged over prompts for k = 1, 2, 4, ...
up to the group size. A reward > 0 counts as correct.

Reference role: miles/utils/metric_utils.py compute_pass_rate (:11-54).
"""
from __future__ import annotations

import numpy as np


def pass_at_k(n: int, c: int, k: int) -> float:
    if n - c < k:
        return 1.0
    i = np.arange(n - c + 1, n + 1, dtype=np.float64)
    return float(1.0 - np.prod(1.0 - k / i))


def compute_pass_rate(flat_rewards: list[float], group_size: int) -> dict[str, float]:
    if group_size <= 0 or not flat_rewards or len(flat_rewards) % group_size:
        return {}
    r = np.asarray(flat_rewards, dtype=np.float64).reshape(-1, group_size)
    correct = (r > 0).sum(1)
    out = {}
    k = 1
    while k <= group_size:
        out[f"pass@{k}"] = float(np.mean([pass_at_k(group_size, int(c), k) for c in correct]))
        k *= 2
    return out
