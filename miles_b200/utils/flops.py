"""Analytic training FLOPs (perf/actor_train_tflops): 3 x forward FLOPs of the trained
sequences (forward + backward at twice the forward), where one sequence of length L costs
2 * active_params * L for the matmuls plus 4 * layers * q_heads * head_dim * L^2 / 2 for causal
attention. Activation recompute is not counted, as in the reference
(miles/utils/train_metric_utils.py:34-35, miles/utils/flops_utils.py)."""
from __future__ import annotations


def forward_flops(cfg, lengths) -> float:
    per_tok = 2.0 * cfg.active_params()
    attn = 4.0 * cfg.num_layers * cfg.num_heads * cfg.head_dim / 2.0
    return float(sum(per_tok * L + attn * L * L for L in lengths))


def train_tflops(cfg, lengths, seconds: float) -> float:
    return 3.0 * forward_flops(cfg, lengths) / max(seconds, 1e-9) / 1e12
