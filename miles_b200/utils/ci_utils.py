"""CI checks of a training run: per-parameter model hashes saved next to a checkpoint and
compared after loading it (--ci-save-model-hash / --ci-check-model-hash), and the gradient
norm of every optimizer step saved or compared against a saved run (--ci-save-grad-norm /
--ci-load-grad-norm, path templates with {role}, {rollout_id}, {step_id}).

Reference: miles/backends/megatron_utils/ci_utils.py (model hashes, :60-100),
miles/backends/training_utils/ci_utils.py (grad norms, :30-60). The hash here is SHA-256 of
each parameter's raw bytes (this rank's shard), keyed by the parameter name.
"""
from __future__ import annotations

import hashlib
import json
import math
import os

import torch


def model_hashes(model) -> dict[str, str]:
    out = {}
    for name, p in sorted(model.params.items()):
        t = p.detach().contiguous().cpu()
        out[name] = hashlib.sha256(t.view(torch.uint8).numpy().tobytes()).hexdigest()
    return out


def _hash_path(base: str, iteration: int, rank: int) -> str:
    d = base if os.path.basename(base.rstrip("/")).startswith("iter_") else os.path.join(
        base, f"iter_{int(iteration):07d}")
    return os.path.join(d, f"model_hash_rank{rank}.json")


def save_model_hashes(args, model, iteration: int, rank: int = 0) -> str | None:
    if not (args.ci_test and args.ci_save_model_hash and args.save):
        return None
    path = _hash_path(args.save, iteration, rank)
    os.makedirs(os.path.dirname(path), exist_ok=True)
    with open(path, "w") as f:
        json.dump(model_hashes(model), f, indent=1, sort_keys=True)
    return path


def check_model_hashes(args, model, iteration: int, rank: int = 0) -> None:
    if not (args.ci_test and args.ci_check_model_hash and args.load):
        return
    path = _hash_path(args.load, iteration, rank)
    if not os.path.isfile(path):
        raise AssertionError(f"[CI hash] hash file missing: {path}")
    with open(path) as f:
        expected = json.load(f)
    actual = model_hashes(model)
    bad = sorted(k for k in expected.keys() | actual.keys() if expected.get(k) != actual.get(k))
    if bad:
        raise AssertionError(f"[CI hash] model hash mismatch after load: {bad[:5]}")


def check_grad_norm(args, grad_norm: float, rollout_id: int, step_id: int, role: str = "actor",
                    rank: int = 0) -> None:
    if rank != 0:
        return
    if getattr(args, "ci_save_grad_norm", None):
        path = args.ci_save_grad_norm.format(role=role, rollout_id=rollout_id, step_id=step_id)
        os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
        torch.save(float(grad_norm), path)
    elif getattr(args, "ci_load_grad_norm", None):
        path = args.ci_load_grad_norm.format(role=role, rollout_id=rollout_id, step_id=step_id)
        expected = float(torch.load(path, weights_only=False))
        if not math.isclose(grad_norm, expected, rel_tol=0.03, abs_tol=0.03):
            raise AssertionError(f"grad norm mismatch: {grad_norm} != {expected}")
