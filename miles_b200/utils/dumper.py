"""Tensor dumper for train / inference numerical comparisons.

Enabled with --dumper-enable (or MILES_B200_DUMPER=1). Code calls `dump(name, tensor)` at
points of interest (layer outputs, log-probs); with the dumper on, each tensor is written to
<dumper-dir>/<phase>/rank<r>/<step>_<name>.pt, where the phase is "train_fwd", "train_bwd" or
"inference" (set by the caller with `phase(...)`). `compare(dir_a, dir_b)` loads two dumps and
reports the max abs / rel difference per tensor name, which is how a train-vs-rollout
mismatch is localised.

Reference: miles/utils/dumper_utils.py:20-150 (SGLang dumper integration per phase).
"""
from __future__ import annotations

import os
from contextlib import contextmanager

import torch

_STATE = {"enabled": bool(os.environ.get("MILES_B200_DUMPER")), "dir": "/tmp/dumper",
          "phase": "inference", "step": 0, "rank": 0}


def configure(args=None, rank: int = 0):
    if args is not None:
        _STATE["enabled"] = bool(getattr(args, "dumper_enable", False)) or _STATE["enabled"]
        _STATE["dir"] = getattr(args, "dumper_dir", _STATE["dir"])
        # which phases dump: inference (rollout engine), fwd_only (log-prob passes), fwd_bwd
        # (training); none selected = all of them
        sel = {p for p, flag in (("inference", "dumper_inference"), ("fwd_only", "dumper_fwd_only"),
                                 ("fwd_bwd", "dumper_fwd_bwd")) if getattr(args, flag, False)}
        _STATE["phases"] = sel or None
    _STATE["rank"] = rank


def enabled() -> bool:
    return _STATE["enabled"]


@contextmanager
def phase(name: str, step: int | None = None):
    old = (_STATE["phase"], _STATE["step"])
    _STATE["phase"] = name
    if step is not None:
        _STATE["step"] = step
    try:
        yield
    finally:
        _STATE["phase"], _STATE["step"] = old


def dump(name: str, t: torch.Tensor):
    if not _STATE["enabled"]:
        return
    phases = _STATE.get("phases")
    if phases is not None and _STATE["phase"] not in phases:
        return
    d = os.path.join(_STATE["dir"], _STATE["phase"], f"rank{_STATE['rank']}")
    os.makedirs(d, exist_ok=True)
    torch.save(t.detach().float().cpu(), os.path.join(d, f"{_STATE['step']:06d}_{name}.pt"))


def compare(dir_a: str, dir_b: str) -> dict:
    out = {}
    for f in sorted(os.listdir(dir_a)):
        pb = os.path.join(dir_b, f)
        if not f.endswith(".pt") or not os.path.exists(pb):
            continue
        a, b = torch.load(os.path.join(dir_a, f)), torch.load(pb)
        if a.shape != b.shape:
            out[f] = {"shape_mismatch": (tuple(a.shape), tuple(b.shape))}
            continue
        d = (a - b).abs()
        out[f] = {"max_abs": float(d.max()) if d.numel() else 0.0,
                  "max_rel": float((d / (b.abs() + 1e-6)).max()) if d.numel() else 0.0,
                  "equal": bool(torch.equal(a, b))}
    return out
