"""Class-based rollout functions (opt-in with MILES_EXPERIMENTAL_ROLLOUT_REFACTOR=1).

With the toggle on, `--rollout-function-path` / `--eval-function-path` may name a class: it is
constructed once with `RolloutFnConstructorInput(args, data_source)` and then called with a
`RolloutFnTrainInput(rollout_id)` or `RolloutFnEvalInput(rollout_id)`; the call may return a
coroutine (it is run to completion) and returns `RolloutFnTrainOutput` / `RolloutFnEvalOutput`
(or the legacy plain values). A plain function keeps the legacy call
fn(args, rollout_id, data_source, evaluation=...).

Reference: miles/utils/environ.py (the toggle), miles/rollout/base_types.py (input / output
types), miles/rollout/inference_rollout/compatibility.py (class or legacy function loading).
"""
from __future__ import annotations

import asyncio
import inspect
import os
from argparse import Namespace
from dataclasses import dataclass
from typing import Any

from miles_b200.rollout.default import RolloutFnTrainOutput
from miles_b200.utils.misc import load_function


def enable_experimental_rollout_refactor() -> bool:
    return bool(int(os.environ.get("MILES_EXPERIMENTAL_ROLLOUT_REFACTOR", "0")))


@dataclass(frozen=True)
class RolloutFnConstructorInput:
    args: Namespace
    data_source: Any


@dataclass(frozen=True)
class RolloutFnTrainInput:
    rollout_id: int

    @property
    def evaluation(self) -> bool:
        return False


@dataclass(frozen=True)
class RolloutFnEvalInput:
    rollout_id: int

    @property
    def evaluation(self) -> bool:
        return True


@dataclass
class RolloutFnEvalOutput:
    data: dict
    metrics: dict | None = None


def load_rollout_callable(path: str, ctor: RolloutFnConstructorInput):
    """A callable with the legacy signature (args, rollout_id, data_source, evaluation) for
    the class or function at `path`; eval outputs come back as their `data` dict."""
    fn = load_function(path)
    if not inspect.isclass(fn):
        return fn
    obj = fn(ctor)

    def call(args, rollout_id, data_source, evaluation=False):
        inp = (RolloutFnEvalInput if evaluation else RolloutFnTrainInput)(rollout_id)
        out = obj(inp)
        if inspect.iscoroutine(out):
            out = asyncio.run(out)
        if isinstance(out, RolloutFnEvalOutput):
            return out.data
        return out

    return call


__all__ = ["RolloutFnConstructorInput", "RolloutFnTrainInput", "RolloutFnEvalInput",
           "RolloutFnTrainOutput", "RolloutFnEvalOutput", "enable_experimental_rollout_refactor",
           "load_rollout_callable"]
