"""Small shared utilities: dotted-path plugin loading, singletons, periodic actions, timers.

Reference: miles/utils/misc.py (load_function :42, SingletonMeta, should_run_periodic_action
:175), miles/utils/timer.py (Timer / timer / inverse_timer :15-89).
"""
from __future__ import annotations

import contextlib
import functools
import importlib
import importlib.util
import os
import time
from collections import defaultdict


def load_function(path: str):
    """Import `pkg.module.attr` (or `/path/file.py:attr`) and return the attribute."""
    if path is None:
        return None
    if ":" in path and path.split(":")[0].endswith(".py"):
        file, attr = path.split(":", 1)
        spec = importlib.util.spec_from_file_location(os.path.basename(file)[:-3], file)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        return getattr(mod, attr)
    mod_name, _, attr = path.rpartition(".")
    mod = importlib.import_module(mod_name)
    return getattr(mod, attr)


class SingletonMeta(type):
    _instances: dict = {}

    def __call__(cls, *a, **k):
        if cls not in cls._instances:
            cls._instances[cls] = super().__call__(*a, **k)
        return cls._instances[cls]


def should_run_periodic_action(rollout_id: int, interval: int | None, num_rollout: int | None = None) -> bool:
    """True on every `interval`-th rollout (1-based) and on the last rollout."""
    if interval is None or interval <= 0:
        return False
    step = rollout_id + 1
    return step % interval == 0 or (num_rollout is not None and step == num_rollout)


class Timer(metaclass=SingletonMeta):
    """Named wall-clock timers accumulated per step; `log_dict()` returns `{name}_time`."""

    def __init__(self):
        self.start_time: dict[str, float] = {}
        self.acc: dict[str, float] = defaultdict(float)

    def start(self, name: str):
        self.start_time[name] = time.perf_counter()

    def end(self, name: str):
        t0 = self.start_time.pop(name, None)
        if t0 is not None:
            self.acc[name] += time.perf_counter() - t0

    def reset(self, name: str | None = None):
        if name is None:
            self.acc.clear()
        else:
            self.acc.pop(name, None)

    def log_dict(self) -> dict[str, float]:
        return {f"{k}_time": v for k, v in self.acc.items()}

    @contextlib.contextmanager
    def context(self, name: str):
        self.start(name)
        try:
            yield
        finally:
            self.end(name)


def timer(name_or_fn=None):
    """Decorator or context manager: `@timer`, `@timer("name")`, `with timer("name"):`."""
    if callable(name_or_fn):
        fn = name_or_fn

        @functools.wraps(fn)
        def wrapper(*a, **k):
            with Timer().context(fn.__name__):
                return fn(*a, **k)

        return wrapper
    name = name_or_fn

    class _Ctx:
        def __enter__(self):
            Timer().start(name)

        def __exit__(self, *exc):
            Timer().end(name)

        def __call__(self, fn):
            @functools.wraps(fn)
            def wrapper(*a, **k):
                with Timer().context(name or fn.__name__):
                    return fn(*a, **k)

            return wrapper

    return _Ctx()


@contextlib.contextmanager
def inverse_timer(name: str):
    """Time the region *outside* the context (e.g. `train_wait` while waiting on rollout)."""
    Timer().end(name)
    try:
        yield
    finally:
        Timer().start(name)
