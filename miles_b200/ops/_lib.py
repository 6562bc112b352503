"""Loader for the in-tree sm_100a extension (miles_b200._C).

On a machine with a CUDA device the extension is mandatory: importing an op module there with
the extension missing raises immediately instead of falling back to eager PyTorch. On a CPU-only
machine ops fall back to their PyTorch reference implementations (used by the CPU test tier and
the gloo plumbing config).
"""
from __future__ import annotations

import torch

_C = None
_IMPORT_ERROR: Exception | None = None
try:
    from miles_b200 import _C as _C  # type: ignore[attr-defined,no-redef]
except Exception as e:  # pragma: no cover - depends on build state
    _IMPORT_ERROR = e


def native_available() -> bool:
    return _C is not None


class KernelLaunchError(RuntimeError):
    pass


class _Checked:
    """Proxy over the extension: every launcher returns a C status code (0 = ok); a non-zero
    code is raised here as KernelLaunchError naming the entry point."""

    def __init__(self, mod):
        self._mod = mod
        self._cache = {}

    def __getattr__(self, name):
        fn = self._cache.get(name)
        if fn is None:
            raw = getattr(self._mod, name)

            def fn(*args, _raw=raw, _name=name):
                global LAUNCHES
                LAUNCHES += 1
                rc = _raw(*args)
                if isinstance(rc, int) and rc != 0:
                    raise KernelLaunchError(f"{_name} failed with status {rc}")
                return rc

            self._cache[name] = fn
        return fn


_CHECKED = None
# Number of native launcher calls issued from Python (each issues >= 1 kernel). Work replayed
# from a captured CUDA graph is added by the engine (launches recorded at capture time).
LAUNCHES = 0


def launch_count() -> int:
    return LAUNCHES


def add_launches(n: int) -> None:
    global LAUNCHES
    LAUNCHES += n


def lib():
    """Return the (status-checked) native module; raise loudly when it is missing."""
    global _CHECKED
    if _C is None:
        raise RuntimeError(
            "miles_b200._C is not built (run `python setup.py build_ext --inplace`): "
            f"{_IMPORT_ERROR!r}"
        )
    if _CHECKED is None:
        _CHECKED = _Checked(_C)
    return _CHECKED


def use_native(t: torch.Tensor) -> bool:
    """Native kernels run for every CUDA tensor; CPU tensors use the PyTorch reference path."""
    if t.is_cuda:
        lib()  # fail loudly if the extension is missing
        return True
    return False


_ERR: dict[int, torch.Tensor] = {}


def err_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 error word written by kernels whose bounded waits time out."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _ERR.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _ERR[idx] = t
    return t


class DeviceKernelError(RuntimeError):
    pass


_ERR_NAMES = {1: "GEMM pipeline wait timed out", 2: "attention pipeline wait timed out",
              3: "peer flag wait timed out", 4: "expert-parallel receive buffer overflow"}


def check_device_error(device: torch.device | None = None, clear: bool = True) -> None:
    """Raise DeviceKernelError if any kernel on `device` reported a timed-out wait."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    t = err_word(device)
    code = int(t.item())
    if code:
        if clear:
            t.zero_()
        raise DeviceKernelError(f"device kernel error {code}: {_ERR_NAMES.get(code, 'unknown')}")


def peek_device_error(device: torch.device | None = None) -> int:
    """The device error word of `device` (0 = none) without clearing it or raising."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    return int(err_word(device).item())
