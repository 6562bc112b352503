"""Environment report: library versions, git revision, GPUs and driver, per process.

    --env-report  ->  printed by rank 0 at start-up (and returned as a dict)

Reference: miles/utils/env_report.py:13-179 (pip / git info per node).
"""
from __future__ import annotations

import os
import platform
import subprocess
import sys


def _git(root: str) -> dict:
    def run(*cmd):
        try:
            return subprocess.run(["git", "-C", root, *cmd], capture_output=True, text=True,
                                  timeout=10).stdout.strip()
        except Exception:  # noqa: BLE001
            return ""
    return {"commit": run("rev-parse", "HEAD"), "dirty": bool(run("status", "--porcelain"))}


def collect(root: str | None = None) -> dict:
    import torch

    root = root or os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    rep = {
        "python": sys.version.split()[0],
        "platform": platform.platform(),
        "host": platform.node(),
        "torch": torch.__version__,
        "cuda_runtime": torch.version.cuda,
        "nccl": ".".join(map(str, torch.cuda.nccl.version())) if torch.cuda.is_available() else None,
        "git": _git(root),
        "gpus": [],
    }
    if torch.cuda.is_available():
        for i in range(torch.cuda.device_count()):
            p = torch.cuda.get_device_properties(i)
            rep["gpus"].append({"name": p.name, "sm": f"{p.major}.{p.minor}",
                                "mem_gb": round(p.total_memory / 2**30, 1),
                                "sms": p.multi_processor_count})
        try:
            import pynvml

            pynvml.nvmlInit()
            rep["driver"] = pynvml.nvmlSystemGetDriverVersion()
        except Exception:  # noqa: BLE001
            pass
    try:
        import importlib.metadata as md

        rep["packages"] = {d.metadata["Name"]: d.version for d in md.distributions()
                           if d.metadata["Name"] in ("numpy", "transformers", "safetensors",
                                                     "fastapi", "uvicorn", "triton")}
    except Exception:  # noqa: BLE001
        pass
    try:
        from miles_b200 import _C  # noqa: F401

        rep["native_extension"] = True
    except Exception:  # noqa: BLE001
        rep["native_extension"] = False
    return rep


def report(rank: int = 0) -> dict:
    rep = collect()
    if rank == 0:
        import json

        print("[env-report] " + json.dumps(rep, default=str), flush=True)
    return rep
