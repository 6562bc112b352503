"""Device / host memory helpers: free cached blocks, report usage, host RSS.

Reference: miles/utils/memory_utils.py:10-44 (clear_memory, print_memory, available memory),
tools/cpu_memory_profiler.py.
"""
from __future__ import annotations

import gc
import os

import torch


def clear_memory():
    gc.collect()
    if torch.cuda.is_available():
        torch.cuda.synchronize()
        torch.cuda.empty_cache()


def available_memory(device=None) -> dict:
    out = {}
    if torch.cuda.is_available():
        free, total = torch.cuda.mem_get_info(device)
        out.update(gpu_free_gb=free / 2**30, gpu_total_gb=total / 2**30,
                   gpu_allocated_gb=torch.cuda.memory_allocated(device) / 2**30,
                   gpu_reserved_gb=torch.cuda.memory_reserved(device) / 2**30,
                   gpu_peak_allocated_gb=torch.cuda.max_memory_allocated(device) / 2**30)
    try:
        import psutil

        p = psutil.Process(os.getpid())
        out["host_rss_gb"] = p.memory_info().rss / 2**30
        out["host_available_gb"] = psutil.virtual_memory().available / 2**30
    except Exception:  # noqa: BLE001
        pass
    return out


def print_memory(msg: str = "", rank: int = 0, only_rank0: bool = True) -> dict:
    m = available_memory()
    if not only_rank0 or rank == 0:
        print(f"[memory] {msg} " + " ".join(f"{k}={v:.2f}" for k, v in m.items()), flush=True)
    return m
