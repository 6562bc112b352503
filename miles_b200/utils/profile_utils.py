"""Per-rank profiling: a torch.profiler window over chosen steps and CUDA memory snapshots.

    --use-pytorch-profiler --profile-target train_overall --profile-step-start 10 \
        --profile-step-end 12            -> <tensorboard dir>/rank<r>/*.pt.trace.json
    --record-memory-history [--memory-snapshot-dir d --memory-snapshot-num-steps n]
                                         -> d/memory_snapshot_rank<r>_step<k>.pickle

Reference: miles/utils/profile_utils.py:13-147 (TrainProfiler: profiler schedule, memory
profiler backends).
"""
from __future__ import annotations

import os

import torch


class TrainProfiler:
    def __init__(self, args, rank: int = 0):
        self.args = args
        self.rank = rank
        self.prof = None
        self.step_id = 0
        out = getattr(args, "tensorboard_dir", None) or "profiles_out"
        self.trace_dir = os.path.join(out, f"rank{rank}")
        if getattr(args, "record_memory_history", False) and torch.cuda.is_available():
            torch.cuda.memory._record_memory_history(max_entries=1_000_000)

    def _active(self, target: str) -> bool:
        a = self.args
        return (getattr(a, "use_pytorch_profiler", False) and target in a.profile_target
                and a.profile_step_start <= self.step_id < a.profile_step_end)

    def start(self, target: str = "train_overall"):
        if self._active(target) and self.prof is None:
            acts = [torch.profiler.ProfilerActivity.CPU]
            if torch.cuda.is_available():
                acts.append(torch.profiler.ProfilerActivity.CUDA)
            os.makedirs(self.trace_dir, exist_ok=True)
            self.prof = torch.profiler.profile(
                activities=acts, record_shapes=True, with_stack=False,
                on_trace_ready=torch.profiler.tensorboard_trace_handler(self.trace_dir))
            self.prof.__enter__()

    def stop(self, target: str = "train_overall"):
        if self.prof is not None and (not getattr(self.args, "use_pytorch_profiler", False)
                                      or self.step_id + 1 >= self.args.profile_step_end):
            self.prof.__exit__(None, None, None)
            self.prof = None

    def step(self):
        if self.prof is not None:
            self.prof.step()
        a = self.args
        n = getattr(a, "memory_snapshot_num_steps", None)
        if getattr(a, "record_memory_history", False) and torch.cuda.is_available() and (
                n is None or self.step_id < n):
            dump_memory_snapshot(a.memory_snapshot_dir, self.rank, self.step_id)
        self.step_id += 1


def dump_memory_snapshot(directory: str, rank: int, step: int) -> str:
    os.makedirs(directory, exist_ok=True)
    path = os.path.join(directory, f"memory_snapshot_rank{rank}_step{step}.pickle")
    torch.cuda.memory._dump_snapshot(path)
    return path
