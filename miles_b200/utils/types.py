"""Trajectory record and batch types.

Reference: miles/utils/types.py:9-277 (Sample with status, loss_mask, rollout_log_probs,
rollout_routed_experts, weight_versions; ParamInfo; RolloutBatch). Field names are kept so
user rollout / reward functions written against the reference keep working.
"""
from __future__ import annotations

import enum
from dataclasses import asdict, dataclass, field
from typing import Any

import numpy as np


@dataclass
class Sample:
    class Status(enum.Enum):
        PENDING = "pending"
        COMPLETED = "completed"
        TRUNCATED = "truncated"
        ABORTED = "aborted"
        FAILED = "failed"

    group_index: int | None = None
    index: int | None = None
    prompt: str | list = ""
    tokens: list[int] = field(default_factory=list)
    multimodal_inputs: Any = None
    response: str = ""
    response_length: int = 0
    label: Any = None
    reward: float | dict | None = None
    loss_mask: list[int] | None = None
    weight_versions: list[str] = field(default_factory=list)
    rollout_log_probs: list[float] | None = None
    rollout_routed_experts: np.ndarray | None = None
    remove_sample: bool = False
    status: "Sample.Status" = Status.PENDING
    metadata: dict = field(default_factory=dict)
    train_metadata: dict | None = None
    non_generation_time: float = 0.0
    spec_info: dict = field(default_factory=dict)
    prefix_cache_info: dict = field(default_factory=dict)

    @property
    def prompt_length(self) -> int:
        return len(self.tokens) - self.response_length

    def effective_response_length(self) -> int:
        return sum(self.loss_mask) if self.loss_mask is not None else self.response_length

    def update_from_meta_info(self, finish_reason: str, weight_version: str | int | None = None):
        """Map an engine finish reason onto the sample status (reference types.py:220-241)."""
        if weight_version is not None:
            self.weight_versions.append(str(weight_version))
        if finish_reason == "length":
            self.status = Sample.Status.TRUNCATED
        elif finish_reason == "abort":
            self.status = Sample.Status.ABORTED
        elif finish_reason == "stop":
            self.status = Sample.Status.COMPLETED
        else:
            self.status = Sample.Status.FAILED

    def reset_for_retry(self):
        """Drop a partial response (aborted groups recycled into the buffer)."""
        if self.response_length:
            self.tokens = self.tokens[: len(self.tokens) - self.response_length]
        self.response = ""
        self.response_length = 0
        self.loss_mask = None
        self.rollout_log_probs = None
        self.rollout_routed_experts = None
        self.reward = None
        self.status = Sample.Status.PENDING

    def to_dict(self) -> dict:
        d = asdict(self)
        d["status"] = self.status.value
        if isinstance(self.rollout_routed_experts, np.ndarray):
            d["rollout_routed_experts"] = self.rollout_routed_experts.tolist()
        return d

    @staticmethod
    def from_dict(d: dict) -> "Sample":
        d = dict(d)
        d["status"] = Sample.Status(d.get("status", "pending"))
        rre = d.get("rollout_routed_experts")
        if rre is not None:
            d["rollout_routed_experts"] = np.asarray(rre, dtype=np.int32)
        return Sample(**d)

    def get_reward_value(self, args) -> float:
        key = getattr(args, "reward_key", None)
        r = self.reward
        return float(r[key] if (key and isinstance(r, dict)) else r)


@dataclass
class ParamInfo:
    """Metadata of one parameter for refit planning (reference types.py:244)."""
    name: str
    dtype: str
    shape: tuple
    attrs: dict = field(default_factory=dict)
    size: int = 0
    src_rank: int = 0


RolloutBatch = dict  # reference types.py:257: dict[str, list] of per-sample training fields
