"""Prompt datasets (jsonl / parquet), chat templating, data sources with resumable state, and
the partial-rollout buffer.

Reference: miles/utils/data.py:25-256 (Dataset, long-prompt filter), miles/rollout/data_source.py
(DataSource :17, RolloutDataSourceWithBuffer :159-219, save/load :119-156).
"""
from __future__ import annotations

import copy
import json
import os
import random
from typing import Callable

import torch

from miles_b200.utils.misc import load_function
from miles_b200.utils.types import Sample


def read_records(path: str) -> list[dict]:
    if path.endswith(".jsonl") or path.endswith(".json"):
        with open(path) as f:
            if path.endswith(".json"):
                data = json.load(f)
                return data if isinstance(data, list) else [data]
            return [json.loads(l) for l in f if l.strip()]
    if path.endswith(".parquet"):
        import pyarrow.parquet as pq

        return pq.read_table(path).to_pylist()
    raise ValueError(f"unsupported dataset format: {path}")


class Dataset:
    """Rows -> prompt Samples. `tokenizer` may be None (prompts given as token id lists)."""

    def __init__(self, path: str, tokenizer=None, max_length: int | None = None,
                 prompt_key: str = "input", label_key: str | None = None,
                 metadata_key: str = "metadata", tool_key: str | None = None,
                 multimodal_keys: dict | None = None, apply_chat_template: bool = False,
                 apply_chat_template_kwargs: dict | None = None, seed: int = 42):
        self.origin_samples = []
        for i, row in enumerate(read_records(path)):
            prompt = row.get(prompt_key)
            if apply_chat_template and tokenizer is not None and isinstance(prompt, list):
                tools = row.get(tool_key) if tool_key else None
                prompt = tokenizer.apply_chat_template(prompt, tools=tools, tokenize=False,
                                                       add_generation_prompt=True,
                                                       **(apply_chat_template_kwargs or {}))
            md = row.get(metadata_key) or {}
            if isinstance(md, str):
                try:
                    md = json.loads(md)
                except json.JSONDecodeError:
                    md = {"raw": md}
            s = Sample(index=i, prompt=prompt, label=row.get(label_key) if label_key else None,
                       metadata=md)
            if multimodal_keys:
                s.multimodal_inputs = {k: row.get(v) for k, v in multimodal_keys.items()}
            if max_length is not None and tokenizer is not None and isinstance(prompt, str):
                if len(tokenizer(prompt, add_special_tokens=False)["input_ids"]) > max_length:
                    continue
            elif max_length is not None and isinstance(prompt, list) and prompt and isinstance(prompt[0], int):
                if len(prompt) > max_length:
                    continue
            self.origin_samples.append(s)
        self.samples = list(self.origin_samples)
        self.seed = seed

    def shuffle(self, epoch_id: int):
        rng = random.Random(self.seed + epoch_id)
        self.samples = list(self.origin_samples)
        rng.shuffle(self.samples)

    def __len__(self):
        return len(self.samples)

    def __getitem__(self, i):
        return self.samples[i]


class DataSource:
    """Interface: produce groups of samples and persist / restore its position."""

    def get_samples(self, num_samples: int) -> list[list[Sample]]:
        raise NotImplementedError

    def add_samples(self, samples: list[list[Sample]]):
        raise NotImplementedError

    def save(self, rollout_id: int):
        pass

    def load(self, rollout_id: int | None = None):
        pass


class RolloutDataSource(DataSource):
    """Global dataset with per-epoch shuffling and resumable (epoch, offset) state. Each prompt
    becomes a group of `n_samples_per_prompt` copies."""

    def __init__(self, args, tokenizer=None):
        self.args = args
        self.epoch_id = 0
        self.sample_offset = 0
        self.sample_group_index = 0
        self.sample_index = 0
        self.dataset = None
        if getattr(args, "prompt_data", None) and not getattr(args, "disable_rollout_global_dataset", False):
            mm = getattr(args, "multimodal_keys", None)
            self.dataset = Dataset(args.prompt_data, tokenizer,
                                   max_length=getattr(args, "rollout_max_prompt_len", None),
                                   prompt_key=args.input_key, label_key=args.label_key,
                                   metadata_key=args.metadata_key, tool_key=args.tool_key,
                                   multimodal_keys=json.loads(mm) if isinstance(mm, str) else mm,
                                   apply_chat_template=args.apply_chat_template,
                                   apply_chat_template_kwargs=json.loads(args.apply_chat_template_kwargs)
                                   if isinstance(args.apply_chat_template_kwargs, str) else args.apply_chat_template_kwargs,
                                   seed=args.rollout_seed)
            if args.rollout_shuffle:
                self.dataset.shuffle(self.epoch_id)

    def get_samples(self, num_samples: int) -> list[list[Sample]]:
        n = self.args.n_samples_per_prompt
        groups: list[list[Sample]] = []
        if self.dataset is None:
            for _ in range(num_samples):
                g = []
                for _ in range(n):
                    g.append(Sample(group_index=self.sample_group_index, index=self.sample_index))
                    self.sample_index += 1
                groups.append(g)
                self.sample_group_index += 1
            return groups
        while len(groups) < num_samples:
            if self.sample_offset >= len(self.dataset):
                self.epoch_id += 1
                self.sample_offset = 0
                if self.args.rollout_shuffle:
                    self.dataset.shuffle(self.epoch_id)
            proto = self.dataset[self.sample_offset]
            self.sample_offset += 1
            g = []
            for _ in range(n):
                s = copy.deepcopy(proto)
                s.group_index = self.sample_group_index
                s.index = self.sample_index
                self.sample_index += 1
                g.append(s)
            self.sample_group_index += 1
            groups.append(g)
        return groups

    def add_samples(self, samples):
        raise RuntimeError("the global dataset source has no buffer; use RolloutDataSourceWithBuffer")

    def state_dict(self) -> dict:
        return {"epoch_id": self.epoch_id, "sample_offset": self.sample_offset,
                "sample_group_index": self.sample_group_index, "sample_index": self.sample_index}

    def load_state_dict(self, d: dict):
        self.epoch_id = d["epoch_id"]
        self.sample_offset = d["sample_offset"]
        self.sample_group_index = d["sample_group_index"]
        self.sample_index = d["sample_index"]
        if self.dataset is not None and self.args.rollout_shuffle:
            self.dataset.shuffle(self.epoch_id)

    def _path(self, rollout_id):
        return os.path.join(self.args.save, "rollout", f"global_dataset_state_dict_{rollout_id}.pt")

    def save(self, rollout_id: int):
        if not getattr(self.args, "save", None):
            return
        os.makedirs(os.path.join(self.args.save, "rollout"), exist_ok=True)
        torch.save(self.state_dict(), self._path(rollout_id))

    def load(self, rollout_id: int | None = None):
        load = getattr(self.args, "load", None)
        if not load or rollout_id is None:
            return
        p = os.path.join(load, "rollout", f"global_dataset_state_dict_{rollout_id}.pt")
        if os.path.exists(p):
            self.load_state_dict(torch.load(p))


def pop_first(args, rollout_id, buffer: list[list[Sample]], num_samples: int):
    """Default buffer filter: take the oldest groups first."""
    n = min(num_samples, len(buffer))
    out = buffer[:n]
    del buffer[:n]
    return out


class RolloutDataSourceWithBuffer(RolloutDataSource):
    """Adds a buffer of partial / aborted groups that is drained before fresh prompts."""

    def __init__(self, args, tokenizer=None):
        super().__init__(args, tokenizer)
        self.buffer: list[list[Sample]] = []
        path = getattr(args, "buffer_filter_path", None)
        self.buffer_filter: Callable = load_function(path) if path else pop_first

    def get_samples(self, num_samples: int) -> list[list[Sample]]:
        out = self.buffer_filter(self.args, None, self.buffer, num_samples) if self.buffer else []
        if len(out) < num_samples:
            out += super().get_samples(num_samples - len(out))
        return out

    def add_samples(self, samples: list[list[Sample]]):
        for g in samples:
            assert isinstance(g, list) and len(g) == self.args.n_samples_per_prompt
            self.buffer.append(g)

    def get_buffer_length(self) -> int:
        return len(self.buffer)
