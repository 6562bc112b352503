"""Rollout manager: data source + rollout function + reward post-processing + conversion of
samples into training data, per data-parallel rank.

Where the reference runs one CPU Ray actor that fans HTTP requests out to every engine and then
splits the batch across DP ranks, here every GPU process owns an engine and a rollout manager
over its own shard of the prompt stream (prompt groups never straddle ranks, so GRPO group
normalisation stays local). The conversion and reward post-processing follow the reference.

Reference: miles/ray/rollout.py (RolloutManager :334-793: generate :445-455, reward
post-process :640-665, convert_samples_to_train_data :667-738, trim to global batch :573-619,
debug dump/load :545-559,621-638, metrics :1197-1305).
"""
from __future__ import annotations

import os
import pickle
import time

import numpy as np
import torch

from miles_b200.rollout.default import GenerateState, RolloutFnTrainOutput
from miles_b200.utils.misc import load_function
from miles_b200.utils.types import Sample


class ShardedDataSource:
    """Wrap a data source so rank r of W only sees groups r, r+W, r+2W, ..."""

    def __init__(self, inner, rank: int, world: int):
        self.inner, self.rank, self.world = inner, rank, world

    def get_samples(self, n: int):
        groups = self.inner.get_samples(n * self.world)
        return groups[self.rank::self.world]

    def add_samples(self, samples):
        if hasattr(self.inner, "add_samples"):
            self.inner.add_samples(samples)

    def save(self, rid):
        if self.rank == 0:
            self.inner.save(rid)

    def load(self, rid=None):
        self.inner.load(rid)


class RolloutManager:
    def __init__(self, args, data_source, client=None, tokenizer=None, rank: int = 0, world: int = 1):
        self.args = args
        self.rank, self.world = rank, world
        self.data_source = ShardedDataSource(data_source, rank, world) if world > 1 else data_source
        self.state = GenerateState(args, client=client, tokenizer=tokenizer)
        GenerateState.set(self.state)
        from miles_b200.rollout.base_types import (RolloutFnConstructorInput,
                                                   enable_experimental_rollout_refactor,
                                                   load_rollout_callable)

        if enable_experimental_rollout_refactor():
            # class-based rollout functions, constructed once with this rank's arguments
            ctor = RolloutFnConstructorInput(self._local_args(), self.data_source)
            load = lambda path: load_rollout_callable(path, ctor)  # noqa: E731
        else:
            load = load_function
        self.rollout_fn = load(args.rollout_function_path)
        self.eval_fn = load(args.eval_function_path) if args.eval_function_path else self.rollout_fn
        self.custom_convert = (load_function(args.custom_convert_samples_to_train_data_path)
                               if args.custom_convert_samples_to_train_data_path else None)
        self.custom_reward_post = (load_function(args.custom_reward_post_process_path)
                                   if args.custom_reward_post_process_path else None)
        self.last_metrics: dict = {}
        # --custom-rollout-log-function-path / --custom-eval-rollout-log-function-path: called
        # with the rollout's samples (eval: its per-dataset data); returning True skips the
        # default metrics (reference miles/ray/rollout.py:1145-1186)
        self.custom_rollout_log = (load_function(args.custom_rollout_log_function_path)
                                   if args.custom_rollout_log_function_path else None)
        self.custom_eval_log = (load_function(args.custom_eval_rollout_log_function_path)
                                if args.custom_eval_rollout_log_function_path else None)

    # ------------------------------------------------------------------ generation
    def _local_args(self):
        """Per-rank copy of the args with the batch split across data-parallel ranks."""
        a = self.args
        if self.world == 1:
            return a
        import copy

        la = copy.copy(a)
        la.rollout_batch_size = max(1, a.rollout_batch_size // self.world)
        la.over_sampling_batch_size = max(la.rollout_batch_size, a.over_sampling_batch_size // self.world)
        return la

    def generate(self, rollout_id: int) -> dict:
        t0 = time.perf_counter()
        if self.args.load_debug_rollout_data:
            with open(self.args.load_debug_rollout_data.format(rollout_id=rollout_id), "rb") as f:
                groups = pickle.load(f)["samples"]
            frac = getattr(self.args, "load_debug_rollout_data_subsample", None)
            if frac is not None and 0 < frac < 1:  # keep a deterministic fraction of the groups
                keep = max(1, int(round(len(groups) * frac)))
                groups = groups[:keep]
            metrics = {}
        else:
            la = self._local_args()
            self.state.args = la
            out = self.rollout_fn(la, rollout_id, self.data_source, evaluation=False)
            if isinstance(out, RolloutFnTrainOutput):
                groups, metrics = out.samples, out.metrics
            else:
                groups, metrics = out, {}
        if self.args.save_debug_rollout_data:
            path = self.args.save_debug_rollout_data.format(rollout_id=rollout_id)
            os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
            with open(path, "wb") as f:
                pickle.dump({"rollout_id": rollout_id, "samples": groups}, f)
        groups = self._trim(groups)
        samples = [s for g in groups for s in g]
        dt = time.perf_counter() - t0
        if self.custom_rollout_log is not None and self.custom_rollout_log(rollout_id, self.args, samples,
                                                                          metrics, dt):
            pass  # the custom logger replaced the default rollout metrics
        else:
            metrics.update(self.rollout_metrics(samples, dt))
        data = self.convert_samples_to_train_data(groups)
        self.last_metrics = metrics
        data["metrics"] = metrics
        return data

    def _trim(self, groups):
        """Drop trailing groups so this rank's sample count is a multiple of its share of
        --global-batch-size (dynamic filtering can return more); --disable-rollout-trim-samples
        keeps them all."""
        a = self.args
        if getattr(a, "disable_rollout_trim_samples", False) or not groups or not a.global_batch_size:
            return groups
        per_rank = max(1, a.global_batch_size // self.world)
        n = sum(len(g) for g in groups)
        if n <= per_rank or n % per_rank == 0:
            return groups
        target = n // per_rank * per_rank
        out, c = [], 0
        for g in groups:
            if c + len(g) > target:
                break
            out.append(g)
            c += len(g)
        return out or groups

    def eval(self, rollout_id: int) -> dict:
        out = self.eval_fn(self.args, rollout_id, self.data_source, evaluation=True)
        metrics = getattr(out, "metrics", {}) if not isinstance(out, dict) else out
        if self.custom_eval_log is not None:
            data = out if isinstance(out, dict) else getattr(out, "data", None)
            if self.custom_eval_log(rollout_id, self.args, data, metrics):
                return {}
        return metrics

    # ------------------------------------------------------------------ rewards / conversion
    def post_process_rewards(self, groups: list[list[Sample]]) -> tuple[list[float], list[float]]:
        """Raw rewards and the rewards used for advantages. For GRPO/GSPO (and RF++ baseline)
        rewards are normalised within each prompt group: minus the group mean and, unless
        --disable-grpo-std-normalization, divided by (group std + 1e-6)."""
        if self.custom_reward_post is not None:
            return self.custom_reward_post(self.args, groups)
        a = self.args
        raw = [s.get_reward_value(a) for g in groups for s in g]
        if a.advantage_estimator in ("grpo", "gspo", "reinforce_plus_plus_baseline") and not a.disable_rewards_normalization:
            out = []
            for g in groups:
                r = np.array([s.get_reward_value(a) for s in g], dtype=np.float64)
                r = r - r.mean()
                if a.advantage_estimator in ("grpo", "gspo") and not a.disable_grpo_std_normalization:
                    r = r / (r.std(ddof=1) + 1e-6) if len(r) > 1 else r
                out.extend(r.tolist())
            return raw, out
        return raw, list(raw)

    def convert_samples_to_train_data(self, groups: list[list[Sample]]) -> dict:
        if self.custom_convert is not None:
            return self.custom_convert(self.args, groups)
        raw, rewards = self.post_process_rewards(groups)
        samples = [s for g in groups for s in g]
        data = {
            "tokens": [s.tokens for s in samples],
            "response_lengths": [s.response_length for s in samples],
            "rewards": rewards,
            "raw_reward": raw,
            "truncated": [1 if s.status == Sample.Status.TRUNCATED else 0 for s in samples],
            "sample_indices": [s.index for s in samples],
            "loss_masks": [s.loss_mask if s.loss_mask is not None else [1] * s.response_length for s in samples],
        }
        if samples and samples[0].rollout_log_probs is not None:
            data["rollout_log_probs"] = [s.rollout_log_probs for s in samples]
        if samples and samples[0].rollout_routed_experts is not None:
            data["rollout_routed_experts"] = [s.rollout_routed_experts for s in samples]
        if samples and samples[0].weight_versions:
            data["weight_versions"] = [s.weight_versions for s in samples]
        if samples and samples[0].metadata.get("teacher_log_probs") is not None:
            data["teacher_log_probs"] = [s.metadata["teacher_log_probs"] for s in samples]
        return data

    # ------------------------------------------------------------------ metrics
    def rollout_metrics(self, samples: list[Sample], rollout_time: float) -> dict:
        if not samples:
            return {}
        lens = np.array([s.response_length for s in samples])
        resp_tokens = int(lens.sum())
        n_gpus = max(1, self.args.rollout_num_gpus // self.world) if self.world > 1 else max(1, self.args.rollout_num_gpus)
        m = {
            "rollout/response_len/mean": float(lens.mean()),
            "rollout/response_len/max": int(lens.max()),
            "rollout/response_len/min": int(lens.min()),
            "rollout/truncated_ratio": float(np.mean([s.status == Sample.Status.TRUNCATED for s in samples])),
            "perf/rollout_time": rollout_time,
            "perf/tokens_per_gpu_per_sec": resp_tokens / rollout_time / n_gpus if rollout_time > 0 else 0.0,
            "perf/longest_sample_tokens_per_sec": int(lens.max()) / rollout_time if rollout_time > 0 else 0.0,
        }
        try:
            r = np.array([s.get_reward_value(self.args) for s in samples], dtype=np.float64)
            m["rollout/raw_reward"] = float(r.mean())
            if self.args.n_samples_per_prompt > 1 and len(r) % self.args.n_samples_per_prompt == 0:
                g = r.reshape(-1, self.args.n_samples_per_prompt)
                m["rollout/zero_std/count"] = int((g.std(1) == 0).sum())
        except Exception:
            pass
        a = self.args
        if getattr(a, "log_correct_samples", False):
            ok = [s for s in samples if (s.get_reward_value(a) or 0) > 0]
            m["rollout/correct_samples"] = len(ok)
            if ok:
                m["rollout/correct_response_len/mean"] = float(np.mean([s.response_length for s in ok]))
        if getattr(a, "log_multi_turn", False):
            turns = [s.metadata.get("num_turns", s.metadata.get("turn", 1)) for s in samples]
            m["rollout/multi_turn/turns_mean"] = float(np.mean(turns))
            m["rollout/multi_turn/turns_max"] = int(np.max(turns))
        cat_key = getattr(a, "log_reward_category", None)
        if cat_key:  # mean reward per value of sample.metadata[<key>] (e.g. the task / source)
            by: dict = {}
            for s in samples:
                by.setdefault(str(s.metadata.get(cat_key, "none")), []).append(s.get_reward_value(a))
            for k, v in by.items():
                m[f"rollout/reward_category/{k}"] = float(np.mean(v))
        wv = [s.weight_versions[-1] for s in samples if s.weight_versions]
        if wv:
            m["rollout/weight_version"] = max(int(v) for v in wv)
        return m
