"""Per-GPU training actor: turns one rollout's data into policy updates.

    train(rollout_id, data):
      old log-probs   (forward with the current = rollout weights; bitwise equal to the
                       engine's, so --use-rollout-logprobs skips it with no change in value)
      ref log-probs   (--use-kl-loss / --kl-coef: weights swapped in from a pinned host backup)
      advantages      (GRPO/GSPO/RF++/RF++-baseline/PPO/OPD)
      num_steps_per_rollout optimizer steps over the rollout's samples
      CI checks       (--ci-test: ppo_kl / clipfrac / kl_loss ~ 0 on-policy; log-prob equality)

Also provides the named weight backups (actor / ref / old_actor) used for model switching.

Reference: megatron_utils/actor.py (train_actor :367-466, switch_model :559-583,
TensorBackuper usage :136-156), utils/tensor_backper.py:10-115,
training_utils/ci_utils.py:12-24, training_utils/log_utils.py:171-200.
"""
from __future__ import annotations

import os
import time

import numpy as np
import torch

from miles_b200.trainer.actor import Actor
from miles_b200.trainer.advantages import compute_advantages, data_to_items


class TensorBackuper:
    """Pinned host copies of the flat parameter buffer under named tags."""

    def __init__(self, model, enabled: bool = True):
        self.model = model
        self.enabled = enabled
        self.backups: dict[str, torch.Tensor] = {}

    def backup(self, tag: str):
        if not self.enabled:
            return
        src = self.model.flat
        dst = self.backups.get(tag)
        if dst is None:
            dst = torch.empty(src.numel(), dtype=src.dtype, pin_memory=src.is_cuda)
            self.backups[tag] = dst
        dst.copy_(src, non_blocking=True)
        if src.is_cuda:
            torch.cuda.current_stream().synchronize()

    def restore(self, tag: str):
        self.model.flat.copy_(self.backups[tag], non_blocking=True)

    def hash(self, tag: str | None = None) -> int:
        t = self.backups[tag] if tag else self.model.flat
        return int(t.view(torch.int16).to(torch.int64).sum().item()) if t.numel() else 0


class TrainActor:
    def __init__(self, args, actor: Actor, dp_group=None, critic=None,
                 data_parallel_size: int | None = None):
        """dp_group reduces gradients (data- x context-parallel ranks); data_parallel_size is
        the number of distinct data shards (the loss normalisation counts samples over them)."""
        self.args = args
        self.actor = actor
        self.critic = critic  # PPO value model (miles_b200/trainer/critic.py) or None
        self.model = actor.model
        self.dp_group = dp_group
        self.data_world = data_parallel_size or (
            torch.distributed.get_world_size(dp_group) if dp_group is not None else 1)
        self.backuper = TensorBackuper(self.model, enabled=not args.disable_weights_backuper)
        self.need_ref = bool(args.use_kl_loss or args.kl_coef)
        self.metrics: dict = {}
        from miles_b200.utils.misc import load_function

        hook = lambda name: (load_function(getattr(args, name)) if getattr(args, name, None)  # noqa: E731
                             else None)
        # user hooks (reference megatron_utils/model.py:279-283, :354-358; actor.py:187-190)
        self._hook_before_lp = hook("custom_megatron_before_log_prob_hook_path")
        self._hook_before_step = hook("custom_megatron_before_train_step_hook_path")
        self._postprocess = hook("rollout_data_postprocess_path")

    def _rank(self) -> int:
        import torch.distributed as dist

        return dist.get_rank() if dist.is_initialized() else 0

    def init_ref(self):
        """Reference policy for the KL terms: the weights of --ref-load (torch_dist iteration
        --ref-ckpt-step, or an HF directory) when given, else the initial weights. With
        --keep-old-actor the initial weights also seed the old-actor / rollout-actor queue
        (reference megatron_utils/actor.py:151-156, :543-552)."""
        a = self.args
        if self.need_ref:
            ref_load = getattr(a, "ref_load", None)
            if ref_load:
                self.backuper.backup("actor")
                self._load_weights(ref_load, getattr(a, "ref_ckpt_step", None))
                self.backuper.backup("ref")
                self.backuper.restore("actor")
            else:
                self.backuper.backup("ref")
        if getattr(a, "keep_old_actor", False):
            self.backuper.backup("old_actor")
            self.backuper.backup("rollout_actor")

    def _load_weights(self, path: str, step: int | None):
        from miles_b200.checkpoint.torch_dist import is_torch_dist, load_checkpoint

        if is_torch_dist(path):
            load_checkpoint(path, self.model, None, load_optim=False, iteration=step)
        else:
            from miles_b200.checkpoint.hf import load_hf

            load_hf(self.model, path)

    def after_update(self, rollout_id: int):
        """Weight bookkeeping after the policy update of `rollout_id`: refresh the reference
        policy every --ref-update-interval rollouts, and advance the --keep-old-actor queue
        (the weights that generated the next rollout become the old actor of its training)."""
        a = self.args
        iv = getattr(a, "ref_update_interval", None)
        if self.need_ref and iv and (rollout_id + 1) % iv == 0:
            self.backuper.backup("ref")
        if getattr(a, "keep_old_actor", False):
            if (getattr(a, "update_weights_interval", 1) or 1) == 1:
                self.backuper.backups["old_actor"].copy_(self.backuper.backups["rollout_actor"])
                self.backuper.backup("rollout_actor")
            else:
                self.backuper.backup("old_actor")

    def _switch(self, tag: str):
        self.backuper.backup("actor")
        self.backuper.restore(tag)

    def train(self, rollout_id: int, data: dict) -> dict:
        a = self.args
        t0 = time.perf_counter()
        if (getattr(a, "balance_data", False) and self.dp_group is not None
                and torch.distributed.get_world_size(self.dp_group) > 1):
            if getattr(self.model, "cp", None) is not None:
                raise ValueError("--balance-data is not supported with context parallelism")
            from miles_b200.utils.seqlen_balancing import rebalance_over_dp

            data = rebalance_over_dp(data, self.dp_group)
        items = data_to_items(data)
        if getattr(a, "save_debug_train_data", None):
            import pickle

            path = a.save_debug_train_data.format(rollout_id=rollout_id, rank=self._rank())
            os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
            with open(path, "wb") as f:
                pickle.dump({k: v for k, v in data.items() if k != "metrics"}, f)
        if self._hook_before_lp is not None:
            self._hook_before_lp(a, self.model, "")
        old = None
        if not a.use_rollout_logprobs and not self.actor.cfg.old_logp_from_forward:
            old_actor = getattr(a, "keep_old_actor", False) and "old_actor" in self.backuper.backups
            if old_actor:  # old log-probs under the weights that generated this rollout
                self._switch("old_actor")
            old = self.actor.compute_logprobs(items)
            if old_actor:
                self.backuper.restore("actor")
            for it, o in zip(items, old):
                it.old_logp = o
        t1 = time.perf_counter()
        ref = None
        if self.need_ref:
            self._switch("ref")
            ref = self.actor.compute_logprobs(items)
            self.backuper.restore("actor")
            for it, r in zip(items, ref):
                it.ref_logp = r
        logp = old if old is not None else [np.asarray(it.rollout_logp) for it in items]
        values = self.critic.values(items) if self.critic is not None else None
        rets = None
        if not a.disable_compute_advantages_and_returns:
            advs, rets = compute_advantages(a, data, log_probs=logp, ref_log_probs=ref,
                                            values=values, dp_group=self.dp_group)
            for it, adv in zip(items, advs):
                it.advantage = adv
        if self._postprocess is not None:
            self._postprocess(a)  # reference hook signature: fn(args), after the advantages
        m = {}
        world = self.data_world
        if self.critic is not None and rets is not None:
            cm = self.critic.train_step(items, rets, values, global_num_samples=len(items) * world)
            m.update({f"critic/{k}": v for k, v in cm.items()})
            if rollout_id < (a.num_critic_only_steps or 0):
                m["perf/log_probs_time"] = t1 - t0
                self.metrics = m
                return m
        if old is not None and items and items[0].rollout_logp is not None:
            d = np.concatenate([np.abs(o - np.asarray(it.rollout_logp, np.float32)) for it, o in zip(items, old)])
            m["train/train_rollout_logprob_abs_diff"] = float(d.mean()) if d.size else 0.0
        steps = a.num_steps_per_rollout or 1
        per = (len(items) + steps - 1) // steps
        if getattr(a, "get_mismatch_metrics", False) and items and items[0].rollout_logp is not None:
            from miles_b200.trainer.mis import mismatch_metrics

            m.update(mismatch_metrics([it.old_logp if it.old_logp is not None else it.rollout_logp
                                       for it in items],
                                      [it.rollout_logp for it in items],
                                      [it.loss_mask for it in items]))
        for s in range(steps):
            sub = items[s * per:(s + 1) * per]
            if not sub:
                continue
            if self._hook_before_step is not None:
                self._hook_before_step(a, rollout_id, s, self.model, self.actor.opt,
                                       getattr(self.actor.cfg, "lr_schedule", None))
            out = self.actor.train_step(sub, global_num_samples=len(sub) * self.data_world)
            if "train_rollout_logprob_abs_diff" in out:  # old log-probs from the training forward
                m["train/train_rollout_logprob_abs_diff"] = out.pop("train_rollout_logprob_abs_diff")
            if getattr(a, "ci_save_grad_norm", None) or getattr(a, "ci_load_grad_norm", None):
                from miles_b200.utils.ci_utils import check_grad_norm

                check_grad_norm(a, out["grad_norm"], rollout_id, s, rank=self._rank())
            for k, v in out.items():
                m[f"train/{k}" if "/" not in k else k] = v
        if getattr(a, "reset_optimizer_states", False) and hasattr(self.actor.opt, "reset_state"):
            self.actor.opt.reset_state()  # fresh Adam moments for every rollout
        t2 = time.perf_counter()
        m["perf/log_probs_time"] = t1 - t0
        m["perf/actor_train_time"] = t2 - t1
        n_tok = sum(len(t) for t in data["tokens"])
        m["perf/actor_train_tok_per_s"] = n_tok / max(t2 - t1, 1e-9)
        from miles_b200.utils.flops import train_tflops

        if getattr(self.model, "cfg", None) is not None:  # the FSDP backend trains an HF module
            m["perf/actor_train_tflops"] = train_tflops(self.model.cfg, [len(t) for t in data["tokens"]],
                                                        t2 - t1)
        if a.ci_test:
            self.ci_checks(rollout_id, m)
        self.metrics = m
        return m

    def ci_checks(self, rollout_id: int, m: dict):
        """On-policy invariants (reference training_utils/ci_utils.py:12-24)."""
        if rollout_id == 0 and not self.args.ci_disable_logprobs_checker:
            d = m.get("train/train_rollout_logprob_abs_diff")
            assert d is None or d < 0.03, f"train/rollout log-prob mismatch {d}"
        if self.args.num_steps_per_rollout in (None, 1) and not self.args.ci_disable_kl_checker:
            w = max(m.get("train/weight", 1.0), 1e-12)
            assert abs(m.get("train/ppo_kl", 0.0) / w) < 1e-6, m.get("train/ppo_kl")
            assert m.get("train/pg_clipfrac", 0.0) / w < 1e-6
