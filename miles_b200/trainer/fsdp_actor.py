"""FSDP2 training backend (`--train-backend fsdp`): HuggingFace models, fully sharded.

For model families this framework's own Transformer does not implement, or when a user wants
the HF module itself, the policy is an `AutoModelForCausalLM` whose decoder layers and root are
wrapped with PyTorch FSDP2 (`fully_shard`): parameters, gradients and AdamW states are sharded
over the data-parallel mesh, each layer's parameters are all-gathered for its forward /
backward and the gradients reduce-scattered. Everything above the model is shared with the
native backend: micro-batch packing, the loss terms (`Actor._mb_prepare`, `Actor._loss`: PPO /
GSPO / TIS / OPSM / KL / SFT / custom losses) and the metric layout.

Samples run one at a time through the HF model (no packed varlen attention in HF modules);
the log-prob / entropy of the response tokens come from the full logits in fp32. The loss is
a sum over the global batch (normalised by the global sample / token count like the native
actor), so it is multiplied by the mesh size to undo FSDP's gradient averaging.

`export_hf_state()` gathers the full parameters under their HF names (collective) — the
rollout engine loads them into its own Transformer (`checkpoint.hf.load_hf_tensors`).

Reference: miles/backends/fsdp_utils/actor.py (FSDPTrainRayActor: fully_shard per decoder layer
and root :667-718, train / log-prob loops), fsdp_utils/parallel.py (device mesh).
"""
from __future__ import annotations

import time

import numpy as np
import torch
import torch.distributed as dist
import torch.nn.functional as F

from miles_b200.ops.rl import METRIC_NAMES
from miles_b200.trainer.actor import Actor, ActorConfig, TrainItem, make_micro_batches


class FSDPActor(Actor):
    def __init__(self, hf_path_or_model, cfg: ActorConfig, dp_group=None, device="cpu",
                 dtype=torch.float32):
        from torch.distributed.device_mesh import DeviceMesh
        from torch.distributed.fsdp import fully_shard

        if isinstance(hf_path_or_model, str):
            from transformers import AutoModelForCausalLM

            hf = AutoModelForCausalLM.from_pretrained(hf_path_or_model, torch_dtype=dtype)
        else:
            hf = hf_path_or_model
        self.dev = torch.device(device)
        hf = hf.to(self.dev)
        self.cfg = cfg
        self.dp_group = dp_group
        self.world = dist.get_world_size(dp_group) if dist.is_initialized() else 1
        if dist.is_initialized():
            group = dp_group or dist.group.WORLD
            ranks = dist.get_process_group_ranks(group)
            mesh = DeviceMesh.from_group(group, self.dev.type, mesh=torch.tensor(ranks))
            for layer in hf.model.layers:
                fully_shard(layer, mesh=mesh)
            fully_shard(hf, mesh=mesh)
        self.hf = hf
        self.model = None  # no native Transformer behind this actor
        self.opt = torch.optim.AdamW(hf.parameters(), lr=cfg.lr, betas=cfg.betas,
                                     weight_decay=cfg.weight_decay, eps=1e-8)
        self.timers: dict = {}
        self._custom_loss = None
        self._custom_tis = None
        self.weight_version = 0

    # ------------------------------------------------------------------ native-actor hooks
    def _ensure_grads(self):
        pass

    def release_grads(self):
        self.opt.zero_grad(set_to_none=True)

    def _replay(self, items):
        return None  # routing replay needs the native MoE layer

    # ------------------------------------------------------------------ model pieces
    def _sample_logprob(self, it: TrainItem, temperature: float):
        toks = torch.tensor(it.tokens, dtype=torch.long, device=self.dev)[None]
        logits = self.hf(toks).logits[0].float() / temperature
        z = logits[it.prompt_len - 1:len(it.tokens) - 1]
        lsm = torch.log_softmax(z, -1)
        tgt = toks[0, it.prompt_len:]
        lp = lsm.gather(1, tgt[:, None])[:, 0]
        ent = -(lsm.exp() * lsm).sum(-1)
        return lp, ent

    @torch.no_grad()
    def compute_logprobs(self, items: list[TrainItem]) -> list[np.ndarray]:
        return [self._sample_logprob(it, self.cfg.temperature)[0].cpu().numpy() for it in items]

    def train_step(self, items: list[TrainItem], global_num_samples: int | None = None,
                   global_num_tokens: int | None = None) -> dict:
        cfg = self.cfg
        t0 = time.perf_counter()
        self.opt.zero_grad(set_to_none=True)
        n_samples = global_num_samples or len(items)
        n_tokens = global_num_tokens or sum(
            (sum(it.loss_mask) if it.loss_mask is not None else it.resp_len) for it in items)
        metrics = torch.zeros(len(METRIC_NAMES) + 1, dtype=torch.float64, device=self.dev)
        mbs = make_micro_batches([len(it.tokens) for it in items], cfg)
        for mb in mbs:
            for i in mb:
                prep = self._mb_prepare([items[i]], n_samples, n_tokens)
                lp, ent = self._sample_logprob(items[i], cfg.temperature)
                loss = self._mb_loss(prep, lp, ent, metrics)
                (loss * self.world).backward()  # FSDP averages gradients over the mesh
        gn = torch.nn.utils.clip_grad_norm_(self.hf.parameters(), cfg.clip_grad)
        gn = gn.full_tensor() if hasattr(gn, "full_tensor") else gn
        if torch.isfinite(gn):
            self.opt.step()
        self.weight_version += 1
        out = {k: float(v) for k, v in zip(METRIC_NAMES + ["entropy"], metrics.tolist())}
        out["grad_norm"] = float(gn)
        out["num_microbatches"] = len(mbs)
        self.timers["train_total"] = time.perf_counter() - t0
        return out

    def export_hf_state(self) -> dict[str, torch.Tensor]:
        """Full parameters under their HF names (every rank takes part)."""
        out = {}
        for name, p in self.hf.named_parameters():
            t = p.detach()
            out[name] = t.full_tensor() if hasattr(t, "full_tensor") else t
        return out
