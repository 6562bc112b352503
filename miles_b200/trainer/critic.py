"""PPO critic: the policy architecture with a scalar value head on the final hidden state.

    values(items)           forward-only values of every response position (V(s_t) is read
                            from the hidden state that predicts token t)
    train_step(items, ret, old_values)
                            clipped value loss 0.5 * max((V - R)^2, (clip(V, V_old +- c) - R)^2)
                            (per-sample token mean, or per-token with --calculate-per-token-loss),
                            backward through the body (flat gradient buffer, same machinery as
                            the actor, sharded optimizer over DP ranks) and the head

Reference: megatron_utils/actor.py train_critic (:336-362), model_provider.py value head
`LinearForLastLayer` (H -> 1), training_utils/loss.py value_loss_function (:719-774).
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from miles_b200.models.transformer import Transformer
from miles_b200.trainer.actor import Actor, ActorConfig, TrainItem, make_micro_batches


class Critic:
    def __init__(self, model: Transformer, cfg: ActorConfig, value_clip: float = 0.2,
                 dp_group=None):
        self.model = model
        self.body = Actor(model, cfg, dp_group=dp_group)
        self.cfg = cfg
        self.value_clip = value_clip
        self.dp_group = dp_group
        H = model.cfg.hidden_size
        self.head = torch.zeros(H, dtype=torch.float32, device=model.device, requires_grad=True)
        self.head_opt = torch.optim.Adam([self.head], lr=cfg.lr, betas=cfg.betas)

    def _values_of(self, sub: list[TrainItem]):
        tok, meta, sel, _ = self.body._mb_inputs(sub)
        h = self.model.forward_train(tok, meta)
        return h.index_select(0, sel).float() @ self.head

    @torch.no_grad()
    def values(self, items: list[TrainItem]) -> list[np.ndarray]:
        out: list[np.ndarray | None] = [None] * len(items)
        for mb in make_micro_batches([len(it.tokens) for it in items], self.cfg):
            sub = [items[i] for i in mb]
            v = self._values_of(sub).cpu().numpy()
            o = 0
            for i in mb:
                n = items[i].resp_len
                out[i] = v[o:o + n]
                o += n
        return out

    def train_step(self, items: list[TrainItem], returns: list[np.ndarray],
                   old_values: list[np.ndarray], global_num_samples: int | None = None) -> dict:
        body = self.body
        body._ensure_grads()
        body.grad_flat.zero_()
        self.head_opt.zero_grad(set_to_none=True)
        n_samples = global_num_samples or len(items)
        c = self.value_clip
        tot = {"value_loss": 0.0, "value_clipfrac": 0.0}
        for mb in make_micro_batches([len(it.tokens) for it in items], self.cfg):
            sub = [items[i] for i in mb]
            T = lambda xs: torch.from_numpy(np.concatenate(xs).astype(np.float32)).to(self.model.device)
            R = T([returns[i] for i in mb])
            old = T([old_values[i] for i in mb])
            w = T([np.asarray(items[i].loss_mask if items[i].loss_mask is not None
                              else [1] * items[i].resp_len, np.float32)
                   / max(1.0, float(np.sum(items[i].loss_mask)) if items[i].loss_mask is not None
                         else float(items[i].resp_len)) / n_samples for i in mb])
            v = self._values_of(sub)
            vc = old + (v - old).clamp(-c, c)
            l1, l2 = (v - R) ** 2, (vc - R) ** 2
            loss = 0.5 * (w * torch.maximum(l1, l2)).sum()
            loss.backward()
            tot["value_loss"] += float(loss.detach())
            tot["value_clipfrac"] += float((w * (l2 > l1).float()).sum())
        for name, p in self.model.params.items():
            if p.grad is not None:
                p.main_grad.add_(p.grad.to(p.main_grad.dtype))
                p.grad = None
        if self.dp_group is not None and dist.get_world_size(self.dp_group) > 1:
            if not body._sharded():
                body._reduce_grads()
            dist.all_reduce(self.head.grad, group=self.dp_group)
        body.opt.step()
        self.head_opt.step()
        tot["critic_grad_norm"] = float(body.opt.grad_norm())
        return tot
