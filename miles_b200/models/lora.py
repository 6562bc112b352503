"""LoRA adapters on the transformer's dense projections.

y = x W^T + (alpha / r) * (x A^T) B^T, with A [r, in] (Kaiming-uniform init) and B [out, r]
(zero init), fp32 master weights cast to bf16 for the GEMMs. The base weights stay frozen;
only the adapters are trained (their own AdamW with global-norm clipping, DP all-reduce of
the adapter gradients). Training and rollout run the same forward code (the transformer's
`_lin`), so the engine generates with the adapters applied and train/rollout log-probs stay
bitwise equal. The adapter GEMMs go through the batch-invariant tcgen05 GEMM like every other
projection.

Target names follow the reference / PEFT convention: q_proj, k_proj, v_proj (-> our fused
qkv_proj), o_proj, gate_proj, up_proj (-> fused gate_up_proj), down_proj, or "all-linear".
MoE expert weights are not adapted.

Reference: miles/backends/megatron_utils/lora_utils.py (:82-472: target modules, adapter
save/load), bridge_lora_helpers.py, arguments.py:1026-1078 (--lora-rank/alpha/dropout/
target-modules/adapter-path).
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

_TARGET_MAP = {
    "q_proj": "self_attn.qkv_proj.weight", "k_proj": "self_attn.qkv_proj.weight",
    "v_proj": "self_attn.qkv_proj.weight", "qkv_proj": "self_attn.qkv_proj.weight",
    "o_proj": "self_attn.o_proj.weight",
    "gate_proj": "mlp.gate_up_proj.weight", "up_proj": "mlp.gate_up_proj.weight",
    "gate_up_proj": "mlp.gate_up_proj.weight", "down_proj": "mlp.down_proj.weight",
}


def resolve_targets(targets) -> set[str]:
    if targets is None or targets == "all-linear" or targets == ["all-linear"]:
        targets = ["qkv_proj", "o_proj", "gate_up_proj", "down_proj"]
    if isinstance(targets, str):
        targets = [t.strip() for t in targets.split(",") if t.strip()]
    out = set()
    for t in targets:
        if t not in _TARGET_MAP:
            raise ValueError(f"unknown LoRA target module {t}")
        out.add(_TARGET_MAP[t])
    return out


class LoRA:
    def __init__(self, model, rank: int, alpha: float, targets=None, dropout: float = 0.0,
                 seed: int = 0, exclude=None):
        """exclude: module names (e.g. "o_proj", "layers.0.") whose weights get no adapter
        even when a target matches (--exclude-modules)."""
        self.rank = rank
        self.scale = alpha / rank
        self.dropout = dropout
        suffixes = resolve_targets(targets)
        g = torch.Generator(device="cpu").manual_seed(seed)
        self.A: dict[str, torch.nn.Parameter] = {}
        self.B: dict[str, torch.nn.Parameter] = {}
        for name, p in model.params.items():
            if p.dim() != 2 or not any(name.endswith(sfx) for sfx in suffixes):
                continue
            if exclude and any(e in name for e in exclude):
                continue
            out_f, in_f = p.shape
            bound = 1.0 / math.sqrt(in_f)  # kaiming-uniform(a=sqrt(5)) bound for A
            a = (torch.rand(rank, in_f, generator=g) * 2 - 1) * bound
            self.A[name] = torch.nn.Parameter(a.to(model.device))
            self.B[name] = torch.nn.Parameter(torch.zeros(out_f, rank, device=model.device))

    def __contains__(self, name: str) -> bool:
        return name in self.A

    def parameters(self):
        for n in self.A:
            yield self.A[n]
            yield self.B[n]

    def delta(self, name: str, x: torch.Tensor) -> torch.Tensor:
        from miles_b200.ops import gemm as G

        A, B = self.A[name], self.B[name] * self.scale
        if self.dropout and torch.is_grad_enabled():
            x = torch.nn.functional.dropout(x, self.dropout)
        pad = (-self.rank) % 16  # the tcgen05 GEMM wants N, K multiples of 16: zero-pad the rank
        if pad and x.is_cuda:
            A = torch.nn.functional.pad(A, (0, 0, 0, pad))
            B = torch.nn.functional.pad(B, (0, pad))
        t = G.linear(x, A.to(x.dtype))
        return G.linear(t, B.to(x.dtype))

    @torch.no_grad()
    def merged(self, name: str, w: torch.Tensor) -> torch.Tensor:
        """W + scale * B A (for export)."""
        return (w.float() + self.scale * (self.B[name] @ self.A[name])).to(w.dtype)

    def state_dict(self) -> dict:
        sd = {}
        for n in self.A:
            sd[f"{n}.lora_A"] = self.A[n].detach().cpu()
            sd[f"{n}.lora_B"] = self.B[n].detach().cpu()
        return sd

    @torch.no_grad()
    def load_state_dict(self, sd: dict):
        for n in self.A:
            self.A[n].copy_(sd[f"{n}.lora_A"])
            self.B[n].copy_(sd[f"{n}.lora_B"])

    def save(self, path: str):
        torch.save({"rank": self.rank, "scale": self.scale, "tensors": self.state_dict()}, path)

    def load(self, path: str):
        blob = torch.load(path, map_location="cpu", weights_only=False)
        self.load_state_dict(blob["tensors"])


class LoRAOptimizer:
    """AdamW over the adapters with global-norm clipping and DP gradient all-reduce (the
    interface the actor expects from its optimizer: step(), grad_norm(), g)."""

    def __init__(self, lora: LoRA, lr: float, betas=(0.9, 0.98), weight_decay: float = 0.0,
                 clip_grad: float = 1.0, dp_group=None):
        self.lora = lora
        self.params = list(lora.parameters())
        self.opt = torch.optim.AdamW(self.params, lr=lr, betas=betas, weight_decay=weight_decay)
        self.clip = clip_grad
        self.dp_group = dp_group
        self.g = None
        self.step_id = 0
        self._norm = torch.zeros(())

    @property
    def lr(self) -> float:
        return self.opt.param_groups[0]["lr"]

    @lr.setter
    def lr(self, v: float) -> None:
        for g in self.opt.param_groups:
            g["lr"] = v

    def grad_norm(self) -> torch.Tensor:
        return self._norm

    @torch.no_grad()
    def step(self):
        self.step_id += 1
        grads = [p.grad for p in self.params if p.grad is not None]
        if self.dp_group is not None and dist.get_world_size(self.dp_group) > 1:
            for g in grads:
                dist.all_reduce(g, group=self.dp_group)
        if grads:
            self._norm = torch.nn.utils.clip_grad_norm_(self.params, self.clip if self.clip > 0 else float("inf"))
        self.opt.step()
        self.opt.zero_grad(set_to_none=True)

    def reset_state(self) -> None:
        self.step_id = 0
        self.opt.state.clear()

    def state_dict(self) -> dict:
        return {"step": self.step_id, "adam": self.opt.state_dict()}

    def load_state_dict(self, sd: dict):
        self.step_id = sd["step"]
        self.opt.load_state_dict(sd["adam"])
