"""Flat-buffer AdamW with device or host-offloaded state.

State placements:
  * "device"  : fp32 master + fp32 m/v on the GPU (the default when it fits)
  * "host"    : bf16 m/v in pinned host memory, streamed through the GPU in chunks on a copy
                stream while the Adam kernel runs on the previous chunk; the bf16 parameters are
                the master copy and updates use stochastic rounding. This is the single-GPU
                placement for models whose fp32 state cannot fit (e.g. a 30B MoE on one B200).
Gradient clipping uses a device-side norm (no host sync); a non-finite gradient skips the
step on the device (the reference's NaN/Inf guard, megatron_utils/model.py:452-461).

Reference role: Megatron distributed optimizer / HybridDeviceOptimizer (--optimizer-cpu-offload).
"""
from __future__ import annotations

import torch

from miles_b200.ops.optim import adam_, nonfinite_, sqnorm_


class FlatAdam:
    def __init__(self, params_flat: torch.Tensor, grads_flat: torch.Tensor, lr: float = 1e-6,
                 betas=(0.9, 0.98), eps: float = 1e-8, weight_decay: float = 0.0,
                 clip_grad: float = 1.0, placement: str = "auto", chunk: int = 1 << 28,
                 seed: int = 1234):
        self.p = params_flat
        self.g = grads_flat
        self.lr = lr
        self.betas = betas
        self.eps = eps
        self.wd = weight_decay
        self.clip = clip_grad
        self.step_id = 0
        self.seed = seed
        self.chunk = chunk
        n = params_flat.numel()
        dev = params_flat.device
        if placement == "auto":
            placement = "device"
            if dev.type == "cuda":
                free, _ = torch.cuda.mem_get_info(dev)
                if 12 * n > 0.8 * free:
                    placement = "host"
        self.placement = placement
        if placement == "device":
            self.master = params_flat.float()
            self.m = torch.zeros(n, dtype=torch.float32, device=dev)
            self.v = torch.zeros(n, dtype=torch.float32, device=dev)
        else:
            self.master = None
            pin = dev.type == "cuda"
            self.m = torch.zeros(n, dtype=torch.bfloat16, pin_memory=pin)
            self.v = torch.zeros(n, dtype=torch.bfloat16, pin_memory=pin)
            if dev.type == "cuda":
                c = min(chunk, n)
                self.stage = [(torch.empty(c, dtype=torch.bfloat16, device=dev),
                               torch.empty(c, dtype=torch.bfloat16, device=dev)) for _ in range(2)]
                self.copy_stream = torch.cuda.Stream(dev)
        self.sq = torch.zeros(1, dtype=torch.float32, device=dev)
        self.skip = torch.zeros(1, dtype=torch.float32, device=dev)

    def grad_norm(self) -> torch.Tensor:
        return self.sq.sqrt()

    @torch.no_grad()
    def step(self) -> None:
        self.step_id += 1
        self.sq.zero_()
        self.skip.zero_()
        sqnorm_(self.g, self.sq)
        nonfinite_(self.sq, self.skip)
        common = dict(lr=self.lr, betas=self.betas, eps=self.eps, weight_decay=self.wd,
                      step=self.step_id, sqnorm=self.sq, max_norm=self.clip,
                      seed=self.seed * 1000003 + self.step_id, skip=self.skip)
        if self.placement == "device":
            adam_(self.p, self.g, self.m, self.v, master=self.master, **common)
            return
        if self.p.device.type != "cuda":
            adam_(self.p, self.g, self.m, self.v, master=None, **common)
            return
        n = self.p.numel()
        cur = torch.cuda.current_stream(self.p.device)
        cs = self.copy_stream
        events = []
        for ci, a in enumerate(range(0, n, self.chunk)):
            b = min(n, a + self.chunk)
            sm, sv = self.stage[ci % 2]
            sm, sv = sm[: b - a], sv[: b - a]
            with torch.cuda.stream(cs):
                if len(events) >= 2:
                    cs.wait_event(events[-2])  # stage buffer free again (its D2H has finished)
                sm.copy_(self.m[a:b], non_blocking=True)
                sv.copy_(self.v[a:b], non_blocking=True)
                loaded = torch.cuda.Event()
                loaded.record(cs)
            cur.wait_event(loaded)
            common["seed"] = self.seed * 1000003 + self.step_id * 4099 + ci
            adam_(self.p[a:b], self.g[a:b], sm, sv, master=None, **common)
            done = torch.cuda.Event()
            done.record(cur)
            with torch.cuda.stream(cs):
                cs.wait_event(done)
                self.m[a:b].copy_(sm, non_blocking=True)
                self.v[a:b].copy_(sv, non_blocking=True)
                back = torch.cuda.Event()
                back.record(cs)
            events.append(back)
        cur.wait_stream(cs)

    def state_dict(self) -> dict:
        return {"step": self.step_id, "m": self.m, "v": self.v, "master": self.master,
                "placement": self.placement}

    def load_state_dict(self, sd: dict) -> None:
        self.step_id = sd["step"]
        self.m.copy_(sd["m"])
        self.v.copy_(sd["v"])
        if self.master is not None and sd.get("master") is not None:
            self.master.copy_(sd["master"])
