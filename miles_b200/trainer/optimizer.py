"""Flat-buffer AdamW with device or host-offloaded state, optionally sharded over data-parallel
ranks (ZeRO-1).

State placements:
  * "device"  : fp32 master + fp32 m/v on the GPU (the default when it fits)
  * "host"    : bf16 m/v in pinned host memory, streamed through the GPU in chunks while the
                Adam kernel runs on the previous chunk (host->device and device->host copies on
                two streams, so both PCIe directions are busy at once); the bf16 parameters are
                the master copy and updates use stochastic rounding. This is the single-GPU
                placement for models whose fp32 state cannot fit (e.g. a 30B MoE on one B200).

Sharding (``dp_group`` with more than one rank): rank r owns elements [r*S, (r+1)*S) of the
flat buffers (S = n / world; the model pads its flat buffer so that n divides evenly). One step
is: reduce-scatter of the gradient into the owned shard (in place, NCCL), the global gradient
norm as an all-reduce of the shard norms, Adam on the shard only (optimizer state is 1/world
of the unsharded size, placed on the device when it fits), and an in-place all-gather of the
updated parameters. Replaces Megatron's distributed optimizer (the reference forces it:
megatron_utils/arguments.py:14; grad reduce-scatter / param all-gather in model.py:537-612).

Gradient clipping uses a device-side norm (no host sync); a non-finite gradient skips the
step on the device (the reference's NaN/Inf guard, megatron_utils/model.py:452-461).

Reference role: Megatron distributed optimizer / HybridDeviceOptimizer (--optimizer-cpu-offload).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from miles_b200.ops.optim import adam_, nonfinite_, sqnorm_


def _is_nccl(group) -> bool:
    try:
        return dist.get_backend(group) == "nccl"
    except Exception:  # noqa: BLE001
        return False


class FlatAdam:
    def __init__(self, params_flat: torch.Tensor, grads_flat: torch.Tensor, lr: float = 1e-6,
                 betas=(0.9, 0.98), eps: float = 1e-8, weight_decay: float = 0.0,
                 clip_grad: float = 1.0, placement: str = "auto", chunk: int = 1 << 28,
                 seed: int = 1234, dp_group=None, norm_group=None, norm_exclude=None,
                 expert_norm=None, host_state=None, memory_margin: int = 0, peer_grads=None):
        """norm_group / norm_exclude: under model parallelism (TP, PP) every rank runs its own
        optimizer over its part of the model; the gradient norm sums the squares over
        `norm_group`, leaving out this rank's flat ranges `norm_exclude` (parameters another
        rank of the group already counts: TP-replicated ones on TP ranks > 0, the last pipeline
        stage's copy of tied embeddings). expert_norm = (offset, groups): under expert
        parallelism the flat tail from `offset` (this rank's experts) is summed over each of
        `groups` in turn (TP when experts are TP-split, then EP) instead of `norm_group`.
        peer_grads: a `parallel.symm.PeerGradBuffer` whose tensor is `grads_flat`; the gradient
        reduce-scatter then runs as the fused peer-memory kernel (sum, cast and shard norm in one
        pass) instead of NCCL."""
        self.p = params_flat
        self.expert_norm = expert_norm
        self.norm_group = norm_group
        self.norm_world = dist.get_world_size(norm_group) if norm_group is not None else 1
        self.norm_exclude = list(norm_exclude or [])
        self.g = grads_flat
        self.peer_grads = peer_grads
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
        self.group = dp_group
        self.world = dist.get_world_size(dp_group) if dp_group is not None else 1
        self.rank = dist.get_rank(dp_group) if dp_group is not None else 0
        if self.world > 1 and n % self.world:
            raise ValueError(f"flat buffer of {n} elements does not split over {self.world} ranks")
        self.shard = n // self.world
        self.lo = self.rank * self.shard
        ns = self.shard
        if placement == "auto":
            placement = "device"
            if dev.type == "cuda":
                free, _ = torch.cuda.mem_get_info(dev)
                if 12 * ns > 0.8 * (free - memory_margin):
                    placement = "host"
        self.placement = placement
        if placement == "device":
            self.master = params_flat[self.lo:self.lo + ns].float()
            self.m = torch.zeros(ns, dtype=torch.float32, device=dev)
            self.v = torch.zeros(ns, dtype=torch.float32, device=dev)
        else:
            self.master = None
            # bf16 m / v in host memory, page-locked on a worker thread (possibly started
            # earlier by the actor: `host_state`); the first step waits for it
            from miles_b200.utils.host_memory import BackgroundPinned

            if host_state is None or host_state[0].tensor.numel() != ns:
                host_state = (BackgroundPinned(ns, torch.bfloat16), BackgroundPinned(ns, torch.bfloat16))
            self._pinning = host_state
            self.m, self.v = host_state[0].tensor, host_state[1].tensor
            if dev.type == "cuda":
                c = min(chunk, ns)
                self.stage = [(torch.empty(c, dtype=torch.bfloat16, device=dev),
                               torch.empty(c, dtype=torch.bfloat16, device=dev)) for _ in range(2)]
                self.h2d = torch.cuda.Stream(dev)
                self.d2h = torch.cuda.Stream(dev)
        self.sq = torch.zeros(1, dtype=torch.float32, device=dev)
        self.skip = torch.zeros(1, dtype=torch.float32, device=dev)

    def grad_norm(self) -> torch.Tensor:
        return self.sq.sqrt()

    # ------------------------------------------------------------------ collectives
    def _reduce_scatter_grads(self) -> bool:
        """Reduce-scatter the gradient into this rank's shard; True when the fused peer kernel
        ran (it also leaves the shard's squared norm in self.sq)."""
        pg = self.peer_grads
        if (pg is not None and self.g.data_ptr() == pg.tensor.data_ptr()
                and self.lo % 8 == 0 and self.shard % 8 == 0):
            pg.reduce_scatter(self.lo, self.shard, self.sq)
            return True
        mine = self.g[self.lo:self.lo + self.shard]
        if _is_nccl(self.group):
            dist.reduce_scatter_tensor(mine, self.g, group=self.group)  # in place
        else:  # gloo has no reduce-scatter: sum everything, keep the shard
            dist.all_reduce(self.g, group=self.group)
        return False

    def _all_gather_params(self) -> None:
        mine = self.p[self.lo:self.lo + self.shard]
        if _is_nccl(self.group):
            dist.all_gather_into_tensor(self.p, mine, group=self.group)  # in place
        else:
            parts = list(self.p.view(self.world, self.shard).unbind(0))
            gathered = [torch.empty_like(mine) for _ in range(self.world)]
            dist.all_gather(gathered, mine.clone(), group=self.group)
            for dst, src in zip(parts, gathered):
                dst.copy_(src)

    # ------------------------------------------------------------------ offload
    @torch.no_grad()
    def offload(self, force: bool = False) -> None:
        """Move device-placed state (fp32 master, m, v) into pinned host buffers and free the
        device copies: colocated training gives that memory to the rollout's KV cache (the
        reference's torch_memory_saver offload of the optimizer). The next step() brings it
        back first. `force` also runs the copy for CPU state (tests)."""
        if self.placement != "device" or getattr(self, "_parked", None) is not None:
            return
        if self.m.device.type != "cuda" and not force:
            return
        pin = self.m.device.type == "cuda"
        keep = {}
        for k in ("master", "m", "v"):
            t = getattr(self, k)
            if t is None:
                continue
            buf = getattr(self, "_pinned", {}).get(k)
            if buf is None or buf.shape != t.shape:
                buf = torch.empty(t.shape, dtype=t.dtype, pin_memory=pin)
            buf.copy_(t, non_blocking=pin)
            keep[k] = buf
        if pin:
            torch.cuda.current_stream(self.m.device).synchronize()
        self._dev = self.m.device
        self._pinned = keep
        self._parked = keep
        for k in keep:
            setattr(self, k, None)
        if pin:
            torch.cuda.empty_cache()

    @torch.no_grad()
    def onload(self) -> None:
        """Bring offloaded state back to the device (no-op when it is there)."""
        parked = getattr(self, "_parked", None)
        if parked is None:
            return
        pin = self._dev.type == "cuda"
        for k, buf in parked.items():
            setattr(self, k, buf.to(self._dev, non_blocking=pin) if pin else buf.clone())
        self._parked = None

    # ------------------------------------------------------------------ step
    @torch.no_grad()
    def step(self) -> None:
        self.onload()
        self.step_id += 1
        fused = self._reduce_scatter_grads() if self.world > 1 else False
        lo, hi = self.lo, self.lo + self.shard
        p, g = self.p[lo:hi], self.g[lo:hi]
        self.skip.zero_()
        if not fused:
            self.sq.zero_()
            sqnorm_(g, self.sq)
        if self.norm_world > 1 and self.norm_exclude:
            sq_x = torch.zeros_like(self.sq)
            for a, b in self.norm_exclude:
                a, b = max(a, lo), min(b, hi)
                if a < b:
                    sqnorm_(self.g[a:b], sq_x)
            self.sq.sub_(sq_x)
        sq_e = None
        if self.expert_norm is not None:
            off, _ = self.expert_norm
            sq_e = torch.zeros_like(self.sq)
            if max(off, lo) < hi:
                sqnorm_(self.g[max(off, lo):hi], sq_e)
            self.sq.sub_(sq_e)
        if self.world > 1:
            dist.all_reduce(self.sq, group=self.group)
        if self.norm_world > 1:
            dist.all_reduce(self.sq, group=self.norm_group)
        if sq_e is not None:
            for grp in self.expert_norm[1]:
                if dist.get_world_size(grp) > 1:
                    dist.all_reduce(sq_e, group=grp)
            self.sq.add_(sq_e)
        nonfinite_(self.sq, self.skip)
        common = dict(lr=self.lr, betas=self.betas, eps=self.eps, weight_decay=self.wd,
                      step=self.step_id, sqnorm=self.sq, max_norm=self.clip,
                      seed=self.seed * 1000003 + self.step_id + 7919 * self.rank, skip=self.skip)
        if self.placement == "device" or p.device.type != "cuda":
            adam_(p, g, self.m, self.v, master=self.master, **common)
        else:
            self._host_step(p, g, common)
        if self.world > 1:
            self._all_gather_params()

    def _host_step(self, p: torch.Tensor, g: torch.Tensor, common: dict) -> None:
        for b in self._pinning:
            b.wait()
        n = p.numel()
        cur = torch.cuda.current_stream(p.device)
        backs: list[torch.cuda.Event] = []
        for ci, a in enumerate(range(0, n, self.chunk)):
            b = min(n, a + self.chunk)
            sm, sv = self.stage[ci % 2]
            sm, sv = sm[: b - a], sv[: b - a]
            with torch.cuda.stream(self.h2d):
                if ci >= 2:
                    self.h2d.wait_event(backs[ci - 2])  # stage buffer free (its D2H finished)
                sm.copy_(self.m[a:b], non_blocking=True)
                sv.copy_(self.v[a:b], non_blocking=True)
                loaded = torch.cuda.Event()
                loaded.record(self.h2d)
            cur.wait_event(loaded)
            common["seed"] = self.seed * 1000003 + self.step_id * 4099 + ci + 7919 * self.rank
            adam_(p[a:b], g[a:b], sm, sv, master=None, **common)
            done = torch.cuda.Event()
            done.record(cur)
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(done)
                self.m[a:b].copy_(sm, non_blocking=True)
                self.v[a:b].copy_(sv, non_blocking=True)
                back = torch.cuda.Event()
                back.record(self.d2h)
            backs.append(back)
        cur.wait_stream(self.d2h)

    def reset_state(self) -> None:
        """--reset-optimizer-states: zero the moments and the step count (master copy kept)."""
        self.onload()
        for b in getattr(self, "_pinning", ()):
            b.wait()
        self.step_id = 0
        self.m.zero_()
        self.v.zero_()

    def state_dict(self) -> dict:
        self.onload()
        return {"step": self.step_id, "m": self.m, "v": self.v, "master": self.master,
                "placement": self.placement, "shard": (self.rank, self.world)}

    def load_state_dict(self, sd: dict) -> None:
        self.onload()
        self.step_id = sd["step"]
        self.m.copy_(sd["m"])
        self.v.copy_(sd["v"])
        if self.master is not None and sd.get("master") is not None:
            self.master.copy_(sd["master"])
