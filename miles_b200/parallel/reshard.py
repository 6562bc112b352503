"""Trainer -> rollout engine weight refit across different parallel layouts (resharding).

The trainer runs any TP x PP layout (e.g. TP8, or TP4 x PP2); the engines run their own TP
layout (e.g. one TP8 engine over eight ranks, or TP1 engines). The flat-buffer broadcast of
`refit.WeightRefit` needs identical layouts on both sides; this refit goes through the
layout-free currency of the HF tensors instead:

  1. Every trainer stage's TP ranks walk their HF tensors (`checkpoint.hf.to_hf_tensors`, fused
     projections already split into q / k / v and gate / up) and all-gather each one to its full
     shape (`parallel.tp.tp_gather_for`, which also restores the per-head block order of the
     Gated DeltaNet projections).
  2. The stage's TP rank 0 packs the full tensors into buckets (`bucket_bytes`) and broadcasts
     each bucket to the engine ranks over a group of {that rank} + engines: bf16, or with
     `mode="fp8"` every 2-D weight as 128 x 128 block-quantised e4m3 + fp32 scales (about half
     the bytes; the quantisation runs on the gathered tensor, so the blocks are those of the
     full weight, like the reference's quantizer at refit).
  3. Every engine takes its own TP slice of each tensor (`parallel.tp.tp_slice_for`, the same
     slicing an HF checkpoint load uses) into its flat parameter buffer, and bumps its weight
     version.

Expert-parallel trainers: every (stage, EP rank) has its own source (its TP rank 0; the lowest
global rank among expert-data-parallel replicas): EP rank 0 sends the dense tensors and its
experts, the other EP ranks only their experts (global expert ids in the HF names), so every
expert crosses once. Engines hold every expert (no EP on the engine side).

Every rank of the job calls `ReshardRefit(...)` (it creates the source groups) and then
`update()` with the same arguments.

Reference: miles/backends/megatron_utils/update_weight/common.py:50-134 (TP all-gather of the
shards, GLU stride fix, PP / EP broadcasts), hf_weight_iterator_direct.py:19-215 (HF-named
bucketed iteration), processors/quantizer_fp8.py:10-109 (128 x 128 fp8 at refit).
"""
from __future__ import annotations

import time

import torch
import torch.distributed as dist

from miles_b200.checkpoint.hf import to_hf_tensors
from miles_b200.ops.quant import fp8_block_dequant, fp8_block_quant
from miles_b200.parallel.tp import tp_gather_for, tp_slice_for


def _stage_of(model) -> int:
    return model.pp.stage if getattr(model, "pp", None) is not None else 0


def _tp_rank(model) -> int:
    return model.tp.rank if getattr(model, "tp", None) is not None else 0


def _ep_rank(model) -> int:
    return model.ep.rank if getattr(model, "ep", None) is not None else 0


def _is_expert(name: str) -> bool:
    return ".mlp.experts." in name


class ReshardRefit:
    def __init__(self, train_model, engine_model, trainer_ranks: list[int], engine_ranks: list[int],
                 bucket_bytes: int = 512 << 20, mode: str = "bf16"):
        """train_model: this rank's trainer model (any TP x PP, no EP) or None; engine_model: this
        rank's engine model (any TP, no PP) or None. A rank may hold both (colocated trainer and
        engine in different layouts on the same GPUs). trainer_ranks / engine_ranks: global
        ranks, the same lists on every rank."""
        if mode not in ("bf16", "fp8"):
            raise ValueError(f"unknown refit mode {mode}")
        if engine_model is not None and getattr(engine_model, "ep", None) is not None:
            raise ValueError("resharding refit: engines hold every expert (no expert parallelism)")
        if engine_model is not None and getattr(engine_model, "pp", None) is not None:
            raise ValueError("resharding refit: engines hold every layer (no pipeline stages)")
        self.train, self.engine, self.mode = train_model, engine_model, mode
        self.bucket = max(1 << 20, int(bucket_bytes))
        self.engines = list(engine_ranks)
        ref = engine_model if engine_model is not None else train_model
        self.wire = ref.flat.dtype  # bf16 on GPUs (fp32 in CPU runs)
        self.esize = ref.flat.element_size()
        me = dist.get_rank()
        # (stage, EP rank, TP rank) of every trainer rank: each (stage, EP rank)'s TP rank 0 with
        # the lowest global rank is its source
        info = None if train_model is None else (_stage_of(train_model), _ep_rank(train_model),
                                                 _tp_rank(train_model))
        allinfo: list = [None] * dist.get_world_size()
        dist.all_gather_object(allinfo, (me, info))
        self.leaders: dict[tuple, int] = {}    # (stage, ep rank) -> global rank of the source
        for r, inf in sorted(allinfo, key=lambda x: x[0]):
            if inf is not None and inf[2] == 0 and r in trainer_ranks:
                self.leaders.setdefault((inf[0], inf[1]), r)
        self.stages = sorted(self.leaders)
        # one broadcast group per source: it + the engines (created by every rank, in the same
        # order)
        self.groups = {s: dist.new_group(sorted({self.leaders[s]} | set(self.engines)))
                       for s in self.stages}
        self.last_stats: dict = {}

    # ------------------------------------------------------------------ packing
    def _encode(self, name: str, t: torch.Tensor) -> list[torch.Tensor]:
        """Payload tensors of one full tensor (flattened bytes)."""
        if self.mode == "fp8" and t.dim() == 2 and t.shape[0] >= 128 and t.shape[1] >= 128:
            q, s = fp8_block_quant(t.contiguous().to(torch.bfloat16), (128, 128))
            return [q.view(torch.uint8).reshape(-1), s.float().contiguous().view(torch.uint8).reshape(-1)]
        return [t.contiguous().to(self.wire).view(torch.uint8).reshape(-1)]

    def _payload_sizes(self, shape: tuple) -> list[int]:
        n = 1
        for d in shape:
            n *= d
        if self.mode == "fp8" and len(shape) == 2 and shape[0] >= 128 and shape[1] >= 128:
            return [n, ((shape[0] + 127) // 128) * ((shape[1] + 127) // 128) * 4]
        return [self.esize * n]

    def _decode(self, shape: tuple, parts: list[torch.Tensor]) -> torch.Tensor:
        if len(parts) == 2:
            q = parts[0].view(torch.float8_e4m3fn).view(*shape)
            s = parts[1].view(torch.float32).view((shape[0] + 127) // 128, (shape[1] + 127) // 128)
            return fp8_block_dequant(q, s, (128, 128), dtype=self.wire)
        return parts[0].view(self.wire).view(*shape)

    # ------------------------------------------------------------------ transfer
    def _apply(self, shapes, buf, targets) -> None:
        """Engine: copy this engine's TP slice of every tensor of a received bucket in place."""
        model, off = self.engine, 0
        for name, shape in shapes:
            parts = []
            for sz in self._payload_sizes(shape):
                parts.append(buf[off:off + sz])
                off += sz
            if name not in targets:
                if name == "lm_head.weight" and model.cfg.tie_embeddings:
                    continue
                raise KeyError(f"engine has no tensor {name}")
            dst = targets[name]
            dst.copy_(tp_slice_for(model, name, self._decode(shape, parts)).to(dst.dtype))

    def _send(self, items, leader: int, grp, targets) -> int:
        """Leader: broadcast one bucket (names + shapes, then the packed payload); an empty
        bucket marks the end of the stage. A leader that is also an engine applies it too."""
        meta = [[(n, tuple(t.shape)) for n, t in items]]
        dist.broadcast_object_list(meta, src=leader, group=grp)
        if not items:
            return 0
        parts = [p for n, t in items for p in self._encode(n, t)]
        buf = torch.cat(parts) if len(parts) > 1 else parts[0]
        dist.broadcast(buf, leader, group=grp)
        if targets is not None:
            self._apply(meta[0], buf, targets)
        return buf.numel()

    def _recv(self, leader: int, grp, dev, targets) -> int:
        """Engine: receive one bucket and apply it; returns the payload bytes, or -1 at the end
        of the stage."""
        meta = [None]
        dist.broadcast_object_list(meta, src=leader, group=grp)
        shapes = meta[0]
        if not shapes:
            return -1
        nbytes = sum(sum(self._payload_sizes(shape)) for _, shape in shapes)
        buf = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        dist.broadcast(buf, leader, group=grp)
        self._apply(shapes, buf, targets)
        return nbytes

    @torch.no_grad()
    def update(self, version: int | None = None) -> dict:
        t0 = time.perf_counter()
        me = dist.get_rank()
        ref = self.engine if self.engine is not None else self.train
        dev = ref.flat.device
        sent = 0
        my_stage = None if self.train is None else (_stage_of(self.train), _ep_rank(self.train))
        targets = dict(to_hf_tensors(self.engine)) if self.engine is not None else None
        for s in self.stages:
            leader, grp = self.leaders[s], self.groups[s]
            if my_stage == s:
                # the stage's TP ranks gather tensor by tensor; the leader streams buckets
                pending: list[tuple[str, torch.Tensor]] = []
                size = 0
                for name, local in to_hf_tensors(self.train):
                    if s[1] != 0 and not _is_expert(name):
                        continue  # dense tensors come from EP rank 0 (same on every TP peer)
                    g = tp_gather_for(self.train, name, local.detach())
                    if me != leader:
                        continue
                    nb = sum(self._payload_sizes(tuple(g.shape)))
                    if pending and size + nb > self.bucket:
                        sent += self._send(pending, leader, grp, targets)
                        pending, size = [], 0
                    pending.append((name, g))
                    size += nb
                if me == leader:
                    if pending:
                        sent += self._send(pending, leader, grp, targets)
                    self._send([], leader, grp, targets)  # end of this stage
                    continue
            if self.engine is not None and me != leader:
                while True:
                    got = self._recv(leader, grp, dev, targets)
                    if got < 0:
                        break
                    sent += got
        if self.engine is not None:
            if version is not None:
                self.engine.weight_version = version
            else:
                self.engine.weight_version += 1
            self.engine._fp8_version = None
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)
        self.last_stats = {"update_weights/bytes": sent, "perf/update_weights_time": time.perf_counter() - t0}
        return self.last_stats
