"""Trainer -> disaggregated rollout engine weight refit.

The trainer and every rollout engine hold the model in the same flat bf16 buffer layout (the
parameter order comes from `param_specs`), so a refit is a broadcast of that buffer, in buckets,
from one trainer rank to all engine ranks over NCCL; no per-parameter gather, rename or
re-layout happens. Modes:

  * "bf16": the flat buffer, bucket by bucket (`--update-weight-buffer-size` bytes each).
  * "fp8" : 2-D weights are block-quantised (128 x 128, e4m3 + fp32 scales) on the trainer,
            broadcast as fp8 + scales (about half the bytes) and dequantised into the engine's
            bf16 buffer; 1-D parameters (norms, biases) go as bf16. The engine then serves the
            fp8-rounded weights, as an fp8 rollout engine would.

After the broadcast every engine bumps its weight version to the trainer's.

Colocated engines need none of this: they read the trainer's buffer in place.

Reference: miles/backends/megatron_utils/update_weight/update_weight_from_distributed.py
(UpdateWeightFromDistributed), mixin.py:34-195 and broadcast.py:20-184 (bucketed NCCL
broadcast to engines), processors/quantizer_fp8.py (fp8 block quantisation at refit).
"""
from __future__ import annotations

import time

import torch
import torch.distributed as dist

from miles_b200.models.transformer import Transformer
from miles_b200.ops.quant import fp8_block_dequant, fp8_block_quant


class WeightRefit:
    def __init__(self, model: Transformer, group, src: int, bucket_bytes: int = 512 << 20,
                 mode: str = "bf16"):
        """group: process group holding the source trainer rank `src` (global rank) and every
        engine rank. Called with the same arguments on all of them."""
        if mode not in ("bf16", "fp8"):
            raise ValueError(f"unknown refit mode {mode}")
        self.model = model
        self.group = group
        self.src = src
        self.mode = mode
        self.bucket = max(1, bucket_bytes // model.flat.element_size())
        self.last_stats: dict = {}

    # ------------------------------------------------------------------ bf16: flat buckets
    def _broadcast_flat(self):
        flat = self.model.flat
        n = flat.numel()
        for a in range(0, n, self.bucket):
            dist.broadcast(flat[a:min(n, a + self.bucket)], self.src, group=self.group)
        return n * flat.element_size()

    # ------------------------------------------------------------------ fp8: per 2-D weight
    def _broadcast_fp8(self, is_src: bool):
        sent = 0
        dev = self.model.flat.device
        for s in self.model.specs:
            p = self.model.params[s.name].data
            if p.dim() == 2 and p.shape[0] >= 128 and p.shape[1] >= 128:
                w = p
            elif p.dim() == 3 and p.shape[1] >= 128 and p.shape[2] >= 128:
                w = p.reshape(-1, p.shape[2])  # stacked experts: blocks never straddle experts
            else:
                dist.broadcast(p, self.src, group=self.group)
                sent += p.numel() * p.element_size()
                continue
            M, N = w.shape
            if is_src:
                q, sc = fp8_block_quant(w)
            else:
                q = torch.empty(M, N, dtype=torch.float8_e4m3fn, device=dev)
                sc = torch.empty((M + 127) // 128, (N + 127) // 128, dtype=torch.float32, device=dev)
            dist.broadcast(q.view(torch.uint8), self.src, group=self.group)
            dist.broadcast(sc, self.src, group=self.group)
            sent += q.numel() + sc.numel() * 4
            if not is_src:
                w.copy_(fp8_block_dequant(q, sc, dtype=w.dtype))
        return sent

    # ------------------------------------------------------------------ API
    @torch.no_grad()
    def sync(self) -> dict:
        """Run the refit on this rank (source or engine). Returns timing / volume stats."""
        is_src = dist.get_rank() == self.src
        if self.model.flat.is_cuda:
            torch.cuda.synchronize(self.model.flat.device)
        t0 = time.perf_counter()
        nbytes = self._broadcast_flat() if self.mode == "bf16" else self._broadcast_fp8(is_src)
        ver = torch.tensor([self.model.weight_version], dtype=torch.int64, device=self.model.flat.device)
        dist.broadcast(ver, self.src, group=self.group)
        if self.model.flat.is_cuda:
            torch.cuda.synchronize(self.model.flat.device)
        dt = time.perf_counter() - t0
        if not is_src:
            self.model.weight_version = int(ver.item())
        self.last_stats = {"perf/update_weights_time": dt, "update_weights/bytes": nbytes,
                           "update_weights/GBps": nbytes / dt / 1e9 if dt > 0 else 0.0}
        return self.last_stats
