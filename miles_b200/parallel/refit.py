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
        fp8 = getattr(self.model, "fp8", {}) or {}
        self._filled = set()
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
                w8 = fp8.get(s.name)
                if w8 is not None and tuple(w8.q.shape) == (M, N):
                    # an engine serving block fp8: keep the trainer's e4m3 values and scales as
                    # they are (no dequantise / re-quantise round trip)
                    w8.q.copy_(q.view(torch.uint8))
                    w8.s.copy_(sc)
                    self._filled.add(s.name)
        return sent

    # ------------------------------------------------------------------ API
    @torch.no_grad()
    def sync(self) -> dict:
        """Run the refit on this rank (source or engine). Returns timing / volume stats."""
        is_src = dist.get_rank() == self.src
        cuda = self.model.flat.is_cuda
        if cuda:
            torch.cuda.synchronize(self.model.flat.device)
            dist.barrier(group=self.group)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        t0 = time.perf_counter()
        nbytes = self._broadcast_flat() if self.mode == "bf16" else self._broadcast_fp8(is_src)
        if cuda:
            e1.record()
        ver = torch.tensor([self.model.weight_version], dtype=torch.int64, device=self.model.flat.device)
        dist.broadcast(ver, self.src, group=self.group)
        if cuda:
            torch.cuda.synchronize(self.model.flat.device)
            # device time of the transfer, max over the group's ranks
            t = torch.tensor([e0.elapsed_time(e1) / 1e3], device=self.model.flat.device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
            dt = float(t)
        else:
            dt = time.perf_counter() - t0
        if not is_src:
            self.model.weight_version = int(ver.item())
            fp8 = getattr(self.model, "fp8", {}) or {}
            if self.mode == "fp8" and fp8 and set(fp8) <= getattr(self, "_filled", set()):
                self.model._fp8_version = self.model.weight_version  # copies already current
        self.last_stats = {"perf/update_weights_time": dt, "update_weights/bytes": nbytes,
                           "update_weights/GBps": nbytes / dt / 1e9 if dt > 0 else 0.0}
        return self.last_stats


# ---------------------------------------------------------------------------------------------
# Peer-memory refit (one node): the trainer's kernels store straight into the engines' staging
# buffers over NVLink, the engines pull from each other.
# ---------------------------------------------------------------------------------------------
class PeerRefit:
    """Same role and API as WeightRefit, over symmetric peer memory instead of NCCL broadcast.

    Every rank of `group` (the source trainer rank and the engine ranks, one node) maps an
    IPC-shared staging area of `bucket_bytes`. Parameters go in buckets; each parameter of a
    bucket has one owner engine (least-loaded first), so the source sends every byte once:

      1. source: for each parameter, the 128x128 block fp8 quantisation kernel reads the local
         bf16 weight and writes the fp8 values and scales straight into the owner engine's
         staging (quantise and transfer in one pass, half the bytes)
      2. device barrier over the group (flags in symmetric memory, bounded waits)
      3. every engine: for each parameter, the dequantisation kernel reads the owner's staging
         (its own or a peer's, over NVLink) and writes the local bf16 weight
      4. device barrier (the staging is reused by the next bucket)
    i.e. a scatter from the source followed by an all-gather among the engines, done by SM
    loads/stores inside the kernels. "bf16" needs no staging: the flat parameter buffers
    themselves are IPC-mapped, the source stores slice j of its buffer into engine j's buffer,
    and every engine loads the remaining slices from the others. A host barrier over the group first puts every rank in the
    refit, so the device barriers only wait for in-flight work.

    Reference: update_weight/update_weight_from_distributed.py + broadcast.py (bucketed NCCL
    broadcast) and update_weight_from_tensor.py (CUDA-IPC handles into colocated engines);
    processors/quantizer_fp8.py (fp8 block quantisation at refit).
    """

    def __init__(self, model: Transformer, group, src: int, bucket_bytes: int = 1 << 30,
                 mode: str = "bf16", timeout_s: float = 5.0):
        from miles_b200.parallel.symm import SymmBuffer

        if mode not in ("bf16", "fp8"):
            raise ValueError(f"unknown refit mode {mode}")
        self.model = model
        self.group = group
        self.src = src
        self.mode = mode
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.src_g = src if group is None else dist.get_group_rank(group, src)
        self.engines = [r for r in range(self.world) if r != self.src_g]
        self.cap = max(1 << 20, bucket_bytes // 16 * 16)
        self.buf = SymmBuffer(256 + self.cap, group, model.flat.device)
        self.flag_ptrs = list(self.buf.peers)
        self.stage = [p + 256 for p in self.buf.peers]
        self.my_flags = self.buf.view(0, (8,), torch.int32)
        self.ctl = torch.zeros(4, dtype=torch.int32, device=model.flat.device)
        self.timeout_ns = int(timeout_s * 1e9)
        self.plan = self._plan() if mode == "fp8" else []
        self.flat_ptrs: list[int] = []
        self._peer_flat = None
        if mode == "bf16":
            from miles_b200.parallel.symm import PeerTensor

            self._peer_flat = PeerTensor(model.flat, group)
            self.flat_ptrs = self._peer_flat.ptrs
        self.last_stats: dict = {}

    # ------------------------------------------------------------------ layout
    @staticmethod
    def _pad(n: int) -> int:
        return _pad256(n)

    def _items(self):
        return refit_units(self.model, self.mode, self.cap)

    def _plan(self):
        return refit_buckets(self._items(), self.engines, self.cap)

    def _view2d(self, name: str) -> torch.Tensor:
        p = self.model.params[name].data
        return p if p.dim() == 2 else p.reshape(-1, p.shape[-1])

    # ------------------------------------------------------------------ transfer
    def _barrier(self):
        from miles_b200.ops._lib import err_word, lib

        lib().symm_barrier(self.flag_ptrs, self.my_flags, self.ctl, self.rank, self.world,
                           self.timeout_ns, err_word(self.model.flat.device))

    def _send(self, bucket):
        from miles_b200.ops._lib import lib

        C = lib()
        sent = 0
        for name, kind, lo, hi, owner, off in bucket:
            dst = self.stage[owner] + off
            if kind == "fp8":
                w = self._view2d(name)[lo:hi]
                M, N = w.shape
                C.fp8_block_cast_ptr(w, 128, 128, dst, dst + self._pad(M * N), False)
                sent += M * N + ((M + 127) // 128) * ((N + 127) // 128) * 4
            else:
                self._copy(self.model.params[name].data_ptr() + lo, dst, hi - lo)
                sent += hi - lo
        return sent

    def _recv(self, bucket):
        from miles_b200.ops._lib import lib

        C = lib()
        for name, kind, lo, hi, owner, off in bucket:
            src = self.stage[owner] + off
            if kind == "fp8":
                w = self._view2d(name)[lo:hi]
                C.fp8_block_dequant_ptr(src, src + self._pad(w.shape[0] * w.shape[1]), 128, 128, w)
            else:
                self._copy(src, self.model.params[name].data_ptr() + lo, hi - lo)

    @staticmethod
    def _copy(src: int, dst: int, nb: int):
        from miles_b200.ops._lib import lib

        body = nb // 16 * 16
        if body:
            lib().symm_copy_ptr(src, dst, body)
        if nb > body:  # ragged tail (never for 256-byte aligned bf16 tensors of even size)
            t_src = _raw_bytes(src + body, nb - body)
            t_dst = _raw_bytes(dst + body, nb - body)
            t_dst.copy_(t_src)

    # ------------------------------------------------------------------ bf16: direct
    def _direct_bf16(self, is_src: bool) -> int:
        """bf16: no staging at all. The flat parameter buffers are IPC-mapped; the source stores
        slice j of its buffer straight into engine j's buffer, then every engine loads the other
        slices from the engine that received them."""
        flat = self.model.flat
        nb = flat.numel() * flat.element_size()
        E = len(self.engines)
        step = (nb // E + 255) // 256 * 256
        slices = [(j * step, min(nb, (j + 1) * step)) for j in range(E)]
        if is_src:
            for j, e in enumerate(self.engines):
                lo, hi = slices[j]
                if hi > lo:
                    self._copy(self.flat_ptrs[self.src_g] + lo, self.flat_ptrs[e] + lo, hi - lo)
        self._barrier()
        if not is_src:
            for j, e in enumerate(self.engines):
                lo, hi = slices[j]
                if e != self.rank and hi > lo:
                    self._copy(self.flat_ptrs[e] + lo, self.flat_ptrs[self.rank] + lo, hi - lo)
        self._barrier()
        return nb

    @torch.no_grad()
    def sync(self) -> dict:
        is_src = self.rank == self.src_g
        dev = self.model.flat.device
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)  # everyone is in the refit before any device wait
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        nbytes = 0
        if self.mode == "bf16":
            nbytes = self._direct_bf16(is_src)
        else:
            for bucket in self.plan:
                if is_src:
                    nbytes += self._send(bucket)
                self._barrier()
                if not is_src:
                    self._recv(bucket)
                self._barrier()
        e1.record()
        ver = torch.tensor([self.model.weight_version], dtype=torch.int64, device=dev)
        dist.broadcast(ver, self.src, group=self.group)
        torch.cuda.synchronize(dev)
        from miles_b200.ops._lib import check_device_error

        check_device_error(dev)
        dt = e0.elapsed_time(e1) / 1e3
        t = torch.tensor([dt], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)  # device time, max over ranks
        dt = float(t)
        nb = torch.tensor([nbytes], dtype=torch.float64, device=dev)
        dist.broadcast(nb, self.src, group=self.group)
        nbytes = int(nb)
        if not is_src:
            self.model.weight_version = int(ver.item())
            fp8 = getattr(self.model, "fp8", {}) or {}
            if self.mode == "fp8" and fp8 and set(fp8) <= getattr(self, "_filled", set()):
                self.model._fp8_version = self.model.weight_version  # copies already current
        self.last_stats = {"perf/update_weights_time": dt, "update_weights/bytes": nbytes,
                           "update_weights/GBps": nbytes / dt / 1e9 if dt > 0 else 0.0}
        return self.last_stats

    def close(self):
        torch.cuda.synchronize(self.model.flat.device)
        dist.barrier(group=self.group)
        if self._peer_flat is not None:
            self._peer_flat.close()
        self.buf.close()


def _raw_bytes(ptr: int, n: int) -> torch.Tensor:
    from miles_b200.ops import _lib

    return _lib._C.from_ptr(ptr, [n], torch.uint8, torch.cuda.current_device())


def _pad256(n: int) -> int:
    return (n + 255) // 256 * 256


def refit_units(model, mode: str, cap: int):
    """Transfer units (name, kind, lo, hi, staging bytes) of a peer refit: kind "fp8" moves rows
    [lo, hi) of a 2-D weight view (multiples of 128 rows, so quantisation blocks never straddle
    units), kind "copy" moves bytes [lo, hi) of the parameter. No unit exceeds `cap` bytes."""
    out = []
    for s in model.specs:
        p = model.params[s.name].data
        w = None
        if mode == "fp8":
            if p.dim() == 2 and p.shape[0] >= 128 and p.shape[1] >= 128 and p.shape[1] % 16 == 0:
                w = p
            elif p.dim() == 3 and p.shape[1] >= 128 and p.shape[2] >= 128 and p.shape[2] % 16 == 0:
                w = p.reshape(-1, p.shape[2])
        if w is not None:
            M, N = w.shape
            gn = (N + 127) // 128
            per_blk = _pad256(128 * N) + _pad256(gn * 4)  # upper bound per 128 rows
            step = max(1, cap // per_blk) * 128
            for r0 in range(0, M, step):
                r1 = min(M, r0 + step)
                rows = r1 - r0
                nb = _pad256(rows * N) + _pad256(((rows + 127) // 128) * gn * 4)
                out.append((s.name, "fp8", r0, r1, nb))
        else:
            total = p.numel() * p.element_size()
            step = cap // 256 * 256
            for b0 in range(0, total, step):
                b1 = min(total, b0 + step)
                out.append((s.name, "copy", b0, b1, _pad256(b1 - b0)))
    return out


def refit_buckets(units, engines: list[int], cap: int):
    """Buckets of (name, kind, lo, hi, owner engine, staging offset): each unit goes to the
    least-loaded engine of the current bucket; a bucket closes when a unit no longer fits."""
    buckets, cur, used = [], [], {e: 0 for e in engines}
    for name, kind, lo, hi, nb in units:
        if nb > cap:
            raise ValueError(f"{name}: one 128-row block needs {nb} staging bytes > {cap}")
        owner = min(engines, key=lambda e: used[e])
        if used[owner] + nb > cap:
            buckets.append(cur)
            cur, used = [], {e: 0 for e in engines}
            owner = engines[0]
        cur.append((name, kind, lo, hi, owner, used[owner]))
        used[owner] += nb
    if cur:
        buckets.append(cur)
    return buckets


def make_refit(model: Transformer, group, src: int, bucket_bytes: int, mode: str,
               transport: str = "auto"):
    """WeightRefit (NCCL broadcast) or PeerRefit (symmetric peer memory). "auto" picks the
    peer transport when every rank of the group is a CUDA process of an NCCL job."""
    if transport == "auto":
        transport = "peer" if (model.flat.is_cuda and dist.get_backend(group) == "nccl") else "nccl"
    if transport == "peer":
        return PeerRefit(model, group, src, bucket_bytes, mode)
    return WeightRefit(model, group, src, bucket_bytes, mode)


def verify_weights_equal(model, group, src: int, exact: bool = True) -> dict:
    """--check-weight-update-equal: after a refit every member of `group` (the source trainer
    and the engines) reduces its flat parameter buffer to a checksum (the bf16 bit patterns
    summed as integers, so equal bits give equal sums); with `exact` (bf16 refit) every engine
    must match the source, otherwise (fp8 refit: engines hold dequantised weights) the engines
    must match each other. Raises AssertionError on a mismatch; every member must call it."""
    flat = model.flat
    csum = flat.view(torch.int16).to(torch.int64).sum().reshape(1)
    world = dist.get_world_size(group)
    got = [torch.zeros_like(csum) for _ in range(world)]
    dist.all_gather(got, csum, group=group)
    vals = [int(g.item()) for g in got]
    ranks = dist.get_process_group_ranks(group) if hasattr(dist, "get_process_group_ranks") else list(range(world))
    src_i = ranks.index(src) if src in ranks else 0
    engines = [v for i, v in enumerate(vals) if i != src_i]
    if exact and any(v != vals[src_i] for v in engines):
        raise AssertionError(f"engine weights differ from the trainer's after refit: {vals}")
    if not exact and len(set(engines)) > 1:
        raise AssertionError(f"engine weights differ from each other after refit: {vals}")
    return {"update_weights/checksum": vals[src_i]}
