"""Symmetric peer memory and the fused collectives built on it (csrc/symm.cu).

`SymmComm(group)` allocates, on every rank of a process group, one device region holding

    flags   int32[8]                       (peers announce epochs here)
    staging bf16 [2][world][cap][hidden]   (double-buffered partials, one slot per source rank)

and exchanges the regions' CUDA IPC handles over the group, so each rank holds device
pointers to every peer's region. On top of it:

  * ``all_reduce(x)``                  one-shot all-reduce: push x into every peer's slot, then
                                       sum the slots in rank order (bitwise identical on all
                                       ranks, deterministic across calls)
  * ``all_reduce_add_norm(x, res, w)`` the same fused with the residual add and RMSNorm that
                                       follow a row-parallel projection
  * ``gemm_all_reduce(a, w)``          fused GEMM + all-reduce: the tcgen05 GEMM's epilogue stores
                                       each output tile straight into every peer's staging slot
                                       over NVLink (no local output, no copy), the reduce kernel
                                       then sums the slots; with ``norm_w`` the reduce also does
                                       the residual add + RMSNorm
  * ``barrier()``                      device-side barrier (flags only)

The epoch counter that sequences calls lives on the device, so all of these can be captured in
CUDA graphs (the rollout engine's decode step). Every wait in the kernels is bounded
(``timeout_s``); a timed-out wait sets the device error word (code 3) instead of hanging, which
`miles_b200.ops.check_device_error` raises on the host.

Reference: the NCCL all-reduces after Megatron's row-parallel layers and SGLang's custom
all-reduce for TP decode (the reference ships both as library code); there is no fused
GEMM + collective in the reference.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from miles_b200.ops import _lib
from miles_b200.ops._lib import err_word, lib

FLAG_BYTES = 256


def _raw():
    if _lib._C is None:
        raise RuntimeError(f"miles_b200._C is not built: {_lib._IMPORT_ERROR!r}")
    return _lib._C


class SymmBuffer:
    """One raw device allocation per rank, IPC-mapped on every other rank of `group`."""

    def __init__(self, nbytes: int, group=None, device: torch.device | None = None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.nbytes = nbytes
        C = _raw()
        self.ptr = C.symm_malloc(nbytes, self.device.index)
        handle = C.ipc_get_handle(self.ptr)
        handles: list = [None] * self.world
        dist.all_gather_object(handles, bytes(handle.numpy().tobytes()), group=group)
        self.peers: list[int] = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.peers.append(self.ptr)
            else:
                t = torch.frombuffer(bytearray(h), dtype=torch.uint8)
                self.peers.append(C.ipc_open(t, self.device.index))
        self._closed = False

    def view(self, offset: int, shape, dtype, rank: int | None = None) -> torch.Tensor:
        """Tensor view of [offset, offset + numel * itemsize) of this rank's (or a peer's) copy."""
        base = self.ptr if rank is None else self.peers[rank]
        return _raw().from_ptr(base + offset, list(shape), dtype, self.device.index)

    def close(self):
        if self._closed:
            return
        C = _raw()
        for r, p in enumerate(self.peers):
            if r != self.rank:
                C.ipc_close(p)
        C.symm_free(self.ptr)
        self._closed = True


class PeerTensor:
    """Device pointers to every rank's copy of a tensor allocated by torch (e.g. a model's flat
    parameter buffer): the storage's CUDA IPC handle and byte offset are exchanged over `group`
    and opened on every other rank."""

    def __init__(self, t: torch.Tensor, group=None):
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        h, off = _raw().ipc_get_handle_range(t.data_ptr())
        handle = bytes(h.numpy().tobytes())
        items: list = [None] * self.world
        dist.all_gather_object(items, (handle, off), group=group)
        C = _raw()
        self._bases: list[int] = []
        self.ptrs: list[int] = []
        for r, (h, o) in enumerate(items):
            if r == self.rank:
                self.ptrs.append(t.data_ptr())
            else:
                base = C.ipc_open(torch.frombuffer(bytearray(h), dtype=torch.uint8), t.device.index)
                self._bases.append(base)
                self.ptrs.append(base + o)

    def close(self):
        C = _raw()
        for b in self._bases:
            C.ipc_close(b)
        self._bases = []


class PeerGradBuffer:
    """The flat bf16 gradient buffer of a data-parallel group in symmetric memory, and the fused
    reduce-scatter over it (csrc/symm.cu grad_rs_kernel): each rank reads its shard of every
    peer's gradient straight over NVLink, sums in rank order in fp32, scales, rounds to bf16
    into its own copy and produces the shard's squared norm, in one kernel. The buffer is
    allocated once (cudaMalloc + IPC handles exchanged once) and stays resident, so a step
    pays no handle exchange.

    Replaces the NCCL reduce-scatter of Megatron's distributed optimizer (reference:
    megatron_utils/model.py:537-612) for the DP gradient."""

    def __init__(self, numel: int, group=None, device: torch.device | None = None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("PeerGradBuffer supports up to 8 ranks (one NVSwitch domain)")
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.numel = numel
        self.buf = SymmBuffer(max(16, (numel * 2 + 15) // 16 * 16), group, self.device)
        self.tensor = self.buf.view(0, (numel,), torch.bfloat16)
        self.partial = torch.zeros(148 * 4, dtype=torch.float32, device=self.device)
        self.counter = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._token = torch.zeros(1, dtype=torch.float32, device=self.device)

    def reduce_scatter(self, lo: int, n: int, sq: torch.Tensor, scale: float = 1.0) -> None:
        """tensor[lo, lo + n) = bf16(scale * sum over ranks), sq[0] = its squared norm. Every
        rank's backward must be complete before any rank reads: a one-element all-reduce on
        the stream orders the kernel after every rank's earlier work. The caller must not
        write the buffer again before every rank's call has finished (the optimizer's
        parameter all-gather that follows is such a point)."""
        if lo % 8 or n % 8:
            raise ValueError(f"fused gradient reduce-scatter needs 8-aligned shards (lo={lo}, n={n})")
        if self.world > 1:
            dist.all_reduce(self._token, group=self.group)
        rc = lib().grad_rs(self.buf.peers, lo, n, scale, self.tensor[lo:lo + n], self.partial,
                           self.counter, sq)
        if rc != 0:
            raise RuntimeError(f"grad_rs launch failed ({rc})")

    def close(self):
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self.buf.close()


class SymmComm:
    def __init__(self, group=None, hidden: int = 4096, cap_rows: int = 256,
                 device: torch.device | None = None, timeout_s: float = 2.0):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("SymmComm supports up to 8 ranks (one NVSwitch domain)")
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.hidden = hidden
        self.cap = cap_rows
        self.slot_elems = cap_rows * hidden
        stage_bytes = 2 * self.world * self.slot_elems * 2
        self.buf = SymmBuffer(FLAG_BYTES + stage_bytes, group, self.device)
        self.flag_ptrs = list(self.buf.peers)
        self.stage_ptrs = [p + FLAG_BYTES for p in self.buf.peers]
        self.my_flags = self.buf.view(0, (8,), torch.int32)
        self.my_stage = self.buf.view(FLAG_BYTES, (2 * self.world * self.slot_elems,), torch.bfloat16)
        # {epoch, done, arrived, pad}: advanced on the device by the last CTA of every call
        self.ctl = torch.zeros(4, dtype=torch.int32, device=self.device)
        self.timeout_ns = int(timeout_s * 1e9)
        self.err = err_word(self.device)
        # GEMM epilogue destinations: this rank's slot in every peer's staging
        self.gemm_dst = [p + self.rank * self.slot_elems * 2 for p in self.stage_ptrs]
        self.calls = 0
        dist.barrier(group=group)

    def _check(self, rows: int, H: int):
        if H != self.hidden or rows > self.cap:
            raise ValueError(f"SymmComm sized for [{self.cap}, {self.hidden}], got [{rows}, {H}]")

    def barrier(self):
        lib().symm_barrier(self.flag_ptrs, self.my_flags, self.ctl, self.rank, self.world,
                           self.timeout_ns, self.err)

    def _reduce(self, src, rows, H, res, norm_w, eps, out, h_out, rstd):
        lib().symm_allreduce(self.flag_ptrs, self.stage_ptrs, self.my_flags, self.ctl,
                             self.my_stage, self.cap, src, rows, H, self.rank, self.world, res,
                             norm_w, eps, out, h_out, rstd, self.timeout_ns, self.err)
        self.calls += 1

    def all_reduce(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        rows, H = x.shape
        self._check(rows, H)
        x = x.contiguous()
        out = torch.empty_like(x) if out is None else out
        self._reduce(x, rows, H, None, None, 0.0, out, None, None)
        return out

    def all_reduce_add_norm(self, x, res, norm_w, eps: float):
        """(y, h): h = allreduce(x) + res, y = rmsnorm(h) * norm_w (res None: h = allreduce(x))."""
        rows, H = x.shape
        self._check(rows, H)
        y = torch.empty_like(x)
        h = torch.empty_like(x) if res is not None else None
        self._reduce(x.contiguous(), rows, H, res, norm_w, eps, y, h, None)
        return y, (h if res is not None else None)

    def gemm_all_reduce(self, a: torch.Tensor, w: torch.Tensor, res=None, norm_w=None,
                        eps: float = 0.0, w_mn: bool = False):
        """allreduce(a @ w^T) (w_mn: allreduce(a @ w)) with the GEMM storing its tiles into the
        peers' staging. With norm_w returns (y, h) as all_reduce_add_norm, else the sum."""
        from miles_b200.ops.gemm import _pick_bn

        M, K = a.shape
        N = w.shape[1] if w_mn else w.shape[0]
        self._check(M, N)
        a = a.contiguous()
        bn = _pick_bn(M, N, a.device, narrow=not w_mn)
        lib().gemm_peer(a, w, w_mn, M, N, K, self.gemm_dst, N, self.ctl,
                        self.world * self.slot_elems, 0, bn, self.err)
        out = torch.empty(M, N, dtype=torch.bfloat16, device=a.device)
        if norm_w is None:
            self._reduce(None, M, N, None, None, 0.0, out, None, None)
            return out
        h = torch.empty_like(out) if res is not None else None
        self._reduce(None, M, N, res, norm_w, eps, out, h, None)
        return out, h

    # ------------------------------------------------------------------ sequence parallel
    def _coll(self, kind, src, rows, H, res, norm_w, eps, out, h_out, rstd):
        lib().symm_collective(kind, self.flag_ptrs, self.stage_ptrs, self.my_flags, self.ctl,
                              self.my_stage, self.cap, src, rows, H, self.rank, self.world, res,
                              norm_w, eps, out, h_out, rstd, self.timeout_ns, self.err)
        self.calls += 1

    def reduce_scatter(self, x: torch.Tensor, res=None, norm_w=None, eps: float = 0.0,
                       rstd: torch.Tensor | None = None):
        """Row block `rank` of sum_r x_r ([rows/world, H]); with norm_w returns (y, h) of the
        fused residual + RMSNorm on that block."""
        rows, H = x.shape
        R = rows // self.world
        if R * self.world != rows:
            raise ValueError(f"{rows} rows do not split over {self.world} ranks")
        self._check(R, H)
        out = torch.empty(R, H, dtype=x.dtype, device=x.device)
        if norm_w is None:
            self._coll(1, x.contiguous(), R, H, None, None, 0.0, out, None, None)
            return out
        h = torch.empty_like(out) if res is not None else None
        self._coll(1, x.contiguous(), R, H, res, norm_w, eps, out, h, rstd)
        return out, h

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        """Rows of every rank in rank order ([world * rows, H])."""
        rows, H = x.shape
        self._check(rows, H)
        out = torch.empty(self.world * rows, H, dtype=x.dtype, device=x.device)
        self._coll(2, x.contiguous(), rows, H, None, None, 0.0, out, None, None)
        return out

    def gemm_reduce_scatter(self, a: torch.Tensor, w: torch.Tensor, w_mn: bool = False):
        """Row block `rank` of sum_r (a_r @ w_r^T): the GEMM epilogue stores every output row only
        into its owner's staging (each element crosses NVLink once), the reduce kernel sums."""
        from miles_b200.ops.gemm import _pick_bn

        M, K = a.shape
        N = w.shape[1] if w_mn else w.shape[0]
        R = M // self.world
        if R * self.world != M:
            raise ValueError(f"{M} rows do not split over {self.world} ranks")
        self._check(R, N)
        a = a.contiguous()
        bn = _pick_bn(M, N, a.device, narrow=not w_mn)
        lib().gemm_peer(a, w, w_mn, M, N, K, self.gemm_dst, N, self.ctl,
                        self.world * self.slot_elems, R, bn, self.err)
        out = torch.empty(R, N, dtype=torch.bfloat16, device=a.device)
        self._coll(1, None, R, N, None, None, 0.0, out, None, None)
        return out

    def close(self):
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self.buf.close()
