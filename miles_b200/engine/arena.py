"""Fixed-address device memory for the rollout engine's KV cache (csrc/vmm.cu).

`DeviceArena(nbytes, device)` reserves a device virtual address range once; `map()` backs it
with physical memory and returns a flat uint8 tensor over it, `unmap()` frees the physical
memory and keeps the range. Every `map()` returns the same addresses, so CUDA graphs that
captured kernels reading the cache stay valid across the colocated release (training) /
resume (rollout) cycle. This is the role of torch_memory_saver's pause / resume in the
reference, which releases the inference engine's KV cache around training.
"""
from __future__ import annotations

import torch

from miles_b200.ops._lib import KernelLaunchError, lib


class DeviceArena:
    def __init__(self, nbytes: int, device: torch.device):
        self.device = torch.device(device)
        idx = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.index = idx
        rc, gran = lib()._mod.vmm_granularity(idx)
        if rc:
            raise KernelLaunchError(f"vmm_granularity failed with status {rc}")
        self.nbytes = (nbytes + gran - 1) // gran * gran
        rc, self.ptr = lib()._mod.vmm_reserve(self.nbytes)
        if rc:
            raise KernelLaunchError(f"vmm_reserve of {self.nbytes} bytes failed with status {rc}")
        self.handle = None

    @property
    def mapped(self) -> bool:
        return self.handle is not None

    def map(self) -> torch.Tensor:
        """Back the range with physical memory; returns the flat uint8 view (same address on
        every call). Raises torch.OutOfMemoryError if the device cannot supply it."""
        if self.handle is None:
            torch.cuda.synchronize(self.device)
            rc, h = lib()._mod.vmm_map(self.ptr, self.nbytes, self.index)
            if rc == -3:
                raise torch.OutOfMemoryError(f"cannot map {self.nbytes / 2**30:.1f} GiB for the KV arena")
            if rc:
                raise KernelLaunchError(f"vmm_map failed with status {rc}")
            self.handle = h
        return lib()._mod.vmm_tensor(self.ptr, self.nbytes, torch.uint8, self.index)

    def unmap(self) -> None:
        """Free the physical memory (the caller drops every view first); the device is
        synchronised so no kernel still reads the range."""
        if self.handle is None:
            return
        torch.cuda.synchronize(self.device)
        rc = lib()._mod.vmm_unmap(self.ptr, self.nbytes, self.handle)
        if rc:
            raise KernelLaunchError(f"vmm_unmap failed with status {rc}")
        self.handle = None

    def close(self) -> None:
        self.unmap()
        if self.ptr:
            lib()._mod.vmm_free(self.ptr, self.nbytes)
            self.ptr = 0
