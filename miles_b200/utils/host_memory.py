"""Host buffers pinned in the background.

`BackgroundPinned(numel, dtype, chunk_bytes)` returns a CPU tensor at once and, on a worker
thread, zero-fills and page-locks it range by range (cudaHostRegister). Call `wait()` before the
first use (the contents are zero only after it). Page-locking 2 x 61 GB of Adam state with one
cudaHostAlloc each took about a minute before the first optimizer step; started when the actor
is built, this runs under the first rollout instead.
"""
from __future__ import annotations

import threading

import torch


class BackgroundPinned:
    def __init__(self, numel: int, dtype: torch.dtype, chunk_bytes: int = 1 << 29):
        # page-aligned start, so the registered ranges (multiples of the page size) never share
        # a page (a second registration of a page fails)
        es = torch.empty((), dtype=dtype).element_size()
        self._raw = torch.empty(numel * es + 4096, dtype=torch.uint8)
        off = (-self._raw.data_ptr()) % 4096
        self.tensor = self._raw[off:off + numel * es].view(dtype)
        self.chunk_bytes = chunk_bytes
        self.registered: list[int] = []   # byte offsets of registered ranges
        self._stop = False
        self.thread = None
        if torch.cuda.is_available() and numel:
            self.thread = threading.Thread(target=self._pin, daemon=True)
            self.thread.start()
        else:
            self.tensor.zero_()

    def _pin(self):
        from miles_b200.ops._lib import lib

        mod = lib()._mod
        es = self.tensor.element_size()
        total = self.tensor.numel() * es
        flat = self.tensor.view(-1)
        for off in range(0, total, self.chunk_bytes):
            n = min(self.chunk_bytes, total - off)
            flat[off // es:(off + n) // es].zero_()
            if self._stop:
                continue
            if mod.host_register(self.tensor, off, n) == 0:
                self.registered.append(off)

    def wait(self):
        if self.thread is not None:
            self.thread.join()

    def release(self):
        """Unregister every range (before the tensor is freed)."""
        self._stop = True
        self.wait()
        if self.registered:
            from miles_b200.ops._lib import lib

            for off in self.registered:
                lib()._mod.host_unregister(self.tensor, off)
            self.registered = []
