"""Host-resident batches through the layer with copies overlapped.

``HostPipeline`` runs ``fn(x_device, out_device)`` over batches that live in
pinned host memory: the host-to-device copy of batch i+1 and the
device-to-host copy of batch i-1 run on their own CUDA streams while batch i
computes (two device buffers each way; events order every reuse). Every
batch is copied in and read back in full; only the overlap differs from a
plain copy → compute → copy loop.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence

import torch
from torch import Tensor


class HostPipeline:
    def __init__(self, fn: Callable[[Tensor, Tensor], object], in_shape: Sequence[int], out_shape: Sequence[int],
                 dtype: torch.dtype, device: torch.device) -> None:
        self.fn = fn
        self.device = torch.device(device)
        self.x = [torch.empty(tuple(in_shape), dtype=dtype, device=self.device) for _ in range(2)]
        self.y = [torch.empty(tuple(out_shape), dtype=dtype, device=self.device) for _ in range(2)]
        self.copy_in = torch.cuda.Stream(self.device)
        self.copy_out = torch.cuda.Stream(self.device)
        self.loaded = [torch.cuda.Event() for _ in range(2)]
        self.computed = [torch.cuda.Event() for _ in range(2)]
        self.stored = [torch.cuda.Event() for _ in range(2)]
        self._used = [False, False]

    def run(self, host_in: Sequence[Tensor], host_out: Sequence[Tensor]) -> None:
        """host_out[i] = fn(host_in[i]) for every i; returns once all copies
        are enqueued (synchronize, or wait on ``self.stored``, before reading
        host_out)."""
        if len(host_in) != len(host_out):
            raise ValueError("host_in and host_out differ in length")
        compute = torch.cuda.current_stream(self.device)
        for i, (hi, ho) in enumerate(zip(host_in, host_out)):
            b = i & 1
            with torch.cuda.stream(self.copy_in):
                if self._used[b]:
                    self.copy_in.wait_event(self.computed[b])  # batch i-2 has read x[b]
                self.x[b].copy_(hi, non_blocking=True)
                self.loaded[b].record(self.copy_in)
            compute.wait_event(self.loaded[b])
            if self._used[b]:
                compute.wait_event(self.stored[b])  # batch i-2 has left y[b]
            self.fn(self.x[b], self.y[b])
            self.computed[b].record(compute)
            with torch.cuda.stream(self.copy_out):
                self.copy_out.wait_event(self.computed[b])
                ho.copy_(self.y[b], non_blocking=True)
                self.stored[b].record(self.copy_out)
            self._used[b] = True

    def last_event(self, n: int) -> torch.cuda.Event:
        """The event that completes with the copy-out of batch n - 1."""
        return self.stored[(n - 1) & 1]
