"""Host-buffer streaming for a device layer: batches arrive in pinned host
memory and results go back to pinned host memory, with the copies of one
batch overlapped with the compute of its neighbours.

Three CUDA streams: host->device copies, compute, device->host copies.
`depth` device slots hold the inputs and outputs of batches in flight, so
while batch i computes, batch i+1's input is copied in and batch i-1's
result is copied out (PCIe/C2C copy engines run both directions at once).
Events order the three streams; the host never blocks inside `submit`.
"""
from __future__ import annotations

import torch


class HostPipeline:
    """Run `layer(x, out=...)` on host batches [T <= max_tokens, width] bf16.

    submit(x_host, out_host) enqueues one batch (both pinned, contiguous) and
    returns the event that marks its result copied to out_host; synchronize()
    waits for every submitted batch.
    """

    def __init__(self, layer, max_tokens: int, width: int, depth: int = 2,
                 device: torch.device | None = None):
        if depth < 1:
            raise ValueError("depth must be >= 1")
        self.layer, self.depth = layer, depth
        dev = device or torch.device("cuda", torch.cuda.current_device())
        self.h2d = torch.cuda.Stream(dev)
        self.compute = torch.cuda.Stream(dev)
        self.d2h = torch.cuda.Stream(dev)
        self.x = [torch.empty((max_tokens, width), dtype=torch.bfloat16, device=dev)
                  for _ in range(depth)]
        self.y = [torch.empty((max_tokens, width), dtype=torch.bfloat16, device=dev)
                  for _ in range(depth)]
        self.in_ready = [torch.cuda.Event() for _ in range(depth)]
        self.in_free = [None] * depth      # compute finished reading x[slot]
        self.out_ready = [torch.cuda.Event() for _ in range(depth)]
        self.out_free = [None] * depth     # d2h finished reading y[slot]
        self.count = 0
        self.last_done: torch.cuda.Event | None = None
        self.max_tokens, self.width = max_tokens, width

    def submit(self, x_host: torch.Tensor, out_host: torch.Tensor) -> torch.cuda.Event:
        T = x_host.shape[0]
        if (x_host.is_cuda or out_host.is_cuda or x_host.shape != out_host.shape
                or T > self.max_tokens or x_host.shape[1] != self.width
                or x_host.dtype != torch.bfloat16 or out_host.dtype != torch.bfloat16):
            raise ValueError("x_host and out_host must be host bf16 [T <= max_tokens, width]")
        if not (x_host.is_pinned() and out_host.is_pinned()):
            raise ValueError("host buffers must be pinned (torch.Tensor.pin_memory())")
        b = self.count % self.depth
        self.count += 1
        xd, yd = self.x[b][:T], self.y[b][:T]
        with torch.cuda.stream(self.h2d):
            if self.in_free[b] is not None:
                self.h2d.wait_event(self.in_free[b])
            xd.copy_(x_host, non_blocking=True)
            self.in_ready[b].record(self.h2d)
        with torch.cuda.stream(self.compute):
            self.compute.wait_event(self.in_ready[b])
            if self.out_free[b] is not None:
                self.compute.wait_event(self.out_free[b])
            self.layer(xd, out=yd)
            ev = torch.cuda.Event()
            ev.record(self.compute)
            self.in_free[b] = ev
            self.out_ready[b].record(self.compute)
        with torch.cuda.stream(self.d2h):
            self.d2h.wait_event(self.out_ready[b])
            out_host.copy_(yd, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self.d2h)
            self.out_free[b] = ev
            self.last_done = ev
        return ev

    def synchronize(self) -> None:
        if self.last_done is not None:
            self.last_done.synchronize()
