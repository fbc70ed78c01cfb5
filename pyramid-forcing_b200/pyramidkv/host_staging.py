"""Overlapped pinned-host staging for layer-steps whose Q/K/V live in host memory.

``MegaCache.update`` / ``MegaCache.attend`` take device tensors.  A caller whose
inputs arrive in host memory would otherwise copy them in, run the layer-step
and copy the output back, all on one stream, so the PCIe transfers and the
kernels take turns.  ``HostStaging`` keeps ``depth`` device copies of the
inputs and moves them on two side streams of its own:

* ``put(host_tensors)`` enqueues the host->device copies of a later
  layer-step on the copy-in stream, once the device slot it reuses has been
  released by the layer-step that last read it;
* ``get()`` returns the device tensors of the oldest ``put`` and makes the
  current stream wait for their copies;
* ``done(out, host_out)`` marks the slot of the last ``get`` free once the work
  already enqueued on the current stream has run, and enqueues the
  device->host copy of ``out`` on the copy-out stream.  It returns the event
  that completes with that copy: wait on it before reading ``host_out``.

With ``put`` of layer-step i+1 issued before layer-step i's kernels, the
host->device copies, the kernels and the device->host copies of neighbouring
layer-steps run at the same time.  Host tensors must be pinned for the copies to
be asynchronous.  This helper has no counterpart in the reference, whose
callers produce Q/K/V on the device.
"""
from __future__ import annotations

from typing import Sequence

import torch


class HostStaging:
    def __init__(self, like: Sequence[torch.Tensor], device, depth: int = 2):
        if depth < 1:
            raise ValueError("HostStaging: depth must be at least 1")
        self.device = torch.device(device)
        self.depth = depth
        self.slots = [[torch.empty(t.shape, dtype=t.dtype, device=self.device) for t in like]
                      for _ in range(depth)]
        self.copy_in = torch.cuda.Stream(self.device)
        self.copy_out = torch.cuda.Stream(self.device)
        self.ready = [torch.cuda.Event() for _ in range(depth)]
        self.free = [torch.cuda.Event() for _ in range(depth)]
        self.n_put = self.n_get = self.n_done = 0

    def put(self, host_tensors: Sequence[torch.Tensor]) -> None:
        if self.n_put - self.n_done >= self.depth:
            raise RuntimeError("HostStaging.put: all slots are in use; call done() first")
        slot = self.n_put % self.depth
        dst = self.slots[slot]
        if len(host_tensors) != len(dst):
            raise ValueError("HostStaging.put: expected %d tensors" % len(dst))
        # a slot's first use waits on an event never recorded: no wait
        self.copy_in.wait_event(self.free[slot])
        with torch.cuda.stream(self.copy_in):
            for d, h in zip(dst, host_tensors):
                d.copy_(h, non_blocking=True)
        self.ready[slot].record(self.copy_in)
        self.n_put += 1

    def get(self) -> list:
        if self.n_get >= self.n_put:
            raise RuntimeError("HostStaging.get: nothing was put")
        if self.n_get > self.n_done:
            raise RuntimeError("HostStaging.get: call done() for the previous get() first")
        slot = self.n_get % self.depth
        torch.cuda.current_stream(self.device).wait_event(self.ready[slot])
        self.n_get += 1
        return self.slots[slot]

    def done(self, out: torch.Tensor, host_out: torch.Tensor) -> torch.cuda.Event:
        if self.n_done >= self.n_get:
            raise RuntimeError("HostStaging.done: no get() to finish")
        slot = self.n_done % self.depth
        cur = torch.cuda.current_stream(self.device)
        self.free[slot].record(cur)
        self.copy_out.wait_event(self.free[slot])
        with torch.cuda.stream(self.copy_out):
            host_out.copy_(out, non_blocking=True)
        # the allocator must not hand out's memory to the current stream
        # before the copy-out stream has read it
        out.record_stream(self.copy_out)
        fin = torch.cuda.Event()
        fin.record(self.copy_out)
        self.n_done += 1
        return fin

    def synchronize(self) -> None:
        self.copy_in.synchronize()
        self.copy_out.synchronize()
