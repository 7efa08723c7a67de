"""Data-parallel gradient exchange: per-layer buckets all-reduced while the
reverse sweep continues.

The reference trains on one device (train_baseline.py:233 hard-codes
data_parallel_world_size 1). Here each rank runs its own microsteps over its
slice of the update window (data.update_batches) and gradients are summed with
all_reduce(SUM) — every rank already divides its loss by the global target
count, so the sum is the global-batch gradient.

GradBuckets holds contiguous slices of the flat gradient buffer. `launch(i)`
is called when bucket i's gradients are final (the trainer calls it as the
last microstep's reverse sweep finishes each layer); on CUDA it orders the
collective after the compute stream's current work with an event and issues
it on a communication stream, so the exchange overlaps the remaining layers.
`finish()` makes the compute stream wait for every launched exchange. On CPU
(gloo) the same calls run the collectives asynchronously and wait for them.
Every rank launches the same buckets in the same order.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class GradBuckets:
    def __init__(self, slices, group=None, device: torch.device | None = None):
        self.slices = list(slices)
        self.group = group
        self.cuda = device is not None and device.type == "cuda"
        self.comm = torch.cuda.Stream(device=device) if self.cuda else None
        self.pending = []
        self.launched = []

    def launch(self, i: int, after=None):
        """All-reduces bucket i after the compute stream's current work, or after
        the given CUDA events (the streams that produced the bucket)."""
        t = self.slices[i]
        self.launched.append(i)
        if self.cuda:
            if after is None:
                ev = torch.cuda.Event()
                ev.record(torch.cuda.current_stream(t.device))
                after = [ev]
            for ev in after:
                self.comm.wait_event(ev)
            with torch.cuda.stream(self.comm):
                dist.all_reduce(t, group=self.group)
        else:
            self.pending.append(dist.all_reduce(t, group=self.group, async_op=True))

    def launch_all(self, order=None):
        for i in (order if order is not None else range(len(self.slices))):
            self.launch(i)

    def finish(self):
        if self.cuda:
            torch.cuda.current_stream(self.slices[0].device).wait_stream(self.comm)
        else:
            for work in self.pending:
                work.wait()
            self.pending.clear()
        order, self.launched = self.launched, []
        return order
