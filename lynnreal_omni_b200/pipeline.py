"""Host-resident batches through the W8A8 block with copies overlapped.

``HostPipeline`` runs a device function over a sequence of batches that live in
pinned host memory: while step i computes on the default stream, the input of
step i+1 is copied host->device on one copy stream and the result of step i-1
device->host on another (B200 has separate copy engines per direction). Every
step still moves its full input and output across PCIe; only the ordering
overlaps. Two device buffers per input alternate between steps.
"""
from __future__ import annotations

from typing import Callable, Sequence

import torch


class HostPipeline:
    def __init__(self, fn: Callable[..., torch.Tensor], device: torch.device,
                 input_templates: Sequence[torch.Tensor]):
        """fn(*device_inputs) -> device output tensor; input_templates give the
        shapes/dtypes of the per-step host inputs."""
        self.fn = fn
        self.device = device
        self.buffers = [[torch.empty(t.shape, dtype=t.dtype, device=device) for t in input_templates]
                        for _ in range(2)]
        self.h2d = torch.cuda.Stream(device)
        self.d2h = torch.cuda.Stream(device)
        self.loaded = [torch.cuda.Event() for _ in range(2)]
        self.consumed = [torch.cuda.Event() for _ in range(2)]
        self.produced = [torch.cuda.Event() for _ in range(2)]

    def _load(self, slot: int, host_inputs: Sequence[torch.Tensor]) -> None:
        with torch.cuda.stream(self.h2d):
            self.h2d.wait_event(self.consumed[slot])  # the step that last read this slot is done
            for dst, src in zip(self.buffers[slot], host_inputs):
                dst.copy_(src, non_blocking=True)
            self.loaded[slot].record(self.h2d)

    def run(self, host_inputs: Sequence[Sequence[torch.Tensor]], host_outputs: Sequence[torch.Tensor]):
        """host_inputs[i]: pinned input tensors of step i; host_outputs[i]: pinned
        tensor receiving step i's result. Returns after enqueueing all work."""
        compute = torch.cuda.current_stream(self.device)
        steps = len(host_inputs)
        for e in self.consumed:
            e.record(compute)
        if steps:
            self._load(0, host_inputs[0])
        for i in range(steps):
            slot = i & 1
            if i + 1 < steps:
                self._load(slot ^ 1, host_inputs[i + 1])
            compute.wait_event(self.loaded[slot])
            out = self.fn(*self.buffers[slot])
            self.consumed[slot].record(compute)
            self.produced[slot].record(compute)
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(self.produced[slot])
                host_outputs[i].copy_(out, non_blocking=True)
                out.record_stream(self.d2h)
        compute.wait_stream(self.d2h)
        compute.wait_stream(self.h2d)
