"""Host-resident inputs through an `AttentionFn` with the copies overlapped.

The reference calls its attention functions on device tensors inside the
DiT (`h3/model.py:375`). A caller whose q, k, v live in host memory (an
offloaded pipeline, a serving front end) pays the PCIe copies on top: for
one config-2 layer 660 MB in and 220 MB out, about eight times the
attention itself. `HostPipeline` keeps the copies off the critical path:

- host -> device copies of call i + 1 run on their own stream while call i
  computes;
- the device -> host copy of call i's output runs on a third stream, in
  parallel with the next call's inputs (PCIe is full duplex);
- the device buffers are double-buffered, with events ordering reuse.

The attention runs unchanged (the same kernels, on the compute stream).
"""

from __future__ import annotations

import torch


class HostPipeline:
    """Runs `fn(q, k, v, layer_index)` on pinned host tensors, overlapping
    the copies of neighbouring calls with the attention.

    `__call__` only enqueues work; `synchronize()` waits for all of it. An
    output host buffer may be read after `synchronize()` (or after the
    event `__call__` returns has completed).
    """

    def __init__(self, fn, shape, dtype=torch.bfloat16,
                 device: torch.device | str = 'cuda', depth: int = 2):
        if depth < 1:
            raise ValueError('depth must be >= 1')
        self.fn = fn
        self.device = torch.device(device)
        self.depth = depth
        self.h2d = torch.cuda.Stream(self.device)
        self.compute = torch.cuda.Stream(self.device)
        self.d2h = torch.cuda.Stream(self.device)
        self.inputs = [[torch.empty(shape, dtype=dtype, device=self.device)
                        for _ in range(3)] for _ in range(depth)]
        self.outputs = [None] * depth
        # Slot i's inputs are free once the compute that read them finished;
        # its output once its device -> host copy finished.
        self.inputs_free = [None] * depth
        self.output_free = [None] * depth
        self.calls = 0

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                 layer_index: int, out: torch.Tensor) -> torch.cuda.Event:
        for name, t in (('q', q), ('k', k), ('v', v), ('out', out)):
            if t.device.type != 'cpu' or not t.is_pinned():
                raise ValueError(f'{name} must be a pinned host tensor')
        slot = self.calls % self.depth
        self.calls += 1
        dev = self.inputs[slot]
        with torch.cuda.stream(self.h2d):
            if self.inputs_free[slot] is not None:
                self.h2d.wait_event(self.inputs_free[slot])
            for d, h in zip(dev, (q, k, v)):
                d.copy_(h, non_blocking=True)
            loaded = torch.cuda.Event()
            loaded.record(self.h2d)
        with torch.cuda.stream(self.compute):
            self.compute.wait_event(loaded)
            if self.output_free[slot] is not None:
                self.compute.wait_event(self.output_free[slot])
            result = self.fn(*dev, layer_index)
            done = torch.cuda.Event()
            done.record(self.compute)
        self.inputs_free[slot] = done
        with torch.cuda.stream(self.d2h):
            self.d2h.wait_event(done)
            result.record_stream(self.d2h)
            out.copy_(result, non_blocking=True)
            copied = torch.cuda.Event()
            copied.record(self.d2h)
        self.outputs[slot] = result
        self.output_free[slot] = copied
        return copied

    def wait_on(self, stream: torch.cuda.Stream) -> None:
        """Makes `stream` wait for every call enqueued so far."""
        for ev in self.output_free:
            if ev is not None:
                stream.wait_event(ev)

    def synchronize(self) -> None:
        for s in (self.h2d, self.compute, self.d2h):
            s.synchronize()
