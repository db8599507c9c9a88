"""Host-resident inputs and outputs for a layer, with transfers overlapped with compute.

A serving loop holds each step's activations and routing in (pinned) host memory and
wants the result back in host memory.  ``HostPipeline`` keeps two device slots of
inputs and outputs: the host->device copies of step i+1 run on one copy stream and the
device->host copy of step i-1 on another while step i computes, so the PCIe time hides
behind the layer instead of adding to it.  Every step still moves its own inputs in and
its own result out; ``drain()`` waits for the last copies.

    pipe = HostPipeline(layer)
    for x_h, ids_h, w_h, out_h in steps:      # pinned CPU tensors
        pipe.submit(x_h, ids_h, w_h, out_h)
    pipe.drain()
"""
from __future__ import annotations

import torch


class HostPipeline:
    """``trace=True`` records CUDA events around every step's copies and forward (``spans()``
    summarises them); it adds event records to the streams and is meant for diagnosis."""

    def __init__(self, layer, slots: int = 2, trace: bool = False):
        self.layer = layer
        dev = layer.device
        self.compute = torch.cuda.current_stream(dev)
        self.h2d = torch.cuda.Stream(dev)
        self.d2h = torch.cuda.Stream(dev)
        self.slots = slots
        self._in = [None] * slots                       # device copies of (x, ids, weights)
        self._out = [torch.empty_like(layer.out_local) for _ in range(slots)]
        self._loaded = [torch.cuda.Event() for _ in range(slots)]   # h2d of the slot done
        self._computed = [torch.cuda.Event() for _ in range(slots)]  # forward of the slot done
        self._stored = [torch.cuda.Event() for _ in range(slots)]    # d2h of the slot done
        self._used = [False] * slots
        self.step = 0
        self.trace = trace
        self._spans: list[tuple] = []   # per traced step: (h2d0, h2d1, fwd0, fwd1, d2h0, d2h1)

    def _device_inputs(self, s: int, x_h, ids_h, w_h):
        cur = self._in[s]
        if cur is None or cur[0].shape != x_h.shape or cur[1].shape != ids_h.shape:
            dev = self.layer.device
            cur = (torch.empty(x_h.shape, dtype=x_h.dtype, device=dev),
                   torch.empty(ids_h.shape, dtype=ids_h.dtype, device=dev),
                   torch.empty(w_h.shape, dtype=w_h.dtype, device=dev))
            self._in[s] = cur
        return cur

    def submit(self, x_h: torch.Tensor, ids_h: torch.Tensor, w_h: torch.Tensor, out_h: torch.Tensor) -> torch.cuda.Event:
        """Enqueue one step; returns the event after which ``out_h`` holds its result."""
        s = self.step % self.slots
        x_d, ids_d, w_d = self._device_inputs(s, x_h, ids_h, w_h)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)] if self.trace else None
        if self._used[s]:
            self.h2d.wait_event(self._computed[s])     # the slot's previous forward has read its inputs
        with torch.cuda.stream(self.h2d):
            if ev:
                ev[0].record(self.h2d)
            x_d.copy_(x_h, non_blocking=True)
            ids_d.copy_(ids_h, non_blocking=True)
            w_d.copy_(w_h, non_blocking=True)
            self._loaded[s].record(self.h2d)
            if ev:
                ev[1].record(self.h2d)
        self.compute.wait_event(self._loaded[s])
        if self._used[s]:
            self.compute.wait_event(self._stored[s])   # the slot's previous result has left the GPU
        if ev:
            ev[2].record(self.compute)
        self.layer.forward(x_d, ids_d, w_d, out=self._out[s])
        self._computed[s].record(self.compute)
        if ev:
            ev[3].record(self.compute)
        self.d2h.wait_event(self._computed[s])
        with torch.cuda.stream(self.d2h):
            if ev:
                ev[4].record(self.d2h)
            out_h.copy_(self._out[s], non_blocking=True)
            self._stored[s].record(self.d2h)
            if ev:
                ev[5].record(self.d2h)
        if ev:
            self._spans.append(tuple(ev))
        self._used[s] = True
        self.step += 1
        return self._stored[s]

    def spans(self) -> dict:
        """Mean ms of the traced steps' host->device copies, forwards and device->host copies,
        the mean interval between forward starts (the steady-state step), and how long a
        forward waited for its inputs after the previous forward ended (copy-bound stalls)."""
        if len(self._spans) < 2:
            return {}
        torch.cuda.synchronize(self.layer.device)
        sp = self._spans
        mean = lambda xs: sum(xs) / len(xs)  # noqa: E731
        return {"h2d_ms": mean([a.elapsed_time(b) for a, b, *_ in sp]),
                "forward_ms": mean([e[2].elapsed_time(e[3]) for e in sp]),
                "d2h_ms": mean([e[4].elapsed_time(e[5]) for e in sp]),
                "step_interval_ms": mean([sp[i][2].elapsed_time(sp[i + 1][2]) for i in range(len(sp) - 1)]),
                "forward_gap_ms": mean([sp[i][3].elapsed_time(sp[i + 1][2]) for i in range(len(sp) - 1)]),
                "steps": len(sp)}

    def drain(self) -> None:
        for s in range(self.slots):
            if self._used[s]:
                self._stored[s].synchronize()
