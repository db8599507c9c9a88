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

    def __init__(self, layer, slots: int = 2, trace: bool = False, chunk_bytes: int = 1 << 20):
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
        # Host copies split into pieces of at most chunk_bytes (0: one copy per tensor).  With
        # several GPUs exchanging over NVLink, whole-tensor PCIe copies in flight beside the
        # layer stretched its forward (DeepSeek-V3 EP8: 1.68 -> 2.99 ms, whatever the all-gather
        # transport); 1 MiB pieces brought the host-fed step from 3.17 to 2.53 ms, against a
        # 1.84 ms floor for the copies alone.
        self.chunk_bytes = chunk_bytes
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
            self._copy(x_d, x_h)
            self._copy(ids_d, ids_h)
            self._copy(w_d, w_h)
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
            self._copy(out_h, self._out[s])
            self._stored[s].record(self.d2h)
            if ev:
                ev[5].record(self.d2h)
        if ev:
            self._spans.append(tuple(ev))
        self._used[s] = True
        self.step += 1
        return self._stored[s]

    def _copy(self, dst: torch.Tensor, src: torch.Tensor) -> None:
        """dst.copy_(src) on the current stream, in row pieces of at most chunk_bytes."""
        row = src[0].numel() * src.element_size() if src.dim() > 0 and src.shape[0] else 0
        if not self.chunk_bytes or row == 0 or src.numel() * src.element_size() <= self.chunk_bytes:
            dst.copy_(src, non_blocking=True)
            return
        rows = max(1, self.chunk_bytes // row)
        for r0 in range(0, src.shape[0], rows):
            dst[r0:r0 + rows].copy_(src[r0:r0 + rows], non_blocking=True)

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
