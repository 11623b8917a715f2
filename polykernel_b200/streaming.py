"""Host-resident inputs and outputs with copies overlapped against compute.

Two forms: `HostStreamed` streams row chunks of one row-independent call (the
MLP block) through two device buffers; `HostStepPipeline` overlaps whole
steps (all of a step's inputs and outputs) with the neighbouring steps'
compute through two device buffer sets.

`HostStreamed(forward, chunks)` runs `forward(x, out)` (a device function that
writes the [rows, d_out] result for a [rows, d] bf16 input into `out`; it must be
row-independent, as the MLP block is) over row chunks of a pinned host tensor: the host->device copy of chunk
i+1 and the device->host copy of chunk i-1 run on their own streams while chunk
i computes, through two device buffers per direction. The copy engines and the
SMs work at the same time, so end-to-end time approaches max(compute, H2D, D2H)
instead of their sum.
"""
from __future__ import annotations

import torch


class HostStreamed:
    def __init__(self, forward, chunks=4):
        self.forward = forward
        self.chunks = max(1, int(chunks))
        self._bufs = None
        # per device buffer: last H2D done / compute done / D2H done. Kept
        # across calls, so a call may start while the previous call's last
        # copies are still in flight (see `sync`).
        self._copied = [None, None]
        self._computed = [None, None]
        self._drained = [None, None]
        self._next = 0  # buffer the next chunk uses

    def _setup(self, xh, d_out, device):
        rows = -(-xh.shape[0] // self.chunks)
        key = (rows, xh.shape[1], d_out, xh.dtype, device)
        if self._bufs is None or self._bufs[0] != key:
            if self._bufs is not None:
                self.wait(torch.cuda.current_stream(self._bufs[0][4]))
            xb = [torch.empty(rows, xh.shape[1], dtype=xh.dtype, device=device) for _ in range(2)]
            yb = [torch.empty(rows, d_out, dtype=xh.dtype, device=device) for _ in range(2)]
            self._bufs = (key, xb, yb, torch.cuda.Stream(device), torch.cuda.Stream(device))
            self._copied, self._computed, self._drained = [None, None], [None, None], [None, None]
            self._next = 0
        return self._bufs

    def __call__(self, xh, yh, device="cuda", sync=True):
        """xh [M, d] pinned host input, yh [M, d_out] pinned host output. Work is
        queued on the current stream (compute) and two side streams (copies).
        With `sync` the current stream then waits for the last copy, so
        synchronising it covers everything; without it the last device->host
        copies may still run while the caller queues more work (the next call
        included), and `wait()` joins them."""
        _, xb, yb, s_in, s_out = self._setup(xh, yh.shape[1], torch.device(device))
        comp = torch.cuda.current_stream(device)
        M = xh.shape[0]
        rows = xb[0].shape[0]
        starts = list(range(0, M, rows))
        bufs = [(self._next + i) % 2 for i in range(len(starts))]

        def issue_h2d(i):
            b = bufs[i]
            lo, hi = starts[i], min(starts[i] + rows, M)
            with torch.cuda.stream(s_in):
                if self._computed[b] is not None:
                    s_in.wait_event(self._computed[b])   # the x buffer is free again
                xb[b][:hi - lo].copy_(xh[lo:hi], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(s_in)
                self._copied[b] = ev

        issue_h2d(0)
        for i, lo in enumerate(starts):
            b = bufs[i]
            hi = min(lo + rows, M)
            if i + 1 < len(starts):
                issue_h2d(i + 1)
            comp.wait_event(self._copied[b])
            if self._drained[b] is not None:
                comp.wait_event(self._drained[b])      # the y buffer is free again
            self.forward(xb[b][:hi - lo], yb[b][:hi - lo])
            ev = torch.cuda.Event()
            ev.record(comp)
            self._computed[b] = ev
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev)
                yh[lo:hi].copy_(yb[b][:hi - lo], non_blocking=True)
                dev = torch.cuda.Event()
                dev.record(s_out)
                self._drained[b] = dev
        self._next = (self._next + len(starts)) % 2
        if sync:
            self.wait(comp)
        return yh

    def wait(self, stream=None):
        """Make `stream` (default: the current stream) wait for every copy queued so far."""
        stream = stream or torch.cuda.current_stream()
        for e in self._drained:
            if e is not None:
                stream.wait_event(e)

    @property
    def copy_streams(self):
        """(host->device, device->host) streams, for callers that queue more copies."""
        return (self._bufs[3], self._bufs[4]) if self._bufs else (None, None)


class HostStepPipeline:
    """Steps over host-resident inputs and outputs with the copies of
    neighbouring steps overlapped against compute.

    `host_inputs` / `host_outputs` are pinned host tensors. Each `step(compute)`
    copies the inputs into one of `depth` device buffer sets on a copy stream,
    runs `compute(device_inputs, device_outputs)` on the current stream, and
    copies the outputs back on a second copy stream. A buffer set is reused
    only after its previous device->host copy finished, so step i+1's inputs
    cross PCIe while step i computes and step i-1's outputs drain: end-to-end
    time approaches max(compute, H2D, D2H) per step. `wait(stream)` makes a
    stream wait for every copy queued so far. The host input tensors must not
    be rewritten until the step that reads them has been joined."""

    def __init__(self, host_inputs, host_outputs, device="cuda", depth=2):
        self.device = torch.device(device)
        self.hin = list(host_inputs)
        self.hout = list(host_outputs)
        self.depth = max(1, int(depth))
        self.din = [[torch.empty(h.shape, dtype=h.dtype, device=self.device) for h in self.hin]
                    for _ in range(self.depth)]
        self.dout = [[torch.empty(h.shape, dtype=h.dtype, device=self.device) for h in self.hout]
                     for _ in range(self.depth)]
        self.s_in = torch.cuda.Stream(self.device)
        self.s_out = torch.cuda.Stream(self.device)
        self._free = [None] * self.depth   # set k's last device->host copy done
        self._i = 0

    @property
    def h2d_bytes(self):
        return sum(h.numel() * h.element_size() for h in self.hin)

    @property
    def d2h_bytes(self):
        return sum(h.numel() * h.element_size() for h in self.hout)

    def step(self, compute):
        k = self._i % self.depth
        self._i += 1
        comp = torch.cuda.current_stream(self.device)
        with torch.cuda.stream(self.s_in):
            if self._free[k] is not None:
                self.s_in.wait_event(self._free[k])    # set k's previous step fully drained
            for h, d in zip(self.hin, self.din[k]):
                d.copy_(h, non_blocking=True)
            copied = torch.cuda.Event()
            copied.record(self.s_in)
        comp.wait_event(copied)
        compute(self.din[k], self.dout[k])
        done = torch.cuda.Event()
        done.record(comp)
        with torch.cuda.stream(self.s_out):
            self.s_out.wait_event(done)
            for h, d in zip(self.hout, self.dout[k]):
                h.copy_(d, non_blocking=True)
            drained = torch.cuda.Event()
            drained.record(self.s_out)
        self._free[k] = drained
        return self.dout[k]

    def wait(self, stream=None):
        stream = stream or torch.cuda.current_stream(self.device)
        for e in self._free:
            if e is not None:
                stream.wait_event(e)
