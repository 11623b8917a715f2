"""Host-resident inputs and outputs with copies overlapped against compute.

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
