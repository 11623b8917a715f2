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

    def _setup(self, xh, d_out, device):
        rows = -(-xh.shape[0] // self.chunks)
        key = (rows, xh.shape[1], d_out, xh.dtype, device)
        if self._bufs is None or self._bufs[0] != key:
            xb = [torch.empty(rows, xh.shape[1], dtype=xh.dtype, device=device) for _ in range(2)]
            yb = [torch.empty(rows, d_out, dtype=xh.dtype, device=device) for _ in range(2)]
            self._bufs = (key, xb, yb, torch.cuda.Stream(device), torch.cuda.Stream(device))
        return self._bufs

    def __call__(self, xh, yh, device="cuda"):
        """xh [M, d] pinned host input, yh [M, d_out] pinned host output. Work is
        queued on the current stream (compute) and two side streams (copies);
        the current stream waits for the last copy, so synchronising it covers
        everything."""
        _, xb, yb, s_in, s_out = self._setup(xh, yh.shape[1], torch.device(device))
        comp = torch.cuda.current_stream(device)
        M = xh.shape[0]
        rows = xb[0].shape[0]
        copied = [None, None]    # H2D of the chunk in buffer b done
        computed = [None, None]  # compute of the chunk in buffer b done (x buffer free)
        drained = [None, None]   # D2H of the chunk in buffer b done (y buffer free)
        starts = list(range(0, M, rows))

        def issue_h2d(i):
            b = i % 2
            lo, hi = starts[i], min(starts[i] + rows, M)
            with torch.cuda.stream(s_in):
                if computed[b] is not None:
                    s_in.wait_event(computed[b])
                xb[b][:hi - lo].copy_(xh[lo:hi], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(s_in)
                copied[b] = ev

        issue_h2d(0)
        for i, lo in enumerate(starts):
            b = i % 2
            hi = min(lo + rows, M)
            if i + 1 < len(starts):
                issue_h2d(i + 1)
            comp.wait_event(copied[b])
            if drained[b] is not None:
                comp.wait_event(drained[b])
            self.forward(xb[b][:hi - lo], yb[b][:hi - lo])
            ev = torch.cuda.Event()
            ev.record(comp)
            computed[b] = ev
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev)
                yh[lo:hi].copy_(yb[b][:hi - lo], non_blocking=True)
                dev = torch.cuda.Event()
                dev.record(s_out)
                drained[b] = dev
        for e in drained:
            if e is not None:
                comp.wait_event(e)
        return yh

    @property
    def copy_streams(self):
        """(host->device, device->host) streams, for callers that queue more copies."""
        return (self._bufs[3], self._bufs[4]) if self._bufs else (None, None)
