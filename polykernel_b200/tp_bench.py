"""Tensor-parallel exchange benchmark: times each part of the TP MLP's exchange
in isolation, one process per GPU.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N \\
        --master-addr 127.0.0.1 --master-port P -m polykernel_b200.tp_bench \\
        [--M 16384 --d 8192 --ffn 28672 --chunks 4 --iters 5]

Rank 0 prints one JSON line per measurement: {"part", "n_gpus", "ms", "gbs"}.
Every time is measured with CUDA events on each rank and reduced as the max
over ranks. Byte counts are per rank, outgoing over NVLink:
* push:  (N-1)/N · M·d·4 (each rank's fp32 partial row blocks to their owners);
* pull:  (N-1)/N · M·d·2 (the reduced bf16 rows from every peer).

Parts:
* gemm2_chunked: GEMM2 in row chunks alone (the window the exchange must hide in);
* nccl_reduce_scatter_fp32 and nccl_all_gather_bf16;
* ce_push, ce_pull, ce_push_pull: copy-engine copies over CUDA IPC mappings,
  each with one stream per peer ("per_peer") or one stream for all ("one_stream");
* ce_push_during_gemm: the pushes issued beside the chunked GEMM2;
* mlp_step_<exchange>: the whole TensorParallelMLP step per exchange.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os

import torch
import torch.distributed as dist


def _time(fn, iters, warmup, dev):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(dev)
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize(dev)
    t = torch.tensor([s.elapsed_time(e) / iters], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class _Shared:
    """A device buffer of this library (pkb200_ipc_alloc) mapped into every
    peer with CUDA IPC; ptrs[p] is rank p's buffer in this process."""

    def __init__(self, nbytes, world, rank):
        from ._lib import check, lib
        self.lib = lib()
        own = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        check(self.lib.pkb200_ipc_alloc(nbytes, ctypes.byref(own), handle), "ipc_alloc")
        gathered = [None] * world
        dist.all_gather_object(gathered, handle.raw)
        self.ptrs, self.opened, self.own = [], [], own.value
        for p in range(world):
            if p == rank:
                self.ptrs.append(own.value)
                continue
            q = ctypes.c_void_p()
            check(self.lib.pkb200_ipc_open(gathered[p], ctypes.byref(q)), "ipc_open")
            self.ptrs.append(q.value)
            self.opened.append(q.value)

    def close(self):
        torch.cuda.synchronize()
        dist.barrier()
        for q in self.opened:
            self.lib.pkb200_ipc_close(q)
        dist.barrier()
        self.lib.pkb200_free(self.own)


def main(argv=None):
    ap = argparse.ArgumentParser(prog="python -m polykernel_b200.tp_bench")
    ap.add_argument("--M", type=int, default=16384)
    ap.add_argument("--d", type=int, default=8192)
    ap.add_argument("--ffn", type=int, default=28672)
    ap.add_argument("--chunks", type=int, default=4)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    args = ap.parse_args(argv)

    from ._lib import check, lib
    from .tp import TensorParallelMLP

    # separate hardware queues for the per-peer copy streams (before CUDA starts)
    os.environ.setdefault("CUDA_DEVICE_MAX_CONNECTIONS", "32")
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev)
    M, d, ffn, C = args.M, args.d, args.ffn, args.chunks
    if ffn % world or M % (C * world):
        raise SystemExit("ffn must divide by N and M by chunks*N")
    F = ffn // world
    per = M // world
    out = []

    def emit(part, ms, nbytes=None, **extra):
        rec = {"part": part, "n_gpus": world, "ms": round(ms, 4),
               "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1) if nbytes else None, **extra}
        out.append(rec)
        if rank == 0:
            print(json.dumps(rec), flush=True)

    g = torch.Generator(device=dev).manual_seed(rank)
    h = torch.randn(M, F, device=dev, generator=g).to(torch.bfloat16)
    w2 = (torch.randn(F, d, device=dev, generator=g) / F ** 0.5).to(torch.bfloat16)
    y32 = torch.empty(M, d, device=dev, dtype=torch.float32)
    rows = M // C
    main_s = torch.cuda.current_stream()

    def gemm2_chunks():
        for i in range(C):
            check(lib().pkb200_matmul_f32out(h[i * rows:(i + 1) * rows].data_ptr(), w2.data_ptr(),
                                             y32[i * rows:(i + 1) * rows].data_ptr(), rows, d, F,
                                             main_s.cuda_stream), "matmul_f32out")
    emit("gemm2_chunked", _time(gemm2_chunks, args.iters, args.warmup, dev))

    part32 = torch.empty(per, d, device=dev, dtype=torch.float32)
    y16 = torch.empty(M, d, device=dev, dtype=torch.bfloat16)
    mine16 = torch.empty(per, d, device=dev, dtype=torch.bfloat16)
    push_bytes = (world - 1) * per * d * 4
    pull_bytes = (world - 1) * per * d * 2
    emit("nccl_reduce_scatter_fp32",
         _time(lambda: dist.reduce_scatter_tensor(part32, y32), args.iters, args.warmup, dev),
         push_bytes)
    emit("nccl_all_gather_bf16",
         _time(lambda: dist.all_gather_into_tensor(y16, mine16), args.iters, args.warmup, dev),
         pull_bytes)

    if world > 1:
        slots = _Shared(M * d * 4, world, rank)     # [world][per][d] fp32 per rank
        rows16 = _Shared(per * d * 2, world, rank)  # [per][d] bf16 per rank
        streams = [torch.cuda.Stream(dev) for _ in range(world)]
        peers = [(rank + k) % world for k in range(1, world)]

        def copies(push, pull, per_peer):
            ev = torch.cuda.Event()
            ev.record(main_s)
            for p in peers:
                s = streams[p if per_peer else 0]
                s.wait_event(ev)
                if push:
                    check(lib().pkb200_copy_async(
                        slots.ptrs[p] + rank * per * d * 4, y32[p * per:(p + 1) * per].data_ptr(),
                        per * d * 4, s.cuda_stream), "copy_async")
                if pull:
                    check(lib().pkb200_copy_async(
                        y16[p * per:(p + 1) * per].data_ptr(), rows16.ptrs[p], per * d * 2,
                        s.cuda_stream), "copy_async")
            for s in (streams if per_peer else streams[:1]):
                main_s.wait_stream(s)

        for mode, per_peer in (("per_peer", True), ("one_stream", False)):
            emit("ce_push", _time(lambda: copies(True, False, per_peer), args.iters,
                                  args.warmup, dev), push_bytes, streams=mode)
            emit("ce_pull", _time(lambda: copies(False, True, per_peer), args.iters,
                                  args.warmup, dev), pull_bytes, streams=mode)
            emit("ce_push_pull", _time(lambda: copies(True, True, per_peer), args.iters,
                                       args.warmup, dev), push_bytes + pull_bytes, streams=mode)

        def push_during_gemm():
            ev = torch.cuda.Event()
            ev.record(main_s)
            for p in peers:
                streams[p].wait_event(ev)
                check(lib().pkb200_copy_async(
                    slots.ptrs[p] + rank * per * d * 4, y32[p * per:(p + 1) * per].data_ptr(),
                    per * d * 4, streams[p].cuda_stream), "copy_async")
            gemm2_chunks()
            for p in peers:
                main_s.wait_stream(streams[p])
        emit("ce_push_during_gemm", _time(push_during_gemm, args.iters, args.warmup, dev),
             push_bytes)
        slots.close()
        rows16.close()

        x = torch.randn(M, d, device=dev, generator=g).to(torch.bfloat16)
        gamma = torch.ones(d, device=dev, dtype=torch.bfloat16)
        w1 = (torch.randn(d, F, device=dev, generator=g) / d ** 0.5).to(torch.bfloat16)
        b1 = torch.zeros(F, device=dev, dtype=torch.bfloat16)
        b2 = torch.zeros(d, device=dev, dtype=torch.bfloat16)
        for reduce in ("nccl", "copy_engine"):
            m = TensorParallelMLP(gamma, w1, b1, w2, b2, 1e-6, chunks=C, reduce=reduce)
            y = torch.empty_like(x)
            emit(f"mlp_step_{reduce}", _time(lambda: m(x, out=y), args.iters, args.warmup, dev))
            m.close()
    dist.destroy_process_group()
    return out


if __name__ == "__main__":
    main()
