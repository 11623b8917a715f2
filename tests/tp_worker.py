"""Worker for tests/test_gpu_tp.py, launched with torchrun (one process per GPU).

mode "parity": the tensor-parallel MLP through every exchange against the
single-GPU block on the same full weights.
mode "timeout": rank 1 leaves between steps (it launches nothing for the second
step); rank 0's bounded host wait must report the missing peer, release its own
stream waits and keep its CUDA context usable.
Rank 0 prints one JSON line prefixed with "RESULT ".
"""
import json
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import polykernel_b200 as pk  # noqa: E402
from polykernel_b200.tp import TensorParallelMLP, shard_weights  # noqa: E402


def setup():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank),
                            timeout=timedelta(seconds=60))
    host = dist.new_group(backend="gloo", timeout=timedelta(seconds=60))
    return rank, world, host


def weights(M, d, ffn):
    g = torch.Generator(device="cuda").manual_seed(0)
    X = torch.randn(M, d, device="cuda", generator=g).bfloat16()
    gm = (1 + 0.1 * torch.randn(d, device="cuda", generator=g)).bfloat16()
    W1 = (torch.randn(d, ffn, device="cuda", generator=g) / d ** 0.5).bfloat16()
    b1 = (0.02 * torch.randn(ffn, device="cuda", generator=g)).bfloat16()
    W2 = (torch.randn(ffn, d, device="cuda", generator=g) / ffn ** 0.5).bfloat16()
    b2 = (0.02 * torch.randn(d, device="cuda", generator=g)).bfloat16()
    return X, gm, W1, b1, W2, b2


def parity(rank, world, host):
    M, d, ffn = 2048, 1024, 4096
    X, gm, W1, b1, W2, b2 = weights(M, d, ffn)
    ref = pk.ops.mlp_block(X, gm, W1, b1, W2, b2, 1e-6)
    w1s, b1s, w2s = shard_weights(W1, b1, W2, rank, world)
    outs, res = {}, {}
    for name, kw in (("copy_engine", dict(reduce="copy_engine")),
                     ("copy_engine_gemm1_chunked", dict(reduce="copy_engine", gemm1_chunked=True)),
                     ("copy_engine_one_stream", dict(reduce="copy_engine", per_peer_streams=False)),
                     ("nccl", dict(reduce="nccl")),
                     ("peer_store", dict(reduce="peer_store"))):
        m = TensorParallelMLP(gm, w1s, b1s, w2s, b2, 1e-6, chunks=4, **kw)
        for _ in range(3):                       # reuse of slots / rows / flags across steps
            X2 = X.clone()
            y = m(X2)
        m.wait(10000) if name.startswith("copy_engine") else torch.cuda.synchronize()
        outs[name] = y
        if name.startswith("copy_engine"):
            res[name + "_joined_streams"] = m.joined_streams()
        # every rank's row block (the owner's reduce + the pulls), separately
        per = M // world
        res[name + "_blocks_exact"] = [
            (y[p * per:(p + 1) * per] == ref[p * per:(p + 1) * per]).float().mean().item()
            for p in range(world)]
        ex = (y == ref).float().mean().item()
        rel = ((y.float() - ref.float()).abs() / ref.float().abs().clamp_min(
            ref.float().pow(2).mean().sqrt())).max().item()
        res[name] = {"bit_exact": ex, "max_err_over_scale": rel}
        if name.startswith("copy_engine"):
            m.close()
    # every rank holds the full output, identical across ranks
    gathered = [torch.empty_like(outs["copy_engine"]) for _ in range(world)]
    dist.all_gather(gathered, outs["copy_engine"])
    res["ranks_agree"] = all(torch.equal(g, gathered[0]) for g in gathered)
    # both copy-engine variants and the peer-store path sum the slots in rank order
    res["ce_eq_one_stream"] = torch.equal(outs["copy_engine"], outs["copy_engine_one_stream"])
    res["ce_eq_gemm1_chunked"] = torch.equal(outs["copy_engine"], outs["copy_engine_gemm1_chunked"])
    res["ce_eq_peer_store"] = torch.equal(outs["copy_engine"], outs["peer_store"])
    res["device_error"] = pk.device_error()
    return res


def timeout(rank, world, host):
    M, d, ffn = 1024, 512, 2048
    X, gm, W1, b1, W2, b2 = weights(M, d, ffn)
    w1s, b1s, w2s = shard_weights(W1, b1, W2, rank, world)
    m = TensorParallelMLP(gm, w1s, b1s, w2s, b2, 1e-6, chunks=2, reduce="copy_engine")
    m(X)
    m.wait(10000)                                # step 1 completes on every rank
    dist.barrier(group=host)
    res = {}
    if rank == 0:
        m(X)                                     # step 2: rank 1 never takes part
        try:
            m.wait(1000)
            res["raised"] = False
        except TimeoutError as e:
            res["raised"] = True
            res["message"] = str(e)
        # the context is still usable after the released waits
        a = torch.randn(256, 256, device="cuda").bfloat16()
        res["context_ok"] = torch.equal(pk.ops.matmul(a, torch.eye(256, device="cuda").bfloat16()), a)
        res["device_error"] = pk.device_error()
    dist.barrier(group=host)                     # rank 1 stays alive until rank 0 is done
    m.close()
    return res


def main():
    rank, world, host = setup()
    res = {"parity": parity, "timeout": timeout}[sys.argv[1]](rank, world, host)
    if rank == 0:
        print("RESULT " + json.dumps(res), flush=True)
    dist.barrier(group=host)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
