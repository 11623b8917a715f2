"""CPU (gloo, world_size 2): the tensor-parallel MLP's sharding and reduction
logic (polykernel_b200/tp.py) with a CPU stand-in for the kernels. The sharded
forward must equal the unsharded golden composition up to fp32 summation order."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import golden_np as O
from oracle import metrics as Mx


def _np(t):
    return t.float().numpy()


def _bf(a):
    return torch.from_numpy(O.bf16(a)).to(torch.bfloat16)


class CpuKern:
    """The four kernels TensorParallelMLP uses, with the golden rounding, on CPU."""

    @staticmethod
    def rmsnorm(x, w, eps):
        return _bf(O.rmsnorm(_np(x), _np(w), eps))

    @staticmethod
    def fused_matmul_bias_gelu(x, w, b):
        return _bf(O.fused_matmul_bias_gelu(_np(x), _np(w), _np(b)))

    @staticmethod
    def matmul_f32out(a, b):
        return torch.from_numpy(np.matmul(_np(a), _np(b)).astype(np.float32))

    @staticmethod
    def bias_residual_f32(y32, b, x, out=None):
        r = _bf(O.add(O.bias(O.bf16(y32.numpy()), _np(b)), _np(x)))
        if out is not None:
            out.copy_(r)
            return out
        return r


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from polykernel_b200.tp import TensorParallelMLP, shard_weights
    rng = np.random.default_rng(5)
    M, d, ffn = 8, 32, 64
    X = _bf(rng.standard_normal((M, d)))
    g = _bf(1 + 0.1 * rng.standard_normal(d))
    W1 = _bf(rng.standard_normal((d, ffn)) / np.sqrt(d))
    b1 = _bf(0.02 * rng.standard_normal(ffn))
    W2 = _bf(rng.standard_normal((ffn, d)) / np.sqrt(ffn))
    b2 = _bf(0.02 * rng.standard_normal(d))
    w1s, b1s, w2s = shard_weights(W1, b1, W2, rank, world)
    assert w1s.shape == (d, ffn // world) and w2s.shape == (ffn // world, d)
    y = TensorParallelMLP(g, w1s, b1s, w2s, b2, 1e-6, kern=CpuKern)(X)
    ref = O.mlp_block(_np(X), _np(g), _np(W1), _np(b1), _np(W2), _np(b2), 1e-6)
    q.put((rank, Mx.report(_np(y), ref)))
    dist.destroy_process_group()


def test_tp_mlp_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    res = dict(q.get() for _ in range(2))
    for r in (0, 1):
        assert res[r]["cosine"] > 0.99999 and res[r]["bit_exact"] > 0.95, res[r]


def test_shard_range_rejects_uneven():
    from polykernel_b200.tp import shard_range
    assert shard_range(28672, 3, 8) == (10752, 14336)
    with pytest.raises(ValueError):
        shard_range(10, 0, 3)


def test_bench_cli_help():
    """bench.py's command line (the TP exchange breakdown and the profiling
    cases included) parses without a GPU."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, os.path.join(root, "bench.py"), "--help"],
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and "--tp-breakdown" in r.stdout and "--profile-case" in r.stdout
