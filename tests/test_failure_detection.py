"""Failure detection without faulting a GPU.

GPU: a bounded device-side wait that nothing satisfies gives up after a short
limit, records its code in the library's error word and returns; the context
keeps working afterwards. CPU (gloo): a tensor-parallel rank that never joins
the collective surfaces as an error on the others within the process-group
timeout instead of a hang."""
import ctypes
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


@pytest.mark.gpu
def test_bounded_wait_gives_up_and_reports(cuda):
    import polykernel_b200 as pk
    lib = pk.lib()
    code = ctypes.c_int(-1)
    assert lib.pkb200_selftest_wait_timeout(2_000_000, ctypes.byref(code)) == 0  # ~1 ms
    assert code.value == 6
    assert pk.device_error() == 0          # reading cleared it
    a = torch.randn(256, 256, device="cuda").bfloat16()
    b = torch.randn(256, 256, device="cuda").bfloat16()
    assert torch.equal(pk.ops.matmul(a, b), pk.ops.matmul(a, b))  # context still usable


def test_selftest_rejects_bad_limits():
    from polykernel_b200._lib import lib
    code = ctypes.c_int(0)
    assert lib().pkb200_selftest_wait_timeout(0, ctypes.byref(code)) != 0
    assert lib().pkb200_selftest_wait_timeout(10 ** 12, ctypes.byref(code)) != 0


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=4))
    from tests.test_tp_cpu import CpuKern
    from polykernel_b200.tp import TensorParallelMLP
    x = torch.randn(4, 8).bfloat16()
    m = TensorParallelMLP(torch.ones(8).bfloat16(), torch.randn(8, 4).bfloat16(),
                          torch.zeros(4).bfloat16(), torch.randn(4, 8).bfloat16(),
                          torch.zeros(8).bfloat16(), kern=CpuKern)
    if rank == 1:
        q.put((1, "left"))       # this rank leaves between steps: it never calls the collective
        q.close()
        q.join_thread()
        os._exit(0)
    try:
        m(x)
        q.put((0, "no error"))
    except Exception as e:       # the collective with the missing rank fails
        q.put((0, type(e).__name__))
    q.close()
    q.join_thread()
    os._exit(0)


def test_missing_rank_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(60)
        assert p.exitcode is not None, "a rank hung"
    res = dict(q.get(timeout=5) for _ in range(2))
    assert res[1] == "left"
    assert res[0] != "no error"
