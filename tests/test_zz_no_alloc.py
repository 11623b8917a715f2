"""GPU: pkb200_fused_rmsnorm_matmul_noalloc, the entry point for callers that
cannot allocate device memory (graph capture in progress, hosts that forbid
allocation after start-up, plugins whose host owns all memory). It must give
the same output as pkb200_fused_rmsnorm_matmul, on consecutive calls that share
its fixed scratch array, and reject shapes beyond that array.

Kept in its own file, collected last, so a run that stops at the first failure
has already run every other test.
"""
import ctypes

import numpy as np
import pytest

from oracle import golden_np as O
from tests.helpers import check_parity, f32_from_t

pytestmark = pytest.mark.gpu


def _call(lib, fn, x, w, g, out, eps):
    import torch
    M, K = x.shape
    N = w.shape[1]
    return getattr(lib, fn)(x.data_ptr(), w.data_ptr(), g.data_ptr() if g is not None else None,
                            out.data_ptr(), M, N, K, ctypes.c_float(eps),
                            torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_allocating_entry_point(cuda):
    import torch
    import polykernel_b200 as pk
    lib = pk.lib()
    gen = torch.Generator(device="cuda").manual_seed(3)
    cases = [(256, 1024, 768), (130, 512, 264)]  # second call is smaller: stale rows must not leak
    for M, K, N in cases:
        x = torch.randn(M, K, device="cuda", generator=gen).to(torch.bfloat16)
        w = (torch.randn(K, N, device="cuda", generator=gen) / K ** 0.5).to(torch.bfloat16)
        g = (1 + 0.1 * torch.randn(K, device="cuda", generator=gen)).to(torch.bfloat16)
        ref = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        out = torch.full((M, N), float("nan"), device="cuda", dtype=torch.bfloat16)
        assert _call(lib, "pkb200_fused_rmsnorm_matmul", x, w, g, ref, 1e-6) == 0
        assert _call(lib, "pkb200_fused_rmsnorm_matmul_noalloc", x, w, g, out, 1e-6) == 0
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
        # and within the parity tolerance of the golden restatement
        xf, wf, gf = (f32_from_t(t) for t in (x, w, g))
        check_parity(f32_from_t(out), O.fused_rmsnorm_matmul(xf, wf, gf, 1e-6),
                     min_exact=0.98)
    assert pk.device_error() == 0


def test_noalloc_rejects_oversize(cuda):
    import torch
    import polykernel_b200 as pk
    lib = pk.lib()
    M, K, N = 2049, 4096, 8  # M*K just above the 8,388,608-element scratch
    x = torch.zeros(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(K, N, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(M, N, device="cuda", dtype=torch.bfloat16)
    assert _call(lib, "pkb200_fused_rmsnorm_matmul_noalloc", x, w, None, out, 1e-5) == 1


def test_noalloc_at_the_scratch_limit(cuda):
    """M*K exactly equal to the scratch array's 8,388,608 elements is accepted
    and gives the allocating entry point's output."""
    import torch
    import polykernel_b200 as pk
    lib = pk.lib()
    gen = torch.Generator(device="cuda").manual_seed(4)
    M, K, N = 2048, 4096, 64
    x = torch.randn(M, K, device="cuda", generator=gen).to(torch.bfloat16)
    w = (torch.randn(K, N, device="cuda", generator=gen) / K ** 0.5).to(torch.bfloat16)
    ref = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    out = torch.full((M, N), float("nan"), device="cuda", dtype=torch.bfloat16)
    assert _call(lib, "pkb200_fused_rmsnorm_matmul", x, w, None, ref, 1e-6) == 0
    assert _call(lib, "pkb200_fused_rmsnorm_matmul_noalloc", x, w, None, out, 1e-6) == 0
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    assert pk.device_error() == 0
