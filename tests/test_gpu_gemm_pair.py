"""The CTA-pair (cta_group::2, two SMs per 256 x 256 tile) tensor-core GEMM
against the single-SM kernel: every epilogue kind, ragged and full-size
shapes, bit for bit (the K reduction order per output is the same: K=16 MMA
steps in K order)."""
import ctypes
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
PAIR = (256, 256, 64, 10, 8, 2, 6)


@pytest.fixture(scope="module")
def pk(cuda):
    import polykernel_b200 as pk
    pk.lib()
    return pk


def _forced(pk, cfg, fn):
    lib = pk.lib()
    arr = (ctypes.c_int * 7)(*cfg) if cfg else None
    assert lib.pkb200_set_gemm_config(arr) == 0
    try:
        out = fn()
        import torch
        torch.cuda.synchronize()
        got = (ctypes.c_int * 7)()
        lib.pkb200_last_gemm_config(got)
        return out, tuple(got)
    finally:
        lib.pkb200_set_gemm_config(None)


@pytest.mark.parametrize("shape", [(256, 512, 512), (300, 264, 520), (2048, 16384, 4096),
                                   (130, 72, 136), (4096, 8192, 28672)],
                         ids=["one_tile", "ragged", "config2_gemm1", "tiny", "config5_gemm2_m4096"])
def test_pair_gemm_bit_identical_every_epilogue(pk, shape):
    import torch
    M, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    a = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(K, N, device="cuda", generator=g) / math.sqrt(K)).bfloat16()
    bias = (0.02 * torch.randn(N, device="cuda", generator=g)).bfloat16()
    res = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    wq = torch.randint(-127, 128, (K, N), device="cuda", generator=g, dtype=torch.int8)
    sc = (0.001 + 0.019 * torch.rand(N, device="cuda", generator=g)).bfloat16().float()
    cases = {
        "matmul": lambda: pk.ops.matmul(a, w),
        "bias_gelu": lambda: pk.ops.fused_matmul_bias_gelu(a, w, bias),
        "bias_resid": lambda: pk.ops.matmul_bias_residual(a, w, bias, res),
        "f32out": lambda: pk.ops.matmul_f32out(a, w),
        "int8_scale": lambda: pk.ops.matmul_int8(a, wq, sc),
    }
    tc_shape = K % 8 == 0 and N % 8 == 0
    for name, fn in cases.items():
        ref, cfg_ref = _forced(pk, None, fn)
        out, cfg = _forced(pk, PAIR, fn)
        if tc_shape:
            assert cfg == PAIR, (name, cfg)
        assert torch.equal(out, ref), (name, shape, (out != ref).float().mean().item())
    assert pk.device_error() == 0


def test_pair_gemm_feeds_next_rmsnorm(pk):
    """The fused GEMM2 + next-layer RMSNorm through the pair kernel."""
    import torch
    M, d, ffn = 512, 1024, 2048
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(M, d, device="cuda", generator=g).bfloat16()
    gm = (1 + 0.1 * torch.randn(d, device="cuda", generator=g)).bfloat16()
    w1 = (torch.randn(d, ffn, device="cuda", generator=g) / 32).bfloat16()
    b1 = (0.02 * torch.randn(ffn, device="cuda", generator=g)).bfloat16()
    w2 = (torch.randn(ffn, d, device="cuda", generator=g) / 45).bfloat16()
    b2 = (0.02 * torch.randn(d, device="cuda", generator=g)).bfloat16()
    fn = lambda: pk.ops.mlp_block_rmsnorm_next(x, gm, w1, b1, w2, b2, gm)  # noqa: E731
    (y0, yn0), _ = _forced(pk, None, fn)
    (y1, yn1), _ = _forced(pk, PAIR, fn)
    assert torch.equal(y0, y1) and torch.equal(yn0, yn1)
    assert pk.device_error() == 0


def test_pair_gemm_speed_config5(pk):
    """Informational: config-5 GEMM1 / GEMM2 (M=16384) with the pair kernel
    against the single-SM default."""
    import torch
    M, d, ffn = 16384, 8192, 28672
    g = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randn(M, d, device="cuda", generator=g).bfloat16()
    w1 = (torch.randn(d, ffn, device="cuda", generator=g) / 90).bfloat16()
    b1 = (0.02 * torch.randn(ffn, device="cuda", generator=g)).bfloat16()
    h = pk.ops.fused_matmul_bias_gelu(x, w1, b1)
    w2 = (torch.randn(ffn, d, device="cuda", generator=g) / 170).bfloat16()
    b2 = (0.02 * torch.randn(d, device="cuda", generator=g)).bfloat16()
    res = {}
    for cfg_name, cfg in (("single_sm", None), ("pair", PAIR)):
        for gname, fn, fl in (("gemm1", lambda: pk.ops.fused_matmul_bias_gelu(x, w1, b1), 2.0 * M * d * ffn),
                              ("gemm2", lambda: pk.ops.matmul_bias_residual(h, w2, b2, x), 2.0 * M * d * ffn)):
            def timed():
                for _ in range(2):
                    fn()
                torch.cuda.synchronize()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(5):
                    fn()
                e1.record()
                torch.cuda.synchronize()
                return e0.elapsed_time(e1) / 5
            ms, _ = _forced(pk, cfg, timed)
            res[f"{cfg_name}_{gname}"] = round(fl / (ms * 1e-3) / 1e12, 1)
    print("TFLOP/s", res)
    assert pk.device_error() == 0
