"""GPU parity of the fp8 (e4m3fn / e5m2) weight path: the encode and decode
kernels exhaustively against the oracle's fp8_round (the reference's CPU
fp8_round, kernels/cpu/matmul_quant.cpp:130-150, pinned to its driver and to
the golden's ml_dtypes cast by tests/test_oracle.py), and the weight-only fp8
GEMM against the golden's matmul_fp8_sim fixtures (the shapes of the
reference's tests/kernels/test_quant.py:205-218) and the oracle at mid sizes."""
import math

import numpy as np
import pytest

from oracle import golden_np as O
from tests.helpers import bits_from_t, check_gate, check_parity, f32_from_t, t_from_bits

pytestmark = pytest.mark.gpu
F = O.from_bits
FMTS = ["e4m3", "e5m2"]


@pytest.fixture(scope="module")
def pk(cuda):
    import polykernel_b200 as pk
    pk.lib()
    return pk


def _codes(t):
    import torch
    return t.view(torch.uint8).cpu().numpy()


@pytest.mark.parametrize("fmt", FMTS)
def test_encode_every_bf16_value(pk, fmt):
    """All 65536 bf16 bit patterns (NaNs, infs, subnormals, both zeros)."""
    allbits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    got = _codes(pk.ops.quantize_fp8(t_from_bits(allbits), fmt))
    x = F(allbits)
    want = O.fp8_bits(O.fp8_round(x, fmt), fmt)
    nan = np.isnan(x)
    assert np.array_equal(got[~nan], want[~nan])
    assert np.all((got[nan] & 0x7F) == 0x7F)


@pytest.mark.parametrize("fmt", FMTS)
def test_decode_every_code(pk, fmt):
    import torch
    codes = np.arange(256, dtype=np.uint8)
    dt = pk.ops.FP8_FORMATS[fmt][1]
    got = f32_from_t(pk.ops.dequantize_fp8(torch.from_numpy(codes).cuda().view(dt)))
    want = O.fp8_decode(codes, fmt)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(O.to_bits(got[~nan]), O.to_bits(want[~nan]))  # signed zeros too


@pytest.mark.parametrize("fmt", FMTS)
def test_unaligned_and_ragged_lengths(pk, fmt):
    """Offsets that break 16-byte alignment and lengths that are not a multiple
    of 8 take the scalar path; results match the vector path element for element."""
    import torch
    rng = np.random.default_rng(5)
    bits = O.to_bits(rng.standard_normal(4099).astype(np.float32) * 3)
    w = t_from_bits(bits)
    full = _codes(pk.ops.quantize_fp8(w, fmt))
    for off, n in ((1, 4095), (3, 17), (0, 4099), (8, 7)):
        part = _codes(pk.ops.quantize_fp8(w[off:off + n], fmt))
        assert np.array_equal(part, full[off:off + n])
    q = pk.ops.quantize_fp8(w, fmt)
    deq = bits_from_t(pk.ops.dequantize_fp8(q[1:4096]))
    assert np.array_equal(deq, O.to_bits(O.fp8_round(F(bits[1:4096]), fmt)))
    # the reference's ABI takes a length of 0 as a no-op
    empty = torch.empty(0, dtype=torch.bfloat16, device="cuda")
    assert pk.ops.quantize_fp8(empty, fmt).numel() == 0


@pytest.mark.parametrize("case", ["e4m3_128x128x128", "e4m3_192x160x224",
                                  "e5m2_128x128x128", "e5m2_192x160x224"])
def test_fp8_sim_vs_golden(golden, pk, case):
    """The reference's fp8-sim fixtures (test_quant.py:205-218) with the
    reference's quant gate (quant_golden.py:46-48) and a bit-exact floor."""
    g = golden("fp8")
    fmt = case.split("_")[0]
    a, w = t_from_bits(g[f"{case}_a"]), t_from_bits(g[f"{case}_w"])
    before = pk.path_counters()
    sim = pk.ops.matmul_fp8_sim(a, w, fmt)
    assert pk.path_counters()["gemm_tc"] > before["gemm_tc"]  # the tcgen05 GEMM ran
    check_gate(f32_from_t(sim), F(g[f"{case}_out"]), rel_ceiling=5e-2, min_exact=0.99, quant=True)
    # weights resident as fp8: the same bits as the simulated path
    res = pk.ops.matmul_fp8(a, pk.ops.quantize_fp8(w, fmt))
    assert np.array_equal(bits_from_t(res), bits_from_t(sim))


@pytest.mark.parametrize("fmt", FMTS)
def test_fp8_gemm_mid_vs_oracle(pk, fmt):
    rng = np.random.default_rng(23)
    for (M, K, N) in ((1024, 2048, 1536), (333, 4096, 264)):
        A = O.to_bits(rng.standard_normal((M, K)).astype(np.float32))
        W = O.to_bits((rng.standard_normal((K, N)) / math.sqrt(K)).astype(np.float32))
        wq = pk.ops.quantize_fp8(t_from_bits(W), fmt)
        out = f32_from_t(pk.ops.matmul_fp8(t_from_bits(A), wq))
        ref = O.matmul_fp8_sim(F(A), F(W), fmt)
        ref64 = O.matmul_fp8_sim(F(A), F(W), fmt, acc=np.float64)
        check_parity(out, ref, ref64, rel_ceiling=5e-2)


def test_fp8_matches_bf16_gemm_of_dequantized_weights(pk):
    """The fp8 GEMM is the bf16 GEMM on the exactly expanded weights."""
    rng = np.random.default_rng(29)
    A = t_from_bits(O.to_bits(rng.standard_normal((512, 1024)).astype(np.float32)))
    W = t_from_bits(O.to_bits((rng.standard_normal((1024, 768)) / 32).astype(np.float32)))
    for fmt in FMTS:
        wq = pk.ops.quantize_fp8(W, fmt)
        assert np.array_equal(bits_from_t(pk.ops.matmul_fp8(A, wq)),
                              bits_from_t(pk.ops.matmul(A, pk.ops.dequantize_fp8(wq))))


def test_fp8_rejects_bad_arguments(pk):
    import torch
    a = torch.zeros(4, 8, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(8, 8, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        pk.ops.matmul_fp8_sim(a, w, "e3m4")
    with pytest.raises(TypeError):
        pk.ops.matmul_fp8(a, w)  # bf16 weights are not fp8 codes
    assert pk.lib().pkb200_matmul_fp8_sim(a.data_ptr(), w.data_ptr(), a.data_ptr(), 4, 8, 8, 7,
                                          None) != 0


_NARROW_SCRIPT = r"""
import sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
import polykernel_b200 as pk
from oracle import golden_np as O
from tests.helpers import bits_from_t, t_from_bits
kind = sys.argv[2]
rng = np.random.default_rng(31)
M, K, N = 640, 1536, 1024
A = t_from_bits(O.to_bits(rng.standard_normal((M, K)).astype(np.float32)))
if kind == "int8":
    q = torch.from_numpy(rng.integers(-128, 128, size=(K, N + 8), dtype=np.int8)).cuda()
    sc = torch.from_numpy((rng.random(N + 8) * 0.02 + 0.001).astype(np.float32)).cuda()
    wide = pk.ops.matmul_int8(A, q, sc)
    narrow = pk.ops.matmul_int8(A, q[:, :N].contiguous(), sc[:N].contiguous())
else:
    W = t_from_bits(O.to_bits((rng.standard_normal((K, N + 8)) / 32).astype(np.float32)))
    wq = pk.ops.quantize_fp8(W, kind)
    wide = pk.ops.matmul_fp8(A, wq)
    narrow = pk.ops.matmul_fp8(A, wq[:, :N].contiguous())
assert np.array_equal(bits_from_t(narrow), bits_from_t(wide[:, :N].contiguous()))
assert pk.device_error() == 0
print("ok")
"""


@pytest.mark.parametrize("kind", ["int8", "e4m3", "e5m2"])
def test_narrow_weights_in_gemm_match_expanded_path(kind):
    """With PKB200_NARROW_GEMM=1, weights stored as 1-byte codes are expanded
    inside the tensor-core GEMM when N is a multiple of 16; other widths expand
    into a bf16 workspace first. Both give the same bits: the same weights
    padded to a width of N + 8 (expanded path) agree with width N (in-GEMM path)
    column for column. Run in a child process, since the switch is read once."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, PKB200_NARROW_GEMM="1")
    r = subprocess.run([sys.executable, "-c", _NARROW_SCRIPT, root, kind], env=env, cwd=root,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr
