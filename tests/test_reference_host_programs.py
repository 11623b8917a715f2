"""The reference's own host programs, built unmodified from its sources by
oracle/Makefile and linked against libpkb200 instead of the reference's
kernels: its .npy launcher (lib/Runtime/cuda_run_main.cpp) and its timing
driver (benchmarks/bench_cuda.cpp). That they link proves the drop-in symbol
boundary (every launch_* they declare, with the reference's mangling). CPU:
link evidence and the usage path. GPU: the reference's harness runs the golden
fixtures through these kernels, and its bench driver times them."""
import json
import os
import subprocess

import numpy as np
import pytest

from oracle import golden_np as O
from tests.helpers import check_gate, check_parity

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_RUN = os.path.join(ROOT, "oracle", "_ref", "ref_cuda_run_over_pkb200")
REF_BENCH = os.path.join(ROOT, "oracle", "_ref", "ref_bench_cuda_over_pkb200")
LIB = os.path.join(ROOT, "polykernel_b200", "_lib", "libpkb200.so")
F = O.from_bits


def _need(path):
    if not os.path.exists(path):
        pytest.skip(f"{os.path.relpath(path, ROOT)} not built (built by __graft_entry__.build())")
    return path


def _run(*args, exe=REF_RUN):
    return subprocess.run([_need(exe), *map(str, args)], capture_output=True, text=True,
                          timeout=300)


def _save(path, bits):
    np.save(path, np.ascontiguousarray(bits, dtype=np.uint16).view("V2"))


def _load(path):
    a = np.load(path)
    assert a.dtype == np.dtype("V2")
    return a.view(np.uint16)


def _nm(path, *flags):
    return subprocess.run(["nm", "-D", *flags, path], capture_output=True, text=True,
                          check=True).stdout


@pytest.mark.parametrize("exe", [REF_RUN, REF_BENCH])
def test_reference_programs_resolve_launch_symbols_here(exe):
    _need(exe)
    undefined = {ln.split()[-1] for ln in _nm(exe, "--undefined-only").splitlines()
                 if "launch_" in ln}
    assert undefined, "expected the reference's launch_* references"
    defined = {ln.split()[-1] for ln in _nm(LIB, "--defined-only").splitlines()}
    assert undefined <= defined, undefined - defined
    ldd = subprocess.run(["ldd", exe], capture_output=True, text=True).stdout
    assert "libpkb200.so" in ldd


def test_reference_harness_usage_path():
    r = _run()
    assert r.returncode == 2 and "usage: cuda_run" in r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["sq", "odd", "tiles"])
def test_reference_harness_gemm_ops(golden, cuda, tmp_path, name):
    g = golden("gemm")
    for k in ("a", "b", "bias"):
        _save(tmp_path / f"{k}.npy", g[f"{name}_{k}"])
    a, b = tmp_path / "a.npy", tmp_path / "b.npy"
    assert _run("matmul", a, b, tmp_path / "mm.npy").returncode == 0
    assert _run("fused_rmsnorm_matmul", a, b, tmp_path / "frm.npy").returncode == 0
    assert _run("fused_matmul_bias_gelu", a, b, tmp_path / "bias.npy",
                tmp_path / "fbg.npy").returncode == 0
    af, bf, biasf = (F(g[f"{name}_{k}"]) for k in ("a", "b", "bias"))
    ref64 = {"mm": O.matmul(af, bf, acc=np.float64),
             "frm": O.fused_rmsnorm_matmul(af, bf, acc=np.float64),
             "fbg": O.fused_matmul_bias_gelu(af, bf, biasf, acc=np.float64)}
    for key in ("mm", "frm", "fbg"):
        check_parity(F(_load(tmp_path / f"{key}.npy")), F(g[f"{name}_{key}"]), ref64[key])


@pytest.mark.gpu
def test_reference_harness_elementwise_ops(golden, cuda, tmp_path):
    g = golden("elementwise")
    _save(tmp_path / "x.npy", g["rms_w_x"])
    _save(tmp_path / "w.npy", g["rms_w_w"])
    assert _run("rmsnorm", tmp_path / "x.npy", tmp_path / "y.npy", "--weight",
                tmp_path / "w.npy").returncode == 0
    check_gate(F(_load(tmp_path / "y.npy")), F(g["rms_w_out"]), min_exact=0.99)
    _save(tmp_path / "gx.npy", g["gelu_x"])
    assert _run("gelu", tmp_path / "gx.npy", tmp_path / "gy.npy").returncode == 0
    check_gate(F(_load(tmp_path / "gy.npy")), F(g["gelu_out"]), min_exact=0.99)
    s = golden("softmax")
    _save(tmp_path / "sx.npy", s["odd_x"])
    assert _run("softmax", tmp_path / "sx.npy", tmp_path / "sy.npy").returncode == 0
    check_gate(F(_load(tmp_path / "sy.npy")), F(s["odd_y"]), min_exact=0.97)


@pytest.mark.gpu
def test_reference_bench_driver_times_these_kernels(cuda):
    r = _run("--M", "512", "--N", "1024", "--K", "1024", "--warmup", "2", "--iters", "5",
             "--tune-iters", "5", "--json", exe=REF_BENCH)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1])
    assert line["measured"] and line["fused"]["median_ms"] > 0
    assert line["shape"] == {"M": 512, "N": 1024, "K": 1024}
