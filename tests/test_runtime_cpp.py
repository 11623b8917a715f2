"""CPU: the C++ runtime (include/pkb200_runtime.h) built with g++ against
libpkb200.so and run GPU-free (tests/cpp/runtime_test.cpp)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "polykernel_b200", "_lib")
CUDA_INC = "/usr/local/cuda/include"
CUDA_LIB = "/usr/local/cuda/lib64"


def test_cpp_runtime(tmp_path):
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    if not os.path.exists(os.path.join(LIBDIR, "libpkb200.so")):
        pytest.skip("libpkb200.so not built")
    exe = tmp_path / "runtime_test"
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-Werror",
           "-I", os.path.join(ROOT, "include"), "-I", CUDA_INC,
           os.path.join(ROOT, "tests", "cpp", "runtime_test.cpp"), "-o", str(exe),
           "-L", LIBDIR, "-lpkb200", f"-Wl,-rpath,{LIBDIR}"]
    if os.path.isdir(CUDA_LIB):
        cmd += ["-L", CUDA_LIB, f"-Wl,-rpath,{CUDA_LIB}", f"-Wl,-rpath-link,{CUDA_LIB}"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    from polykernel_b200 import tuning as T
    corr = {"cosine": 1.0, "max_rel_err": 0.0, "pcc": 1.0}
    doc = T.merge({"version": 1, "entries": []}, [
        T.entry("sm_100", "fused_matmul_bias_gelu", 2048, 16384, 4096,
                dict(T.DEFAULT, block_n=128, shared_memory_stages=6), 0.12, True, corr),
        T.entry("sm_100", "matmul", 64, 64, 64, T.DEFAULT, None, False, corr)])
    T.save(doc, tmp_path / "py_cache.json")
    r = subprocess.run([str(exe), str(tmp_path), str(tmp_path / "py_cache.json")],
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and "ALL PASSED" in r.stdout, r.stdout + r.stderr


def test_cpp_runtime_real_detectors(tmp_path):
    """CudaDeviceDetector (built with PKB200_RUNTIME_CUDA) and the library-backed
    detector agree: "sm_100" on a B200, a typed detection failure without one."""
    if shutil.which("g++") is None or not os.path.isdir(CUDA_LIB):
        pytest.skip("g++ or the CUDA runtime library not available")
    if not os.path.exists(os.path.join(LIBDIR, "libpkb200.so")):
        pytest.skip("libpkb200.so not built")
    exe = tmp_path / "detect_probe"
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-Werror", "-DPKB200_RUNTIME_CUDA",
           "-I", os.path.join(ROOT, "include"), "-I", CUDA_INC,
           os.path.join(ROOT, "tests", "cpp", "detect_probe.cpp"), "-o", str(exe),
           "-L", LIBDIR, "-lpkb200", f"-Wl,-rpath,{LIBDIR}",
           "-L", CUDA_LIB, "-lcudart", f"-Wl,-rpath,{CUDA_LIB}"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    import torch
    if torch.cuda.is_available():
        assert "cuda=sm_100 library=sm_100" in r.stdout
        assert "no tuned kernel for sm_100/matmul/M=8,N=8,K=8,bf16" in r.stdout
    else:
        assert "cuda=none library=none" in r.stdout
        assert "device detection failed" in r.stdout
