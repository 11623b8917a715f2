"""The .npy launcher harness (polykernel_b200/_lib/cuda_run), the reference's
`cuda_run <op> ...` command line (lib/Runtime/cuda_run_main.cpp:356) over this
library. CPU: usage/exit codes. GPU: ops against the golden fixtures, as the
reference's tests/kernels/test_cuda_run.py drives its harness."""
import os
import subprocess

import numpy as np
import pytest

from oracle import golden_np as O
from tests.helpers import check_attention, check_gate, check_parity

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "polykernel_b200", "_lib", "cuda_run")
F = O.from_bits


def _exe():
    if not os.path.exists(EXE):
        pytest.skip("cuda_run not built")
    return EXE


def _run(*args):
    return subprocess.run([_exe(), *map(str, args)], capture_output=True, text=True, timeout=300)


def _save(path, bits):
    np.save(path, np.ascontiguousarray(bits, dtype=np.uint16).view("V2"))


def _load(path):
    a = np.load(path)
    assert a.dtype == np.dtype("V2")
    return a.view(np.uint16)


def test_usage_exit_codes():
    assert _run().returncode == 2
    assert _run("no_such_op").returncode == 2
    assert _run("matmul", "only_one.npy").returncode == 2
    assert _run("rmsnorm", "a.npy", "b.npy", "--bogus", "1").returncode == 2


def test_missing_input_is_runtime_error(tmp_path):
    r = _run("gelu", tmp_path / "missing.npy", tmp_path / "out.npy")
    assert r.returncode == 1 and "cannot open" in r.stderr


def _bf(tmp_path, name, shape):
    path = tmp_path / f"{name}.npy"
    _save(path, np.zeros(shape, np.uint16))
    return path


def _bf0d(tmp_path, name):
    path = tmp_path / f"{name}.npy"
    np.save(path, np.zeros((), np.uint16).view("V2"))
    return path


def _i8(tmp_path, name, shape):
    path = tmp_path / f"{name}.npy"
    np.save(path, np.zeros(shape, np.int8))
    return path


def _f4(tmp_path, name, shape):
    path = tmp_path / f"{name}.npy"
    np.save(path, np.zeros(shape, np.float32))
    return path


@pytest.mark.parametrize("case", [
    "matmul_k", "matmul_rank", "matmul_0d", "frm_gamma", "fbg_bias", "int8_scale", "rmsnorm_w",
    "mlp_w1", "mlp_b1", "mlp_w2", "mlp_gamma", "attn_bhd", "attn_v", "kv_d", "append_cache",
    "append_scache", "fp8_k"])
def test_mismatched_shapes_rejected_before_device_work(tmp_path, case):
    """Every operand is checked against the primary one before any device
    allocation: a mismatched file exits 1 with a shape error (no GPU needed)."""
    t = tmp_path
    out = t / "out.npy"
    a = _bf(t, "a", (8, 16))
    args = {
        "matmul_k": lambda: ("matmul", a, _bf(t, "b", (15, 4)), out),
        "matmul_rank": lambda: ("matmul", a, _bf(t, "b", (16,)), out),
        "matmul_0d": lambda: ("matmul", _bf0d(t, "z"), _bf(t, "b", (1, 4)), out),
        "frm_gamma": lambda: ("fused_rmsnorm_matmul", a, _bf(t, "b", (16, 4)), out, "--weight",
                      _bf(t, "g", (15,))),
        "fbg_bias": lambda: ("fused_matmul_bias_gelu", a, _bf(t, "b", (16, 4)), _bf(t, "bias", (5,)), out),
        "int8_scale": lambda: ("matmul_int8", a, _i8(t, "wq", (16, 4)), _f4(t, "s", (3,)), out),
        "rmsnorm_w": lambda: ("rmsnorm", a, out, "--weight", _bf(t, "w", (8,))),
        "mlp_w1": lambda: ("mlp_block", a, _bf(t, "g", (16,)), _bf(t, "w1", (8, 32)), _bf(t, "b1", (32,)),
                   _bf(t, "w2", (32, 16)), _bf(t, "b2", (16,)), out),
        "mlp_b1": lambda: ("mlp_block", a, _bf(t, "g", (16,)), _bf(t, "w1", (16, 32)), _bf(t, "b1", (31,)),
                   _bf(t, "w2", (32, 16)), _bf(t, "b2", (16,)), out),
        "mlp_w2": lambda: ("mlp_block", a, _bf(t, "g", (16,)), _bf(t, "w1", (16, 32)), _bf(t, "b1", (32,)),
                   _bf(t, "w2", (32, 8)), _bf(t, "b2", (16,)), out),
        "mlp_gamma": lambda: ("mlp_block", a, _bf(t, "g", (17,)), _bf(t, "w1", (16, 32)),
                      _bf(t, "b1", (32,)), _bf(t, "w2", (32, 16)), _bf(t, "b2", (16,)), out),
        "attn_bhd": lambda: ("attention_prefill", _bf(t, "q", (1, 2, 8, 32)), _bf(t, "k", (1, 3, 8, 32)),
                     _bf(t, "v", (1, 3, 8, 32)), out),
        "attn_v": lambda: ("attention_prefill", _bf(t, "q", (1, 2, 8, 32)), _bf(t, "k", (1, 2, 8, 32)),
                   _bf(t, "v", (1, 2, 7, 32)), out),
        "kv_d": lambda: ("kv_cache_update", _bf(t, "c", (1, 2, 8, 32)), _bf(t, "n", (1, 2, 4, 16)), out),
        "append_cache": lambda: ("attention_append", _bf(t, "q", (1, 2, 8, 32)), _bf(t, "kn", (1, 2, 8, 32)),
                         _bf(t, "vn", (1, 2, 8, 32)), _bf(t, "kc", (1, 2, 16, 64)),
                         _bf(t, "vc", (1, 2, 16, 64)), out, t / "ko.npy", t / "vo.npy"),
        "append_scache": lambda: ("attention_append", _bf(t, "q", (1, 2, 8, 32)), _bf(t, "kn", (1, 2, 8, 32)),
                          _bf(t, "vn", (1, 2, 8, 32)), _bf(t, "kc", (1, 2, 16, 32)),
                          _bf(t, "vc", (1, 2, 16, 32)), out, t / "ko.npy", t / "vo.npy",
                          "--s-cache", "9"),
        "fp8_k": lambda: ("fp8sim", "e4m3", a, _bf(t, "w", (12, 4)), out),
    }[case]()
    r = _run(*args)
    assert r.returncode == 1 and "shape error" in r.stderr, (r.returncode, r.stderr)
    assert not out.exists()


@pytest.mark.gpu
def test_dev_and_neg(cuda):
    r = _run("dev")
    assert r.returncode == 0 and "COMPUTE_CAPABILITY 10.0" in r.stderr
    r = _run("neg")
    assert r.returncode == 1 and "PASS" in r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["sq", "odd", "tiles"])
def test_gemm_ops_through_harness(golden, cuda, tmp_path, name):
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
def test_rmsnorm_gelu_through_harness(golden, cuda, tmp_path):
    g = golden("elementwise")
    _save(tmp_path / "x.npy", g["rms_w_x"])
    _save(tmp_path / "w.npy", g["rms_w_w"])
    assert _run("rmsnorm", tmp_path / "x.npy", tmp_path / "y.npy", "--weight",
                tmp_path / "w.npy").returncode == 0
    check_gate(F(_load(tmp_path / "y.npy")), F(g["rms_w_out"]), min_exact=0.99)
    _save(tmp_path / "gx.npy", g["gelu_x"])
    assert _run("gelu", tmp_path / "gx.npy", tmp_path / "gy.npy").returncode == 0
    check_gate(F(_load(tmp_path / "gy.npy")), F(g["gelu_out"]), min_exact=0.99)


@pytest.mark.gpu
def test_mlp_and_attention_through_harness(golden, cuda, tmp_path):
    g = golden("mlp")
    names = ("x", "gamma", "w1", "b1", "w2", "b2")
    for k in names:
        _save(tmp_path / f"{k}.npy", g[f"mid_{k}"])
    assert _run("mlp_block", *[tmp_path / f"{k}.npy" for k in names], tmp_path / "y.npy",
                "--epsilon", "1e-6").returncode == 0
    check_parity(F(_load(tmp_path / "y.npy")), F(g["mid_y"]), min_exact=0.98)
    a = golden("attention")
    for k in ("q", "k", "v"):
        _save(tmp_path / f"{k}.npy", a[f"d128_{k}"])
    assert _run("attention_prefill", tmp_path / "q.npy", tmp_path / "k.npy", tmp_path / "v.npy",
                tmp_path / "o.npy").returncode == 0
    ref64 = O.attention_prefill(F(a["d128_q"]), F(a["d128_k"]), F(a["d128_v"]), True,
                                acc=np.float64)
    check_attention(F(_load(tmp_path / "o.npy")), F(a["d128_o"]), s_kv=256, ref64_f32=ref64)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_fp8sim_through_harness(golden, cuda, tmp_path, fmt):
    """`fp8sim <fmt> A W OUT`, the argument order of the reference's CPU driver
    (kernels/cpu/matmul_quant.cpp `fp8sim`), against its golden fixture."""
    g = golden("fp8")
    case = f"{fmt}_192x160x224"
    _save(tmp_path / "a.npy", g[f"{case}_a"])
    _save(tmp_path / "w.npy", g[f"{case}_w"])
    r = _run("fp8sim", fmt, tmp_path / "a.npy", tmp_path / "w.npy", tmp_path / "c.npy")
    assert r.returncode == 0 and "path=fp8_sim" in r.stderr, r.stderr
    check_gate(F(_load(tmp_path / "c.npy")), F(g[f"{case}_out"]), rel_ceiling=5e-2,
               min_exact=0.99, quant=True)


def test_fp8sim_usage():
    assert _run("fp8sim", "e3m4", "a.npy", "w.npy", "c.npy").returncode == 2


@pytest.mark.gpu
def test_softmax_through_harness(golden, cuda, tmp_path):
    """`softmax IN OUT [--axis A]` with the reference's arguments (last axis only)."""
    g = golden("softmax")
    _save(tmp_path / "x.npy", g["flat3d_x"])
    assert _run("softmax", tmp_path / "x.npy", tmp_path / "y.npy").returncode == 0
    check_gate(F(_load(tmp_path / "y.npy")), F(g["flat3d_y"]), min_exact=0.97)
    assert _run("softmax", tmp_path / "x.npy", tmp_path / "y.npy", "--axis", "0").returncode == 1


def test_softmax_usage():
    assert _run("softmax", "only_in.npy").returncode == 2
