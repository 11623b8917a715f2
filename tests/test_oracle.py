"""CPU: the NumPy oracle pinned against the reference golden's fixtures and the
reference's own C++ CPU code (oracle/_ref, built from its sources)."""
import ctypes
import os

import numpy as np
import pytest

from oracle import golden_np as O
from oracle import metrics as Mx
from tests.helpers import check_gate

F = O.from_bits
REF_LIB = os.path.join(os.path.dirname(os.path.dirname(__file__)), "oracle", "_ref",
                       "liboracle_ref.so")


def test_bf16_rounding_rne_and_nan():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, np.inf, -0.0, 3.0e38], np.float32)
    # 1 + 2^-8 is a tie -> even (1.0); 1 + 3*2^-8 -> rounds up to 1 + 2^-6
    assert O.bf16(x)[0] == 1.0 and O.bf16(x)[1] == 1.0 and O.bf16(x)[2] == 1.015625
    assert np.isinf(O.bf16(x)[4]) and np.signbit(O.bf16(x)[5])
    assert np.isnan(O.bf16(np.array([np.nan], np.float32)))[0]


def test_known_answers(golden):
    g = golden("known")
    mm = O.matmul(F(g["mm_a"]), F(g["mm_b"]))
    assert np.array_equal(mm, np.array([[19, 22], [43, 50]], np.float32))
    assert np.array_equal(O.to_bits(mm), g["mm_out"])
    assert np.array_equal(O.to_bits(O.gelu(F(g["gelu_in"]))), g["gelu_out"])
    assert O.gelu(F(g["gelu_in"]))[0] == 0.0
    assert abs(O.gelu(F(g["gelu_in"]))[1] - 0.8413) < 4e-3
    assert np.array_equal(O.to_bits(O.rmsnorm(F(g["rms_in"]))), g["rms_out"])


def test_elementwise_bit_exact(golden):
    g = golden("elementwise")
    assert np.array_equal(O.to_bits(O.rmsnorm(F(g["rms_w_x"]), F(g["rms_w_w"]))), g["rms_w_out"])
    assert np.array_equal(O.to_bits(O.rmsnorm(F(g["rms_odd_x"]))), g["rms_odd_out"])
    assert np.array_equal(O.to_bits(O.gelu(F(g["gelu_x"]))), g["gelu_out"])


@pytest.mark.parametrize("name", ["sq", "odd", "rect", "bigk", "tiles"])
def test_gemm_family_bit_exact(golden, name):
    g = golden("gemm")
    a, b, bias = F(g[f"{name}_a"]), F(g[f"{name}_b"]), F(g[f"{name}_bias"])
    assert np.array_equal(O.to_bits(O.matmul(a, b)), g[f"{name}_mm"])
    assert np.array_equal(O.to_bits(O.fused_rmsnorm_matmul(a, b)), g[f"{name}_frm"])
    assert np.array_equal(O.to_bits(O.fused_matmul_bias_gelu(a, b, bias)), g[f"{name}_fbg"])


def test_config1_bit_exact(golden):
    g = golden("config1")
    out = O.fused_rmsnorm_matmul(F(g["x"]), F(g["w"]), F(g["gamma"]), 1e-6)
    assert np.array_equal(O.to_bits(out), g["out"])


@pytest.mark.parametrize("name", ["mini", "mid"])
def test_mlp_block_bit_exact(golden, name):
    g = golden("mlp")
    a = {k: F(g[f"{name}_{k}"]) for k in ("x", "gamma", "w1", "b1", "w2", "b2")}
    y = O.mlp_block(a["x"], a["gamma"], a["w1"], a["b1"], a["w2"], a["b2"], 1e-6)
    assert np.array_equal(O.to_bits(y), g[f"{name}_y"])


@pytest.mark.parametrize("name", ["sq32", "mh", "d40", "s33", "d128", "d64odd"])
def test_attention_matches_golden(golden, name):
    g = golden("attention")
    o = O.attention_prefill(F(g[f"{name}_q"]), F(g[f"{name}_k"]), F(g[f"{name}_v"]), True)
    # The golden divides by sqrt(D) and masks with an additive -1e9; the oracle
    # multiplies by 1/sqrt(D) and masks with -inf: equal up to fp32 rounding.
    check_gate(o, F(g[f"{name}_o"]), min_exact=0.97)


def test_attention_full_matches_golden(golden):
    g = golden("attention")
    o = O.attention_prefill(F(g["full_q"]), F(g["full_k"]), F(g["full_v"]), False)
    check_gate(o, F(g["full_o"]), min_exact=0.97)


@pytest.mark.parametrize("name", ["app32", "app128", "app64odd"])
def test_attention_append_matches_golden(golden, name):
    g = golden("attention")
    t = {k: F(g[f"{name}_{k}"]) for k in ("q", "kn", "vn", "kc", "vc", "o", "nk", "nv")}
    B, H, Sc, D = t["kc"].shape
    Sn = t["kn"].shape[2]
    kc = np.zeros((B, H, Sc + Sn + 7, D), np.float32)
    vc = np.zeros_like(kc)
    kc[:, :, :Sc], vc[:, :, :Sc] = t["kc"], t["vc"]
    o, nk, nv = O.attention_prefill_kv_append(t["q"], t["kn"], t["vn"], kc, vc, Sc)
    check_gate(o, t["o"], min_exact=0.97)
    assert np.array_equal(nk[:, :, :Sc + Sn], t["nk"]) and np.array_equal(nv[:, :, :Sc + Sn], t["nv"])
    assert not nk[:, :, Sc + Sn:].any()


def test_leaky_mask_fails_gate(golden):
    # Negative pin (tests/kernels/test_attention.py:447-463): dropping the causal
    # mask must fail the gate.
    g = golden("attention")
    leaked = O.attention_prefill(F(g["sq32_q"]), F(g["sq32_k"]), F(g["sq32_v"]), False)
    assert Mx.cosine(leaked, F(g["sq32_o"])) < 0.99


def test_int8_matches_quant_golden(golden):
    g = golden("int8")
    out = O.matmul_int8(F(g["a"]), g["wq"], g["scale"])
    assert np.array_equal(O.to_bits(out), g["out"])
    out = O.matmul_int8(F(g["a"]), g["wq_pc"], g["scale_pc"])
    assert np.array_equal(O.to_bits(out), g["out_pc"])
    # wrong per-channel scale must fail the quant gate (test_quant.py:224-260)
    bad = O.matmul_int8(F(g["a"]), g["wq"], g["scale"][::-1].copy())
    assert not Mx.passes(Mx.report(bad, F(g["out"])), quant=True)


# ------------------------------------------------ reference C++ CPU (oracle/_ref)
@pytest.fixture(scope="module")
def reflib():
    if not os.path.exists(REF_LIB):
        pytest.skip("oracle/_ref not built (built by __graft_entry__.build())")
    lib = ctypes.CDLL(REF_LIB)
    return lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def test_reference_cpu_mlp_matches_oracle(golden, reflib):
    g = golden("mlp")
    name = "mini"
    x = g[f"{name}_x"]
    M, d = x.shape
    ffn = g[f"{name}_w1"].shape[1]
    y = np.zeros_like(x)
    args = [np.ascontiguousarray(g[f"{name}_{k}"]) for k in ("x", "gamma", "w1", "b1", "w2", "b2")]
    reflib.ref_mlp_rows(*[_p(a) for a in args], _p(y), ctypes.c_int64(M), ctypes.c_int64(d),
                        ctypes.c_int64(ffn), ctypes.c_float(1e-6))
    # The C++ reference sums in a sequential order, NumPy in blocks: near-exact.
    check_gate(F(y), F(g[f"{name}_y"]), rel_ceiling=5e-2, min_exact=0.95)


def test_reference_cpu_fused_rmsnorm_matmul_matches_oracle(golden, reflib):
    g = golden("gemm")
    a, b = np.ascontiguousarray(g["sq_a"]), np.ascontiguousarray(g["sq_b"])
    out = np.zeros((a.shape[0], b.shape[1]), np.uint16)
    reflib.ref_fused_rmsnorm_matmul(_p(a), _p(b), _p(out), ctypes.c_int64(a.shape[0]),
                                    ctypes.c_int64(b.shape[1]), ctypes.c_int64(a.shape[1]),
                                    ctypes.c_float(1e-5))
    check_gate(F(out), F(g["sq_frm"]), min_exact=0.95)


def test_parity_rule_accepts_reference_cpu_at_config1(golden, reflib):
    """The GPU parity rule (tests/helpers.check_parity) is pinned to the
    reference's own behaviour: its C++ CPU code, run on BASELINE config 1,
    passes it (while missing the strict max_rel_err <= 1e-2 on near-zero outputs)."""
    from tests.helpers import check_parity
    g = golden("config1")
    x, w, gm = (np.ascontiguousarray(g[k]) for k in ("x", "w", "gamma"))
    xn = np.zeros_like(x)
    out = np.zeros((x.shape[0], w.shape[1]), np.uint16)
    reflib.ref_rmsnorm(_p(x), _p(gm), _p(xn), ctypes.c_int64(128), ctypes.c_int64(512),
                       ctypes.c_float(1e-6))
    reflib.ref_matmul(_p(xn), _p(w), _p(out), ctypes.c_int64(128), ctypes.c_int64(512),
                      ctypes.c_int64(512))
    m = check_parity(F(out), F(g["out"]))
    assert m["max_rel_err"] > Mx.MAX_REL_ERR_THRESHOLD  # the strict gate alone would reject it


def test_next_row_fragments_bit_exact(golden):
    g = golden("next")
    out = O.fused_residual_rmsnorm(F(g["frr_x"]), F(g["frr_res"]), F(g["frr_w"]), 1e-6)
    assert np.array_equal(O.to_bits(out), g["frr_out"])
    q, k, v = O.qkv_projection(F(g["qkv_x"]), F(g["qkv_w"]), 4)
    for a, key in ((q, "qkv_q"), (k, "qkv_k"), (v, "qkv_v")):
        assert np.array_equal(O.to_bits(a), g[key])


# ----------------------------------------------------------- fp8 weight path
@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_fp8_rounding_matches_golden_cast(golden, fmt):
    """fp8_round + fp8_bits reproduce the golden's ml_dtypes cast code for code
    on ties, subnormals, values next to max-finite and signed zeros."""
    g = golden("fp8")
    x = F(g[f"{fmt}_edge_in"])
    r = O.fp8_round(x, fmt)
    assert np.array_equal(O.fp8_bits(r, fmt), g[f"{fmt}_edge_code"])
    assert np.array_equal(O.fp8_decode(g[f"{fmt}_edge_code"], fmt), r)


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_fp8_code_table_round_trip(fmt):
    codes = np.arange(256, dtype=np.uint8)
    v = O.fp8_decode(codes, fmt)
    finite = np.isfinite(v)
    assert np.array_equal(O.fp8_bits(O.fp8_round(v[finite], fmt), fmt), codes[finite])
    assert np.array_equal(O.bf16(v[finite]), v[finite])  # every fp8 value is a bf16 value


@pytest.mark.parametrize("case", ["e4m3_128x128x128", "e4m3_192x160x224",
                                  "e5m2_128x128x128", "e5m2_192x160x224"])
def test_fp8_sim_matmul_bit_exact(golden, case):
    g = golden("fp8")
    fmt = case.split("_")[0]
    out = O.matmul_fp8_sim(F(g[f"{case}_a"]), F(g[f"{case}_w"]), fmt)
    assert np.array_equal(O.to_bits(out), g[f"{case}_out"])


def fp8_edge_weights(fmt):
    """Values that exercise saturation and rounding at the top of the range,
    where the golden's ml_dtypes cast and the reference's CPU code differ."""
    lim = 448.0 if fmt == "e4m3" else 57344.0
    v = np.array([lim, lim * 1.03, lim * 1.07, lim * 4, 1e30, 3e38, 1.0, 1.0625, 1.1875,
                  2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -11, 2.0 ** -16, 2.0 ** -17, 3 * 2.0 ** -18,
                  0.0], np.float32)
    return O.bf16(np.concatenate([v, -v]))


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_reference_cpu_fp8_rounding_matches_oracle(tmp_path, fmt):
    """The reference's own CPU driver (oracle/_ref/matmul_quant fp8sim) with an
    identity A returns fp8(W) itself: pins fp8_round's saturation and rounding."""
    import subprocess
    exe = os.path.join(os.path.dirname(REF_LIB), "matmul_quant")
    if not os.path.exists(exe):
        pytest.skip("oracle/_ref not built (built by __graft_entry__.build())")
    w = fp8_edge_weights(fmt).reshape(4, 8)
    eye = np.eye(4, dtype=np.float32)
    np.save(tmp_path / "a.npy", O.to_bits(eye).view("V2"))
    np.save(tmp_path / "w.npy", O.to_bits(w).view("V2"))
    subprocess.run([exe, "fp8sim", fmt, str(tmp_path / "a.npy"), str(tmp_path / "w.npy"),
                    str(tmp_path / "c.npy")], check=True, capture_output=True)
    c = F(np.load(tmp_path / "c.npy").view(np.uint16))
    # compared as values: the driver's fp32 sum turns fp8(-0) into +0
    assert np.array_equal(c, O.fp8_round(w, fmt))


@pytest.mark.parametrize("name", ["tokens_vocab", "odd", "flat3d", "long"])
def test_softmax_bit_exact(golden, name):
    g = golden("softmax")
    assert np.array_equal(O.to_bits(O.softmax(F(g[f"{name}_x"]))), g[f"{name}_y"])


@pytest.mark.parametrize("name", ["sq", "odd", "tiles"])
def test_fused_equals_unfused_bit_exact(golden, name):
    """The fused ops are the unfused chains with the same rounding points
    (the reference's test_golden_self.py:91-124)."""
    g = golden("gemm")
    a, b, bias = F(g[f"{name}_a"]), F(g[f"{name}_b"]), F(g[f"{name}_bias"])
    assert np.array_equal(O.to_bits(O.fused_rmsnorm_matmul(a, b)),
                          O.to_bits(O.matmul(O.rmsnorm(a), b)))
    assert np.array_equal(O.to_bits(O.fused_matmul_bias_gelu(a, b, bias)),
                          O.to_bits(O.gelu(O.bias(O.matmul(a, b), bias))))


def test_gate_rejects_transposed_operand_and_corruption(golden):
    """Negative pins on the CPU oracle: a transposed B (the reference's mma_bad,
    test_mma.py:288-328) and a scaled output (--corrupt, test_mlp_correctness.py:
    199-208) both fail the gate the GPU tests apply."""
    from tests.helpers import check_parity
    g = golden("gemm")
    a, b = F(g["sq_a"]), F(g["sq_b"])
    ref = F(g["sq_mm"])
    with pytest.raises(AssertionError):
        check_parity(O.matmul(a, np.ascontiguousarray(b.T)), ref)
    with pytest.raises(AssertionError):
        check_parity(O.bf16(ref * 1.5), ref)
    check_parity(O.matmul(a, b), ref)
