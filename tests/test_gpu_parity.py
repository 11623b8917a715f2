"""GPU parity: the CUDA library (through the C ABI) against the reference golden
fixtures and the oracle, at fixture sizes, mid sizes and (row/head samples of)
the BASELINE configs' full sizes.

Gate (the reference's own, tests/golden/metrics.py:20-23 and
tests/kernels/test_cuda_run.py:262-288): cosine >= 0.999, PCC >= 0.99, bit-exact
fraction floor, and max_rel_err <= 1e-2 for short reductions (K <= 128) or the
reference's calibrated 5e-2 for long reductions (test_cuda_run.py:93). For the
full-size MLP rows the near-zero outputs make max_rel_err reduction-order noise
(the reference's own CPU code misses 1e-2 against its golden there); those tests
also bound the error against an fp64-accumulated oracle.
"""
import math

import numpy as np
import pytest

from oracle import golden_np as O
from oracle import metrics as Mx
from tests.helpers import (bits_from_t, check_attention, check_chain, check_gate, check_parity,
                           f32_from_t,
                           t_from_bits)

pytestmark = pytest.mark.gpu
F = O.from_bits


@pytest.fixture(scope="module")
def pk(cuda):
    import polykernel_b200 as pk
    pk.lib()
    return pk


def _counters(pk):
    return pk.path_counters()


def _used(pk, before, key):
    return pk.path_counters()[key] > before[key]


@pytest.mark.parametrize("name", ["sq", "odd", "rect", "bigk", "tiles"])
def test_gemm_family_vs_golden(golden, pk, name):
    g = golden("gemm")
    a, b, bias = (t_from_bits(g[f"{name}_{k}"]) for k in ("a", "b", "bias"))
    af, bf, biasf = (F(g[f"{name}_{k}"]) for k in ("a", "b", "bias"))
    K = a.shape[1]
    c0 = _counters(pk)
    outs = {"mm": pk.ops.matmul(a, b), "frm": pk.ops.fused_rmsnorm_matmul(a, b),
            "fbg": pk.ops.fused_matmul_bias_gelu(a, b, bias)}
    ref64 = {"mm": O.matmul(af, bf, acc=np.float64),
             "frm": O.fused_rmsnorm_matmul(af, bf, acc=np.float64),
             "fbg": O.fused_matmul_bias_gelu(af, bf, biasf, acc=np.float64)}
    for key, out in outs.items():
        print(name, key, check_parity(f32_from_t(out), F(g[f"{name}_{key}"]), ref64[key]))
    aligned = (K % 8 == 0) and (b.shape[1] % 8 == 0)
    assert _used(pk, c0, "gemm_tc" if aligned else "gemm_simt")
    assert pk.device_error() == 0


def test_config1_fused_rmsnorm_matmul(golden, pk):
    g = golden("config1")
    x, w, gamma = (t_from_bits(g[k]) for k in ("x", "w", "gamma"))
    c0 = _counters(pk)
    out = f32_from_t(pk.ops.fused_rmsnorm_matmul(x, w, gamma, eps=1e-6))
    assert _used(pk, c0, "gemm_tc")
    ref64 = O.fused_rmsnorm_matmul(F(g["x"]), F(g["w"]), F(g["gamma"]), 1e-6, acc=np.float64)
    print("config1", check_parity(out, F(g["out"]), ref64))


@pytest.mark.parametrize("name", ["mini", "mid"])
def test_mlp_block_vs_golden(golden, pk, name):
    g = golden("mlp")
    t = {k: t_from_bits(g[f"{name}_{k}"]) for k in ("x", "gamma", "w1", "b1", "w2", "b2")}
    f = {k: F(g[f"{name}_{k}"]) for k in ("x", "gamma", "w1", "b1", "w2", "b2")}
    y = pk.ops.mlp_block(t["x"], t["gamma"], t["w1"], t["b1"], t["w2"], t["b2"], eps=1e-6)
    ref64 = O.mlp_block(f["x"], f["gamma"], f["w1"], f["b1"], f["w2"], f["b2"], 1e-6,
                        acc=np.float64)
    print(name, check_parity(f32_from_t(y), F(g[f"{name}_y"]), ref64, min_exact=0.98))
    assert pk.device_error() == 0


@pytest.mark.parametrize("name", ["sq32", "mh", "d40", "s33", "d128", "d64odd"])
def test_attention_vs_golden(golden, pk, name):
    g = golden("attention")
    q, k, v = (t_from_bits(g[f"{name}_{x}"]) for x in ("q", "k", "v"))
    c0 = _counters(pk)
    o = pk.ops.attention_prefill(q, k, v, causal=True)
    ref64 = O.attention_prefill(F(g[f"{name}_q"]), F(g[f"{name}_k"]), F(g[f"{name}_v"]), True,
                                acc=np.float64)
    m = check_attention(f32_from_t(o), F(g[f"{name}_o"]), s_kv=k.shape[2], ref64_f32=ref64)
    print(name, m)
    tc = q.shape[3] in (64, 128)
    assert _used(pk, c0, "attn_tc" if tc else "attn_simt")
    assert pk.device_error() == 0


def test_attention_noncausal_vs_golden(golden, pk):
    g = golden("attention")
    q, k, v = (t_from_bits(g[f"full_{x}"]) for x in ("q", "k", "v"))
    o = pk.ops.attention_prefill(q, k, v, causal=False)
    ref64 = O.attention_prefill(F(g["full_q"]), F(g["full_k"]), F(g["full_v"]), False,
                                acc=np.float64)
    print("full", check_attention(f32_from_t(o), F(g["full_o"]), s_kv=k.shape[2], ref64_f32=ref64))


def test_attention_leaky_mask_fails(golden, pk):
    g = golden("attention")
    q, k, v = (t_from_bits(g[f"d128_{x}"]) for x in ("q", "k", "v"))
    o = pk.ops.attention_prefill(q, k, v, causal=False)
    assert Mx.cosine(f32_from_t(o), F(g["d128_o"])) < 0.99


@pytest.mark.parametrize("name", ["app32", "app128", "app64odd"])
def test_attention_kv_append_vs_golden(golden, pk, name):
    import torch
    g = golden("attention")
    t = {k: t_from_bits(g[f"{name}_{k}"]) for k in ("q", "kn", "vn", "kc", "vc")}
    B, H, Sc, D = t["kc"].shape
    Sn = t["kn"].shape[2]
    Smax = Sc + Sn + 37
    gen = torch.Generator(device="cuda").manual_seed(7)
    kc = torch.randn(B, H, Smax, D, device="cuda", generator=gen).to(torch.bfloat16)
    vc = torch.randn(B, H, Smax, D, device="cuda", generator=gen).to(torch.bfloat16)
    kc[:, :, :Sc] = t["kc"]
    vc[:, :, :Sc] = t["vc"]
    tail_k, tail_v = kc[:, :, Sc + Sn:].clone(), vc[:, :, Sc + Sn:].clone()
    o = pk.ops.attention_prefill_kv_append(t["q"], t["kn"], t["vn"], kc, vc, Sc, causal=True)
    ref64 = O.attention_prefill(F(g[f"{name}_q"]), F(g[f"{name}_nk"]), F(g[f"{name}_nv"]), True,
                                acc=np.float64)
    print(name, check_attention(f32_from_t(o), F(g[f"{name}_o"]), s_kv=Sc + Sn, ref64_f32=ref64))
    assert np.array_equal(bits_from_t(kc[:, :, :Sc + Sn]), g[f"{name}_nk"])
    assert np.array_equal(bits_from_t(vc[:, :, :Sc + Sn]), g[f"{name}_nv"])
    assert torch.equal(kc[:, :, Sc + Sn:], tail_k) and torch.equal(vc[:, :, Sc + Sn:], tail_v)
    assert pk.device_error() == 0


def test_kv_cache_update_bit_exact(pk):
    import torch
    for D in (32, 40, 128):
        cache = torch.randn(2, 3, 9, D, device="cuda").to(torch.bfloat16)
        new = torch.randn(2, 3, 14, D, device="cuda").to(torch.bfloat16)
        out = pk.ops.kv_cache_update(cache, new)
        assert torch.equal(out, torch.cat([cache, new], dim=2))


def test_rmsnorm_gelu_vs_golden(golden, pk):
    g = golden("elementwise")
    y = pk.ops.rmsnorm(t_from_bits(g["rms_w_x"]), t_from_bits(g["rms_w_w"]))
    check_gate(f32_from_t(y), F(g["rms_w_out"]), min_exact=0.99)
    y = pk.ops.rmsnorm(t_from_bits(g["rms_odd_x"]))
    check_gate(f32_from_t(y), F(g["rms_odd_out"]), min_exact=0.99)
    y = pk.ops.gelu(t_from_bits(g["gelu_x"]))
    check_gate(f32_from_t(y), F(g["gelu_out"]), min_exact=0.99)


def test_int8_vs_quant_golden(golden, pk):
    import torch
    g = golden("int8")
    a = t_from_bits(g["a"])
    for wq, sc, out in (("wq", "scale", "out"), ("wq_pc", "scale_pc", "out_pc")):
        w = torch.from_numpy(g[wq]).cuda()
        s = torch.from_numpy(g[sc].astype(np.float32)).cuda()
        c = pk.ops.matmul_int8(a, w, s)
        check_gate(f32_from_t(c), F(g[out]), rel_ceiling=5e-2, quant=True)


# ------------------------------------------------------------- mid sizes ----
def _rand_bits(rng, shape, std=1.0, mean=0.0):
    return O.to_bits((mean + std * rng.standard_normal(shape)).astype(np.float32))


def test_gemm_mid_vs_oracle(pk):
    rng = np.random.default_rng(11)
    for (M, K, N) in ((1024, 2048, 1536), (333, 4096, 264), (2048, 512, 4096)):
        A = _rand_bits(rng, (M, K))
        B = _rand_bits(rng, (K, N), 1 / math.sqrt(K))
        out = f32_from_t(pk.ops.matmul(t_from_bits(A), t_from_bits(B)))
        ref = O.matmul(F(A), F(B))
        ref64 = O.matmul(F(A), F(B), acc=np.float64)
        m = Mx.report(out, ref, ref64)
        print((M, K, N), m)
        assert m["cosine"] >= 0.9999 and m["bit_exact"] >= 0.9


def test_mlp_mid_vs_oracle(pk):
    rng = np.random.default_rng(12)
    M, d, ffn = 512, 1024, 4096
    X = _rand_bits(rng, (M, d)); gm = _rand_bits(rng, (d,), 0.1, 1.0)
    W1 = _rand_bits(rng, (d, ffn), 1 / math.sqrt(d)); b1 = _rand_bits(rng, (ffn,), 0.02)
    W2 = _rand_bits(rng, (ffn, d), 1 / math.sqrt(ffn)); b2 = _rand_bits(rng, (d,), 0.02)
    y = pk.ops.mlp_block(*(t_from_bits(a) for a in (X, gm, W1, b1, W2, b2)), eps=1e-6)
    ref = O.mlp_block(F(X), F(gm), F(W1), F(b1), F(W2), F(b2), 1e-6)
    m = Mx.report(f32_from_t(y), ref)
    print("mlp mid", m)
    assert m["cosine"] >= 0.9999 and m["pcc"] >= 0.99 and m["bit_exact"] >= 0.9


def test_attention_mid_vs_oracle(pk):
    rng = np.random.default_rng(13)
    B, H, S, D = 1, 4, 1024, 128
    q, k, v = (_rand_bits(rng, (B, H, S, D)) for _ in range(3))
    o = pk.ops.attention_prefill(*(t_from_bits(a) for a in (q, k, v)), causal=True)
    ref = O.attention_prefill(F(q), F(k), F(v), True)
    ref64 = O.attention_prefill(F(q), F(k), F(v), True, acc=np.float64)
    print("attn mid", check_attention(f32_from_t(o), ref, s_kv=S, ref64_f32=ref64))


def test_fused_residual_rmsnorm_vs_golden(golden, pk):
    g = golden("next")
    x, res, w = (t_from_bits(g[k]) for k in ("frr_x", "frr_res", "frr_w"))
    out, ssum = pk.ops.fused_residual_rmsnorm(x, res, w, eps=1e-6, return_sum=True)
    check_gate(f32_from_t(out), F(g["frr_out"]), min_exact=0.99)
    assert np.array_equal(bits_from_t(ssum), O.to_bits(O.add(F(g["frr_x"]), F(g["frr_res"]))))


def test_qkv_projection_feeds_attention(golden, pk):
    g = golden("next")
    x, w = t_from_bits(g["qkv_x"]), t_from_bits(g["qkv_w"])
    q, k, v = pk.ops.qkv_projection(x, w, num_heads=4)
    Kd = g["qkv_w"].shape[0]
    xf, wf = F(g["qkv_x"]), F(g["qkv_w"])
    ref64 = np.split(O.matmul(xf, wf, acc=np.float64), 3, axis=-1)
    for t, key, r64 in ((q, "qkv_q", ref64[0]), (k, "qkv_k", ref64[1]), (v, "qkv_v", ref64[2])):
        gold = F(g[key]).transpose(0, 2, 1, 3)                 # golden [B,S,H,Dh] -> [B,H,S,Dh]
        r64 = r64.reshape(gold.shape[0], gold.shape[2], gold.shape[1], gold.shape[3]).transpose(0, 2, 1, 3)
        print(key, check_parity(f32_from_t(t), np.ascontiguousarray(gold), r64))
    o = pk.ops.attention_prefill(q, k, v, causal=True)       # the layout attention consumes
    qf, kf, vf = (f32_from_t(t) for t in (q, k, v))
    check_attention(f32_from_t(o), O.attention_prefill(qf, kf, vf), s_kv=k.shape[2],
                    ref64_f32=O.attention_prefill(qf, kf, vf, acc=np.float64))
    assert Kd == 256


# ---------------------------------------------------------------- softmax ----
@pytest.mark.parametrize("name", ["tokens_vocab", "odd", "flat3d", "long"])
def test_softmax_vs_golden(golden, pk, name):
    """launch_softmax (the op the reference's cuda_run_main.cpp:64 declares)
    against the golden's softmax fixtures (test_cuda_run.py:366-378 shapes plus
    a long row): CUDA expf vs NumPy exp and the sum order differ by a few fp32
    ulps, so a few bf16 outputs may sit one ulp away."""
    g = golden("softmax")
    x = t_from_bits(g[f"{name}_x"])
    y = pk.ops.softmax(x)
    assert tuple(y.shape) == tuple(x.shape)
    check_gate(f32_from_t(y), F(g[f"{name}_y"]), min_exact=0.97)


# ------------------------------------------------- fused == unfused, negatives ----
@pytest.mark.parametrize("name", ["sq", "odd", "tiles"])
def test_device_fused_equals_unfused(golden, pk, name):
    """On the device the fused entry points give the unfused chains' bits
    (the reference's test_golden_self.py:91-124, here through the C ABI)."""
    g = golden("gemm")
    a, b, bias = (t_from_bits(g[f"{name}_{k}"]) for k in ("a", "b", "bias"))
    assert np.array_equal(bits_from_t(pk.ops.fused_rmsnorm_matmul(a, b)),
                          bits_from_t(pk.ops.matmul(pk.ops.rmsnorm(a), b)))
    # bias + GELU: the epilogue and the standalone GELU kernel share one GELU
    # routine; the bias add rounds to bf16 in both (torch's bf16 add rounds
    # the fp32 sum to nearest even, as golden.bias does)
    unfused = pk.ops.gelu((pk.ops.matmul(a, b) + bias).contiguous())
    fused = pk.ops.fused_matmul_bias_gelu(a, b, bias)
    exact = float(np.mean(bits_from_t(fused) == bits_from_t(unfused)))
    assert exact >= 0.999, exact
    check_gate(f32_from_t(fused), f32_from_t(unfused), min_exact=0.999)


def test_device_gate_rejects_transposed_operand_and_corruption(golden, pk):
    """A GEMM fed the transposed B (the reference's mma_bad) and a corrupted
    output (--corrupt) fail the gate the passing kernel meets."""
    g = golden("gemm")
    a, b = t_from_bits(g["sq_a"]), t_from_bits(g["sq_b"])
    ref = F(g["sq_mm"])
    good = f32_from_t(pk.ops.matmul(a, b))
    check_parity(good, ref)
    bad = f32_from_t(pk.ops.matmul(a, b.t().contiguous()))
    with pytest.raises(AssertionError):
        check_parity(bad, ref)
    with pytest.raises(AssertionError):
        check_parity(O.bf16(good * 1.5), ref)


# ----------------------------------------------- fp16 P.V range fallback --
def _attn_case(rng, shape, v_scale=1.0):
    q, k = (_rand_bits(rng, shape) for _ in range(2))
    v = O.to_bits(O.bf16(rng.standard_normal(shape).astype(np.float32) * np.float32(v_scale)))
    return q, k, v


def test_attention_normal_values_take_no_exact_fallback(pk):
    rng = np.random.default_rng(21)
    q, k, v = _attn_case(rng, (2, 4, 384, 128))
    before = pk.attention_exact_ctas()
    o = pk.ops.attention_prefill(*(t_from_bits(a) for a in (q, k, v)), causal=True)
    assert pk.attention_exact_ctas() == before
    check_attention(f32_from_t(o), O.attention_prefill(F(q), F(k), F(v), True), s_kv=384,
                    ref64_f32=O.attention_prefill(F(q), F(k), F(v), True, acc=np.float64))


@pytest.mark.parametrize("kind", ["beyond_fp16_max", "all_tiny"])
def test_attention_values_outside_fp16_take_exact_fallback(pk, kind):
    """V values fp16 cannot carry (|v| >= 2^16, a head whose values are all
    tiny) make the affected CTAs recompute their rows exactly: the output still
    meets the gate, and the counter shows the fallback ran."""
    rng = np.random.default_rng(22)
    shape = (1, 3, 320, 64)
    if kind == "all_tiny":
        q, k, v = _attn_case(rng, shape, v_scale=1e-7)
    else:
        q, k, v = _attn_case(rng, shape)
        vf = F(v)
        vf[0, 1, 5, 3] = 2.0 ** 17
        v = O.to_bits(vf)
    before = pk.attention_exact_ctas()
    o = pk.ops.attention_prefill(*(t_from_bits(a) for a in (q, k, v)), causal=True)
    assert pk.attention_exact_ctas() > before
    got, ref = f32_from_t(o), O.attention_prefill(F(q), F(k), F(v), True)
    check_attention(got, ref, s_kv=320,
                    ref64_f32=O.attention_prefill(F(q), F(k), F(v), True, acc=np.float64))
    assert pk.device_error() == 0


def test_attention_append_with_fallback_keeps_cache_bf16(pk):
    """The appended V rows are the caller's bf16 values even when the tile is
    also rewritten as fp16 for the P.V pass (and when the fallback runs)."""
    import torch
    rng = np.random.default_rng(23)
    B, H, Sc, Sn, D, Smax = 1, 2, 128, 256, 128, 512
    q, kn, vn = _attn_case(rng, (B, H, Sn, D))
    vnf = F(vn)
    vnf[0, 0, 200, 7] = 3.0e5          # beyond fp16 range: bf16 keeps it
    vn = O.to_bits(vnf)
    kc = torch.zeros(B, H, Smax, D, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    kcf, vcf = (_rand_bits(rng, (B, H, Sc, D)) for _ in range(2))
    kc[:, :, :Sc] = t_from_bits(kcf)
    vc[:, :, :Sc] = t_from_bits(vcf)
    o = pk.ops.attention_prefill_kv_append(*(t_from_bits(a) for a in (q, kn, vn)), kc, vc, Sc,
                                           causal=True)
    assert np.array_equal(bits_from_t(vc[:, :, Sc:Sc + Sn]), vn)
    assert np.array_equal(bits_from_t(kc[:, :, Sc:Sc + Sn]), kn)
    keys = np.concatenate([F(kcf), F(kn)], axis=2)
    vals = np.concatenate([F(vcf), F(vn)], axis=2)
    ref = O.attention_prefill(F(q), keys, vals, True)
    check_attention(f32_from_t(o), ref, s_kv=Sc + Sn,
                    ref64_f32=O.attention_prefill(F(q), keys, vals, True, acc=np.float64))
    assert pk.device_error() == 0


@pytest.mark.parametrize("cols", [1032, 4096, 8192])
@pytest.mark.parametrize("with_gamma", [True, False])
def test_rmsnorm_wide_rows_vs_oracle(pk, cols, with_gamma):
    """Rows of 1025..8192 columns take the register-resident kernel (one CTA per
    row); same rounding as the golden (golden.py:83-90)."""
    rng = np.random.default_rng(cols)
    x = _rand_bits(rng, (67, cols))
    g = _rand_bits(rng, (cols,), 0.1, 1.0) if with_gamma else None
    c0 = _counters(pk)
    out = pk.ops.rmsnorm(t_from_bits(x), t_from_bits(g) if with_gamma else None, 1e-6)
    assert _used(pk, c0, "other")
    ref = O.rmsnorm(F(x), F(g) if with_gamma else None, 1e-6)
    got = f32_from_t(out)
    assert np.mean(got == ref) >= 0.99
    # any difference is one bf16 ulp (the fp32 sum of squares in another order)
    diff = np.abs(got - ref)
    assert np.all(diff <= 2.0 ** -7 * np.abs(ref) + 1e-30)


@pytest.mark.parametrize("shape", [(256, 512, 1024), (300, 1024, 2048), (130, 72, 136)],
                         ids=["tiles", "ragged_m", "simt_fallback"])
def test_mlp_block_with_next_rmsnorm_vs_golden(pk, shape):
    """Y = MLP block and Yn = rmsnorm(Y; gamma2) (golden.fused_residual_rmsnorm
    on the block's output and residual) with the sum of squares taken from
    GEMM2's epilogue; Y is bit-identical to pkb200_mlp_block."""
    M, d, ffn = shape
    rng = np.random.default_rng(M + d)
    X = _rand_bits(rng, (M, d)); gm = _rand_bits(rng, (d,), 0.1, 1.0)
    W1 = _rand_bits(rng, (d, ffn), 1 / math.sqrt(d)); b1 = _rand_bits(rng, (ffn,), 0.02)
    W2 = _rand_bits(rng, (ffn, d), 1 / math.sqrt(ffn)); b2 = _rand_bits(rng, (d,), 0.02)
    g2 = _rand_bits(rng, (d,), 0.1, 1.0)
    t = [t_from_bits(a) for a in (X, gm, W1, b1, W2, b2, g2)]
    y, yn = pk.ops.mlp_block_rmsnorm_next(*t[:6], gamma_next=t[6], eps=1e-6, eps_next=1e-5)
    y_ref_dev = pk.ops.mlp_block(*t[:6], eps=1e-6)
    import torch
    assert torch.equal(y, y_ref_dev)
    # the golden composition on the device's Y (isolates the fused normalisation)
    ref = O.fused_residual_rmsnorm(
        O.bias(O.matmul(O.fused_matmul_bias_gelu(O.rmsnorm(F(X), F(gm), 1e-6), F(W1), F(b1)),
                        F(W2)), F(b2)), F(X), F(g2), 1e-5)
    on_y = O.rmsnorm(f32_from_t(y), F(g2), 1e-5)
    got = f32_from_t(yn)
    assert np.mean(got == on_y) >= 0.99
    assert np.all(np.abs(got - on_y) <= 2.0 ** -7 * np.abs(on_y) + 1e-30)
    # against the golden composition from X: the bf16 chain's one-ulp flips in
    # Y propagate (the rule of the full-size chain tests)
    print(shape, check_chain(got, ref))
    assert pk.device_error() == 0


def test_next_rmsnorm_timing_vs_unfused(pk):
    """Informational: GEMM2 + the standalone row RMSNorm against the fused
    epilogue + apply pass, config-2 shape."""
    import time

    import torch
    M, d, ffn = 2048, 4096, 16384
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(M, d, device="cuda", generator=g).bfloat16()
    gm = (1 + 0.1 * torch.randn(d, device="cuda", generator=g)).bfloat16()
    w1 = (torch.randn(d, ffn, device="cuda", generator=g) / 64).bfloat16()
    b1 = (0.02 * torch.randn(ffn, device="cuda", generator=g)).bfloat16()
    w2 = (torch.randn(ffn, d, device="cuda", generator=g) / 128).bfloat16()
    b2 = (0.02 * torch.randn(d, device="cuda", generator=g)).bfloat16()

    def unfused():
        y = pk.ops.mlp_block(x, gm, w1, b1, w2, b2)
        return pk.ops.rmsnorm(y, gm, 1e-6)

    def fused():
        return pk.ops.mlp_block_rmsnorm_next(x, gm, w1, b1, w2, b2, gm)[1]

    res = {}
    for name, fn in (("unfused", unfused), ("fused", fused)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(10):
            fn()
        torch.cuda.synchronize()
        res[name] = (time.perf_counter() - t0) / 10 * 1e3
    print("ms", res)
    # the same normalisation up to the order of the fp32 sum of squares
    assert (unfused() == fused()).float().mean().item() >= 0.99
