"""Generate the golden fixtures in this directory from the REFERENCE's own golden
module (meillaya/polykernel tests/golden/golden.py, quant_golden.py).

Run in a container where the reference checkout exists:
    python tests/golden/make_fixtures.py [--ref /path/to/polykernel]
The fixtures (golden_*.npz, bf16 stored as raw uint16 bits) are committed; the
GPU tests and the oracle self-tests read only those files, never the reference.

Cases mirror the reference's own tests (test_golden_self.py, test_cuda_run.py,
test_attention.py, test_quant.py incl. its fp8 simulation, tests/e2e mini-MLP) plus the BASELINE config-1
fragment and shapes that exercise the tensor-core tiles (multi-tile, partial
tiles, two-source KV).
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=None,
                    help="reference checkout (default: $PK_REFERENCE, else BASELINE.json's "
                         "reference_path)")
    args = ap.parse_args()
    if args.ref is None:
        sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
        from __graft_entry__ import reference_checkout
        args.ref = reference_checkout()
        if args.ref is None:
            raise SystemExit("reference checkout not found: pass --ref or set PK_REFERENCE")
    sys.path.insert(0, os.path.join(args.ref, "tests", "golden"))
    import ml_dtypes  # noqa: F401
    import golden as G  # the reference golden
    import quant_golden as QG

    BF = ml_dtypes.bfloat16
    bits = lambda a: np.asarray(a, dtype=BF).view(np.uint16)  # noqa: E731
    rng = np.random.default_rng(0xC0FFEE)  # the reference's fixture seed (conftest.py:15)

    def uni(shape):  # reference fixtures: uniform[-1, 1) (tests/kernels/conftest.py:82-83)
        return rng.uniform(-1.0, 1.0, size=shape).astype(np.float32).astype(BF)

    def causal_mask(sq, skv):  # tests/kernels/test_attention.py:299-303
        i = np.arange(sq)[:, None]
        j = np.arange(skv)[None, :]
        return np.where(j <= (skv - sq + i), 0.0, -1e9).astype(BF).reshape(1, 1, sq, skv)

    # ---------------------------------------------------------- known answers
    ka = {}
    a = np.array([[1, 2], [3, 4]], dtype=np.float32).astype(BF)
    b = np.array([[5, 6], [7, 8]], dtype=np.float32).astype(BF)
    ka["mm_a"], ka["mm_b"], ka["mm_out"] = bits(a), bits(b), bits(G.matmul(a, b))
    g_in = np.array([0.0, 1.0, -1.0, 2.0, -3.0, 0.5], dtype=np.float32).astype(BF)
    ka["gelu_in"], ka["gelu_out"] = bits(g_in), bits(G.gelu(g_in))
    r_in = np.array([[1, 2, 3, 4]], dtype=np.float32).astype(BF)
    ka["rms_in"], ka["rms_out"] = bits(r_in), bits(G.rmsnorm(r_in))
    np.savez_compressed(os.path.join(HERE, "golden_known.npz"), **ka)

    # ----------------------------------------------------------- elementwise
    ew = {}
    x = uni((4, 64)); w = uni((64,))
    ew["rms_w_x"], ew["rms_w_w"], ew["rms_w_out"] = bits(x), bits(w), bits(G.rmsnorm(x, w))
    x = uni((5, 33))
    ew["rms_odd_x"], ew["rms_odd_out"] = bits(x), bits(G.rmsnorm(x))
    x = (rng.standard_normal(1000) * 3).astype(np.float32).astype(BF)
    ew["gelu_x"], ew["gelu_out"] = bits(x), bits(G.gelu(x))
    np.savez_compressed(os.path.join(HERE, "golden_elementwise.npz"), **ew)

    # ---------------------------------------------------------------- GEMMs
    gm = {}
    for name, (M, K, N) in {"sq": (128, 128, 128), "odd": (130, 65, 127), "rect": (64, 128, 96),
                            "bigk": (64, 1024, 64), "tiles": (300, 256, 520)}.items():
        A, B = uni((M, K)), uni((K, N))
        bias_ = uni((N,))
        gm[f"{name}_a"], gm[f"{name}_b"], gm[f"{name}_bias"] = bits(A), bits(B), bits(bias_)
        gm[f"{name}_mm"] = bits(G.matmul(A, B))
        gm[f"{name}_frm"] = bits(G.fused_rmsnorm_matmul(A, B))
        gm[f"{name}_fbg"] = bits(G.fused_matmul_bias_gelu(A, B, bias_))
    np.savez_compressed(os.path.join(HERE, "golden_gemm.npz"), **gm)

    # ------------------------------------------ BASELINE config 1 (seed 0, N(0,1))
    r0 = np.random.default_rng(0)
    X = r0.standard_normal((128, 512)).astype(np.float32).astype(BF)
    gamma = (1 + 0.1 * r0.standard_normal(512)).astype(np.float32).astype(BF)
    W = (r0.standard_normal((512, 512)) / np.sqrt(512)).astype(np.float32).astype(BF)
    c1 = {"x": bits(X), "gamma": bits(gamma), "w": bits(W),
          "out": bits(G.fused_rmsnorm_matmul(X, W, gamma, 1e-6))}
    np.savez_compressed(os.path.join(HERE, "golden_config1.npz"), **c1)

    # -------------------------------------------------------------- MLP block
    mlp = {}
    for name, (M, d, ffn) in {"mini": (32, 64, 128), "mid": (192, 256, 512)}.items():
        r = np.random.default_rng(1 if name == "mini" else 2)
        X = r.standard_normal((M, d)).astype(np.float32).astype(BF)
        g_ = (1 + 0.1 * r.standard_normal(d)).astype(np.float32).astype(BF)
        W1 = (r.standard_normal((d, ffn)) / np.sqrt(d)).astype(np.float32).astype(BF)
        b1 = (0.02 * r.standard_normal(ffn)).astype(np.float32).astype(BF)
        W2 = (r.standard_normal((ffn, d)) / np.sqrt(ffn)).astype(np.float32).astype(BF)
        b2 = (0.02 * r.standard_normal(d)).astype(np.float32).astype(BF)
        h = G.fused_matmul_bias_gelu(G.rmsnorm(X, g_, 1e-6), W1, b1)
        Y = G.add(G.bias(G.matmul(h, W2), b2), X)
        for k_, v_ in dict(x=X, gamma=g_, w1=W1, b1=b1, w2=W2, b2=b2, y=Y).items():
            mlp[f"{name}_{k_}"] = bits(v_)
    np.savez_compressed(os.path.join(HERE, "golden_mlp.npz"), **mlp)

    # -------------------------------------------------------------- attention
    at = {}
    cases = {"sq32": (1, 2, 32, 32), "mh": (2, 4, 16, 64), "d40": (1, 1, 24, 40),
             "s33": (1, 2, 33, 32), "d128": (1, 2, 256, 128), "d64odd": (1, 2, 200, 64)}
    for name, (B_, H_, S_, D_) in cases.items():
        q, k, v = uni((B_, H_, S_, D_)), uni((B_, H_, S_, D_)), uni((B_, H_, S_, D_))
        empty = np.zeros((B_, H_, 0, D_), dtype=BF)
        o, _, _ = G.fused_kv_append_attention(q, k, v, empty, empty, causal_mask(S_, S_))
        at[f"{name}_q"], at[f"{name}_k"], at[f"{name}_v"], at[f"{name}_o"] = map(bits, (q, k, v, o))
    # non-causal
    q, k, v = uni((1, 2, 128, 128)), uni((1, 2, 192, 128)), uni((1, 2, 192, 128))
    empty = np.zeros((1, 2, 0, 128), dtype=BF)
    o, _, _ = G.fused_kv_append_attention(q, k, v, empty, empty, None)
    at["full_q"], at["full_k"], at["full_v"], at["full_o"] = map(bits, (q, k, v, o))
    # fused append (preallocated cache semantics are checked in the tests)
    for name, (B_, H_, Sc, Sn, D_) in {"app32": (1, 2, 8, 16, 32), "app128": (1, 2, 128, 256, 128),
                                       "app64odd": (1, 2, 100, 160, 64)}.items():
        q = uni((B_, H_, Sn, D_))
        kn, vn = uni((B_, H_, Sn, D_)), uni((B_, H_, Sn, D_))
        kc, vc = uni((B_, H_, Sc, D_)), uni((B_, H_, Sc, D_))
        o, nk, nv = G.fused_kv_append_attention(q, kn, vn, kc, vc, causal_mask(Sn, Sc + Sn))
        for k_, v_ in dict(q=q, kn=kn, vn=vn, kc=kc, vc=vc, o=o, nk=nk, nv=nv).items():
            at[f"{name}_{k_}"] = bits(v_)
    np.savez_compressed(os.path.join(HERE, "golden_attention.npz"), **at)

    # ------------------------------------------------------------------- int8
    q8 = {}
    A = uni((64, 128))
    wq = rng.integers(-127, 128, size=(128, 96)).astype(np.int8)
    sc = rng.uniform(0.001, 0.02, size=96).astype(np.float32).astype(BF).astype(np.float32)
    q8["a"], q8["wq"], q8["scale"], q8["out"] = bits(A), wq, sc, bits(QG.matmul_int8(A, wq, sc))
    Wf = uni((128, 96))
    wq2, sc2 = QG.quantize_per_channel(Wf)
    q8["w_float"], q8["wq_pc"], q8["scale_pc"] = bits(Wf), wq2, sc2
    q8["out_pc"] = bits(QG.matmul_int8(A, wq2, sc2))
    np.savez_compressed(os.path.join(HERE, "golden_int8.npz"), **q8)
    # ------------------------------------------- next-row ops (residual+norm, QKV)
    nx = {}
    x = uni((6, 256)); res = uni((6, 256)); w = uni((256,))
    nx["frr_x"], nx["frr_res"], nx["frr_w"] = bits(x), bits(res), bits(w)
    nx["frr_out"] = bits(G.fused_residual_rmsnorm(x, res, w, 1e-6))
    B_, S_, H_, Dh = 2, 64, 4, 64
    x = uni((B_, S_, H_ * Dh)); wqkv = uni((H_ * Dh, 3 * H_ * Dh))
    q, k, v = G.qkv_projection(x, wqkv, num_heads=H_)   # [B, S, H, Dh] each
    nx["qkv_x"], nx["qkv_w"] = bits(x), bits(wqkv)
    nx["qkv_q"], nx["qkv_k"], nx["qkv_v"] = bits(q), bits(k), bits(v)
    np.savez_compressed(os.path.join(HERE, "golden_next.npz"), **nx)
    # -------------------------------------------- fp8 weight path (simulated)
    f8 = {}
    for fmt, dt in (("e4m3", ml_dtypes.float8_e4m3fn), ("e5m2", ml_dtypes.float8_e5m2)):
        for (m, k, n) in ((128, 128, 128), (192, 160, 224)):  # test_quant.py:205-206
            a, w = uni((m, k)), uni((k, n))
            key = f"{fmt}_{m}x{k}x{n}"
            f8[f"{key}_a"], f8[f"{key}_w"] = bits(a), bits(w)
            f8[f"{key}_out"] = bits(QG.matmul_fp8_sim(a, w, fmt))
        # rounding edge values within the format's range: ties, subnormals,
        # values next to max-finite, signed zeros (the golden's ml_dtypes cast)
        lim = 448.0 if fmt == "e4m3" else 57344.0
        mags = np.concatenate([
            rng.uniform(0, 1, 512), rng.uniform(0, lim, 512),
            np.exp2(rng.uniform(-20, -5, 512)), [0.0, lim, lim * 0.97, 2.0 ** -9, 2.0 ** -16,
                                                 1.0625, 1.1875, 0.015625 * 1.0625]])
        sgn = np.where(rng.uniform(size=mags.shape) < 0.5, -1.0, 1.0)
        e = (sgn * mags).astype(np.float32).astype(BF)
        e = e[np.abs(e.astype(np.float32)) <= lim]
        f8[f"{fmt}_edge_in"] = bits(e)
        f8[f"{fmt}_edge_code"] = e.astype(dt).view(np.uint8)
    np.savez_compressed(os.path.join(HERE, "golden_fp8.npz"), **f8)
    # -------------------------------------------------- softmax (cuda_run op)
    sm = {}
    for name, shape in (("tokens_vocab", (64, 256)), ("odd", (32, 127)),  # test_cuda_run.py:366-378
                        ("flat3d", (2, 16, 64)), ("long", (4, 5000))):
        x = uni(shape) if name != "long" else (4 * rng.standard_normal(shape)).astype(np.float32).astype(BF)
        sm[f"{name}_x"], sm[f"{name}_y"] = bits(x), bits(G.softmax(x))
    np.savez_compressed(os.path.join(HERE, "golden_softmax.npz"), **sm)
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
