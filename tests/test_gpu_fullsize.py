"""GPU parity at the BASELINE configs' full sizes, checked on samples the oracle
can afford: the MLP block is row-independent, so a few token rows of the full
[M, d] output are recomputed by the oracle from the same full weights; attention
is independent per (batch, head), so a few heads of the full [B, H, S, D] problem
are recomputed. Inputs follow BASELINE.json's distributions (seeded)."""
import math

import numpy as np
import pytest

from oracle import golden_np as O
from tests.helpers import bits_from_t, check_attention, check_chain, f32_from_t

pytestmark = pytest.mark.gpu


def _mlp_case(torch, M, d, ffn, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    bf = torch.bfloat16
    x = torch.randn(M, d, device="cuda", generator=g).to(bf)
    gamma = (1 + 0.1 * torch.randn(d, device="cuda", generator=g)).to(bf)
    w1 = (torch.randn(d, ffn, device="cuda", generator=g) / math.sqrt(d)).to(bf)
    b1 = (0.02 * torch.randn(ffn, device="cuda", generator=g)).to(bf)
    w2 = (torch.randn(ffn, d, device="cuda", generator=g) / math.sqrt(ffn)).to(bf)
    b2 = (0.02 * torch.randn(d, device="cuda", generator=g)).to(bf)
    return x, gamma, w1, b1, w2, b2


@pytest.mark.parametrize("cfg", [(2048, 4096, 16384), (16384, 8192, 28672)],
                         ids=["config2", "config5"])
def test_mlp_block_full_size_sampled_rows(cuda, cfg):
    import torch
    import polykernel_b200 as pk
    M, d, ffn = cfg
    x, gamma, w1, b1, w2, b2 = _mlp_case(torch, M, d, ffn, seed=0)
    y = pk.ops.mlp_block(x, gamma, w1, b1, w2, b2, eps=1e-6)
    rows = np.random.default_rng(1).choice(M, 8, replace=False)
    rows.sort()
    f = [f32_from_t(t) for t in (gamma, w1, b1, w2, b2)]
    ref = O.mlp_block(f32_from_t(x[rows]), *f, eps=1e-6)
    print(cfg, check_chain(f32_from_t(y[rows]), ref))
    assert pk.device_error() == 0


def test_int8_mlp_full_size_sampled_rows(cuda):
    import torch
    import polykernel_b200 as pk
    M, d, ffn = 4096, 4096, 14336
    g = torch.Generator(device="cuda").manual_seed(4)
    bf = torch.bfloat16
    x = torch.randn(M, d, device="cuda", generator=g).to(bf)
    gamma = (1 + 0.1 * torch.randn(d, device="cuda", generator=g)).to(bf)
    q1 = torch.randint(-127, 128, (d, ffn), device="cuda", generator=g, dtype=torch.int8)
    q2 = torch.randint(-127, 128, (ffn, d), device="cuda", generator=g, dtype=torch.int8)
    s1 = (0.001 + 0.019 * torch.rand(ffn, device="cuda", generator=g)).to(bf).float()
    s2 = (0.001 + 0.019 * torch.rand(d, device="cuda", generator=g)).to(bf).float()
    b1 = (0.02 * torch.randn(ffn, device="cuda", generator=g)).to(bf)
    b2 = (0.02 * torch.randn(d, device="cuda", generator=g)).to(bf)
    y = pk.ops.mlp_block_int8(x, gamma, q1, s1, b1, q2, s2, b2, eps=1e-6)
    rows = np.sort(np.random.default_rng(2).choice(M, 8, replace=False))
    args = (f32_from_t(x[rows]), f32_from_t(gamma), q1.cpu().numpy(), s1.cpu().numpy(),
            f32_from_t(b1), q2.cpu().numpy(), s2.cpu().numpy(), f32_from_t(b2))
    ref = O.mlp_block_int8(*args, eps=1e-6)
    print("config4", check_chain(f32_from_t(y[rows]), ref))


@pytest.mark.parametrize("s_cache", [0, 2048])
def test_attention_full_size_sampled_heads(cuda, s_cache):
    import torch
    import polykernel_b200 as pk
    B, H, S, D, S_max = 4, 32, 2048, 128, 4096
    g = torch.Generator(device="cuda").manual_seed(3)
    bf = torch.bfloat16
    q, kn, vn = (torch.randn(B, H, S, D, device="cuda", generator=g).to(bf) for _ in range(3))
    kc = torch.randn(B, H, S_max, D, device="cuda", generator=g).to(bf)
    vc = torch.randn(B, H, S_max, D, device="cuda", generator=g).to(bf)
    tail = kc[:, :, s_cache + S:].clone()
    o = pk.ops.attention_prefill_kv_append(q, kn, vn, kc, vc, s_cache, causal=True)
    assert torch.equal(kc[:, :, s_cache:s_cache + S], kn)           # appended in place
    assert torch.equal(kc[:, :, s_cache + S:], tail)                 # rest untouched
    for (b, h) in ((0, 0), (3, 31), (2, 17)):
        keys = f32_from_t(kc[b:b + 1, h:h + 1, :s_cache + S])
        vals = f32_from_t(vc[b:b + 1, h:h + 1, :s_cache + S])
        qh = f32_from_t(q[b:b + 1, h:h + 1])
        ref = O.attention_prefill(qh, keys, vals, causal=True)
        ref64 = O.attention_prefill(qh, keys, vals, causal=True, acc=np.float64)
        print(s_cache, (b, h), check_attention(f32_from_t(o[b:b + 1, h:h + 1]), ref,
                                               s_kv=s_cache + S, ref64_f32=ref64))
    assert pk.device_error() == 0


@pytest.mark.parametrize("shape", [(2048, 16384, 4096), (16384, 28672, 8192)],
                         ids=["config2_gemm2", "config5_gemm2"])
def test_gemm_bit_identical_to_cublas(cuda, shape):
    """The tensor-core GEMM matches the vendor library bit for bit (same fp32
    accumulation behaviour), and both sit at the golden's accuracy against an
    fp64 product once rounded to bf16."""
    import torch
    import polykernel_b200 as pk
    M, K, N = shape
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    b = (torch.randn(K, N, device="cuda", generator=g) / math.sqrt(K)).bfloat16()
    ours = pk.ops.matmul(a, b)
    lib_ref = torch.matmul(a, b)
    assert torch.equal(ours, lib_ref)
    rows = np.sort(np.random.default_rng(1).choice(M, 8, replace=False))
    gold = O.matmul(f32_from_t(a[rows]), f32_from_t(b))
    print(shape, check_chain(f32_from_t(ours[rows]), gold, min_exact=0.98))


# ------------------------------------------ the reference arm's exact inputs --
# bench.py's seeded NumPy draws (numpy.random.default_rng; fixed draw order per
# config), the same arrays the reference-CPU arm of bench.py consumes.
def _dev_bits(bits):
    import torch
    return torch.from_numpy(np.ascontiguousarray(bits).astype(np.int16)).view(torch.bfloat16).cuda()


@pytest.mark.parametrize("cfg", [(2048, 4096, 16384), (16384, 8192, 28672)],
                         ids=["config2", "config5"])
def test_mlp_block_full_size_on_reference_arm_inputs(cuda, cfg):
    import bench
    import polykernel_b200 as pk
    M, d, ffn = cfg
    host = bench.synthetic_host_weights(M, d, ffn, seed=0)
    y = pk.ops.mlp_block(*(_dev_bits(a) for a in host), eps=1e-6)
    rows = np.sort(np.random.default_rng(1).choice(M, 8, replace=False))
    x, gamma, w1, b1, w2, b2 = (O.from_bits(a) for a in host)
    ref = O.mlp_block(x[rows], gamma, w1, b1, w2, b2, eps=1e-6)
    print(cfg, check_chain(f32_from_t(y[rows]), ref))
    assert pk.device_error() == 0


def test_int8_mlp_full_size_on_seeded_inputs(cuda):
    import torch
    import bench
    import polykernel_b200 as pk
    M, d, ffn = 4096, 4096, 14336
    x, gamma, q1, s1, b1, q2, s2, b2 = bench.synthetic_host_int8(M, d, ffn, seed=0)
    dq = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    y = pk.ops.mlp_block_int8(_dev_bits(x), _dev_bits(gamma), dq(q1), dq(s1), _dev_bits(b1),
                              dq(q2), dq(s2), _dev_bits(b2), eps=1e-6)
    rows = np.sort(np.random.default_rng(2).choice(M, 8, replace=False))
    ref = O.mlp_block_int8(O.from_bits(x)[rows], O.from_bits(gamma), q1, s1, O.from_bits(b1),
                           q2, s2, O.from_bits(b2), eps=1e-6)
    print("config4", check_chain(f32_from_t(y[rows]), ref))


def test_attention_full_size_on_reference_arm_inputs(cuda):
    import torch
    import bench
    import polykernel_b200 as pk
    B, H, S, D, S_max = 4, 32, 2048, 128, 4096
    q, k, v = bench.synthetic_host_attention(B, H, S, D, seed=1)
    kc = torch.zeros(B, H, S_max, D, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    o = pk.ops.attention_prefill_kv_append(_dev_bits(q), _dev_bits(k), _dev_bits(v), kc, vc, 0,
                                           causal=True)
    assert np.array_equal(bits_from_t(kc[:, :, :S]), k) and np.array_equal(bits_from_t(vc[:, :, :S]), v)
    for (b, h) in ((0, 0), (0, 1), (3, 31)):        # (0,0), (0,1): heads the reference arm times
        qf, kf, vf = (O.from_bits(a[b:b + 1, h:h + 1]) for a in (q, k, v))
        ref = O.attention_prefill(qf, kf, vf, causal=True)
        ref64 = O.attention_prefill(qf, kf, vf, causal=True, acc=np.float64)
        print((b, h), check_attention(f32_from_t(o[b:b + 1, h:h + 1]), ref, s_kv=S, ref64_f32=ref64))
    assert pk.device_error() == 0
