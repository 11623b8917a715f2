"""GPU: the serving-engine entry point polykernel_fused_mlp_block (the ctypes
ABI the reference's Modal app binds, modal/app.py:206-215) over host fp32 rows."""
import ctypes

import numpy as np
import pytest

from oracle import golden_np as O
from tests.helpers import check_parity

pytestmark = pytest.mark.gpu


def test_engine_mlp_block_host_fp32(golden, cuda):
    from polykernel_b200._lib import lib
    L = lib()
    g = golden("mlp")
    f = {k: np.ascontiguousarray(g[f"mid_{k}"]) for k in ("x", "gamma", "w1", "b1", "w2", "b2")}
    M, d = f["x"].shape
    ffn = f["w1"].shape[1]
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    x32 = O.from_bits(f["x"]).astype(np.float32)      # bf16-exact fp32 input
    out = np.zeros_like(x32)
    assert L.polykernel_fused_mlp_block(P(x32), P(out), M, d, d) == 2   # no weights yet
    assert L.pkb200_engine_load_mlp(P(f["gamma"]), P(f["w1"]), P(f["b1"]), P(f["w2"]), P(f["b2"]),
                                    d, ffn, ctypes.c_float(1e-6)) == 0
    assert L.polykernel_fused_mlp_block(P(x32), P(out), M, d, d + 1) != 0  # N must equal d
    for _ in range(2):
        out[:] = 0
        assert L.polykernel_fused_mlp_block(P(x32), P(out), M, d, d) == 0
        check_parity(out, O.from_bits(g["mid_y"]), min_exact=0.98)


def test_host_streamed_matches_device_and_pipelines_across_calls():
    """HostStreamed (pinned host in/out, copies overlapped with compute) gives
    the device result bit for bit, with ragged chunks, and back-to-back calls
    without a sync in between do not race on the reused device buffers."""
    import torch

    import polykernel_b200 as pk
    from polykernel_b200.streaming import HostStreamed
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    g = torch.Generator(device="cuda").manual_seed(3)
    M, d, ffn = 1000, 256, 512
    gm = (1 + 0.1 * torch.randn(d, device="cuda", generator=g)).bfloat16()
    w1 = (torch.randn(d, ffn, device="cuda", generator=g) / 16).bfloat16()
    b1 = (0.02 * torch.randn(ffn, device="cuda", generator=g)).bfloat16()
    w2 = (torch.randn(ffn, d, device="cuda", generator=g) / 22).bfloat16()
    b2 = (0.02 * torch.randn(d, device="cuda", generator=g)).bfloat16()
    xs = [torch.randn(M, d, device="cuda", generator=g).bfloat16() for _ in range(3)]
    refs = [pk.ops.mlp_block(x, gm, w1, b1, w2, b2, 1e-6) for x in xs]
    fwd = lambda xx, out: pk.ops.mlp_block(xx, gm, w1, b1, w2, b2, 1e-6, out=out)  # noqa: E731
    st = HostStreamed(fwd, chunks=3)
    xh = [x.cpu().pin_memory() for x in xs]
    yh = [torch.empty(M, d, dtype=torch.bfloat16).pin_memory() for _ in xs]
    for a, b in zip(xh, yh):
        st(a, b, "cuda", sync=False)
    st.wait()
    torch.cuda.synchronize()
    for y, r in zip(yh, refs):
        assert torch.equal(y, r.cpu())


def test_additive_launch_entries_match_c_abi():
    """launch_mlp_block / launch_fused_rmsnorm_matmul_gamma /
    launch_attention_prefill_kv_append (reference-style C++ symbols, library
    workspace) give the same bits as the C ABI calls they wrap."""
    import torch

    import polykernel_b200 as pk
    from polykernel_b200._lib import lib
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    L = lib()
    P = ctypes.c_void_p
    g = torch.Generator(device="cuda").manual_seed(9)
    M, d, ffn = 256, 512, 1024
    X = torch.randn(M, d, device="cuda", generator=g).bfloat16()
    gm = (1 + 0.1 * torch.randn(d, device="cuda", generator=g)).bfloat16()
    w1 = (torch.randn(d, ffn, device="cuda", generator=g) / 22).bfloat16()
    b1 = (0.02 * torch.randn(ffn, device="cuda", generator=g)).bfloat16()
    w2 = (torch.randn(ffn, d, device="cuda", generator=g) / 32).bfloat16()
    b2 = (0.02 * torch.randn(d, device="cuda", generator=g)).bfloat16()
    s = torch.cuda.current_stream().cuda_stream
    y = torch.empty_like(X)
    fn = getattr(L, "_Z16launch_mlp_blockPK13__nv_bfloat16S1_S1_S1_S1_S1_PS_iiifPv")
    fn.restype = None
    fn(*[P(t.data_ptr()) for t in (X, gm, w1, b1, w2, b2, y)], M, d, ffn, ctypes.c_float(1e-6),
       P(s))
    assert torch.equal(y, pk.ops.mlp_block(X, gm, w1, b1, w2, b2, 1e-6))
    out = torch.empty(M, ffn, dtype=torch.bfloat16, device="cuda")
    fn = getattr(L, "_Z33launch_fused_rmsnorm_matmul_gammaPK13__nv_bfloat16S1_S1_PS_iiifPv")
    fn.restype = None
    fn(P(X.data_ptr()), P(w1.data_ptr()), P(gm.data_ptr()), P(out.data_ptr()), M, ffn, d,
       ctypes.c_float(1e-6), P(s))
    assert torch.equal(out, pk.ops.fused_rmsnorm_matmul(X, w1, gm, 1e-6))
    B, H, S, D, Smax = 1, 2, 160, 64, 256
    q, kn, vn = (torch.randn(B, H, S, D, device="cuda", generator=g).bfloat16() for _ in range(3))
    kc = torch.zeros(B, H, Smax, D, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    o = torch.empty_like(q)
    fn = getattr(L, "_Z34launch_attention_prefill_kv_appendPK13__nv_bfloat16S1_S1_PS_S2_S2_iiiiiifiPv")
    fn.restype = None
    fn(*[P(t.data_ptr()) for t in (q, kn, vn, kc, vc, o)], B, H, S, 0, Smax, D,
       ctypes.c_float(D ** -0.5), 1, P(s))
    kc2, vc2 = torch.zeros_like(kc), torch.zeros_like(vc)
    o2 = pk.ops.attention_prefill_kv_append(q, kn, vn, kc2, vc2, 0, True)
    assert torch.equal(o, o2) and torch.equal(kc, kc2) and torch.equal(vc, vc2)
    assert pk.device_error() == 0
