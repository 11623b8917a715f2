"""Python host interface over the C ABI, mirroring the reference's operator set
(tests/golden/golden.py names; kernels/generated/*.cu launch_* semantics).

Every function takes bf16 CUDA tensors (contiguous, row-major), allocates the
output with torch, and launches on the current torch CUDA stream. Shapes are
validated here with the same meaning as the reference launchers; the C library
re-validates and returns cudaErrorInvalidValue for anything it cannot run.
"""
from __future__ import annotations

import math

import torch

from ._lib import check, lib

BF16 = torch.bfloat16


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


def _req(t, name, dtype=BF16, dims=None):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if dims is not None and t.dim() != dims:
        raise ValueError(f"{name} must have {dims} dims, got shape {tuple(t.shape)}")
    return t


def rmsnorm(x, weight=None, eps=1e-5):
    """golden.rmsnorm over the last axis (launch_rmsnorm, rmsnorm.cu:106)."""
    _req(x, "x")
    cols = x.shape[-1]
    if weight is not None:
        _req(weight, "weight")
        if weight.numel() != cols:
            raise ValueError("weight must have cols elements")
    y = torch.empty_like(x)
    check(lib().pkb200_rmsnorm(_ptr(x), _ptr(weight), _ptr(y), x.numel() // max(cols, 1), cols,
                               float(eps), _stream()), "rmsnorm")
    return y


def gelu(x):
    """golden.gelu (launch_gelu, gelu.cu:56)."""
    _req(x, "x")
    y = torch.empty_like(x)
    check(lib().pkb200_gelu(_ptr(x), _ptr(y), x.numel(), _stream()), "gelu")
    return y


def softmax(x):
    """golden.softmax over the last axis (launch_softmax, softmax.cu)."""
    _req(x, "x")
    cols = x.shape[-1] if x.dim() else 1
    rows = x.numel() // max(cols, 1)
    y = torch.empty_like(x)
    check(lib().pkb200_softmax(_ptr(x), _ptr(y), rows, cols, _stream()), "softmax")
    return y


def _mk(a, b):
    _req(a, "a")
    _req(b, "b", dims=2)
    K = a.shape[-1]
    if b.shape[0] != K:
        raise ValueError(f"inner dims differ: a {tuple(a.shape)} b {tuple(b.shape)}")
    M = a.numel() // max(K, 1) if K else a.numel()
    return M, b.shape[1], K


def matmul(a, b):
    """golden.matmul: [..., M, K] @ [K, N] (launch_matmul, matmul.cu:78)."""
    M, N, K = _mk(a, b)
    c = torch.empty(*a.shape[:-1], N, dtype=BF16, device=a.device)
    check(lib().pkb200_matmul(_ptr(a), _ptr(b), _ptr(c), M, N, K, _stream()), "matmul")
    return c


def matmul_f32out(a, b):
    """fp32 partial sums A @ B (the tensor-parallel rank's contribution)."""
    M, N, K = _mk(a, b)
    c = torch.empty(*a.shape[:-1], N, dtype=torch.float32, device=a.device)
    check(lib().pkb200_matmul_f32out(_ptr(a), _ptr(b), _ptr(c), M, N, K, _stream()),
          "matmul_f32out")
    return c


def fused_rmsnorm_matmul(x, w, weight=None, eps=1e-5):
    """golden.fused_rmsnorm_matmul (launch_fused_rmsnorm_matmul,
    fused_rmsnorm_matmul.cu:114; optional gamma as in golden.py:96-100)."""
    M, N, K = _mk(x, w)
    if weight is not None:
        _req(weight, "weight")
    c = torch.empty(*x.shape[:-1], N, dtype=BF16, device=x.device)
    check(lib().pkb200_fused_rmsnorm_matmul(_ptr(x), _ptr(w), _ptr(weight), _ptr(c), M, N, K,
                                            float(eps), _stream()), "fused_rmsnorm_matmul")
    return c


def fused_matmul_bias_gelu(x, w, b):
    """golden.fused_matmul_bias_gelu (fused_matmul_bias_gelu.cu:104)."""
    M, N, K = _mk(x, w)
    _req(b, "bias")
    if b.numel() != N:
        raise ValueError("bias must have N elements")
    c = torch.empty(*x.shape[:-1], N, dtype=BF16, device=x.device)
    check(lib().pkb200_fused_matmul_bias_gelu(_ptr(x), _ptr(w), _ptr(b), _ptr(c), M, N, K,
                                              _stream()), "fused_matmul_bias_gelu")
    return c


def matmul_bias_residual(a, w, b, resid):
    """add(bias(matmul(a, w), b), resid) with every op rounded (golden.py:48-60)."""
    M, N, K = _mk(a, w)
    _req(b, "bias")
    _req(resid, "resid")
    if resid.numel() != M * N or b.numel() != N:
        raise ValueError("bias/resid shape mismatch")
    c = torch.empty(*a.shape[:-1], N, dtype=BF16, device=a.device)
    check(lib().pkb200_matmul_bias_residual(_ptr(a), _ptr(w), _ptr(b), _ptr(resid), _ptr(c), M,
                                            N, K, _stream()), "matmul_bias_residual")
    return c


def bias_residual_f32(y32, b, resid, out=None):
    """bf16(bf16(bf16(y32) + b) + resid) for fp32 partial-sum totals."""
    _req(y32, "y32", dtype=torch.float32)
    _req(b, "bias")
    _req(resid, "resid")
    N = b.numel()
    M = y32.numel() // N
    if out is None:
        out = torch.empty(y32.shape, dtype=BF16, device=y32.device)
    else:
        _req(out, "out")
    check(lib().pkb200_bias_residual_f32(_ptr(y32), _ptr(b), _ptr(resid), _ptr(out), M, N,
                                         _stream()), "bias_residual_f32")
    return out


def matmul_int8(a, wq, scale):
    """quant_golden.matmul_int8 (launch_matmul_int8, matmul_int8.cu:97)."""
    _req(a, "a")
    _req(wq, "wq", dtype=torch.int8, dims=2)
    _req(scale, "scale", dtype=torch.float32)
    K = a.shape[-1]
    N = wq.shape[1]
    if wq.shape[0] != K or scale.numel() != N:
        raise ValueError("shape mismatch")
    M = a.numel() // max(K, 1)
    c = torch.empty(*a.shape[:-1], N, dtype=BF16, device=a.device)
    check(lib().pkb200_matmul_int8(_ptr(a), _ptr(wq), _ptr(scale), _ptr(c), M, N, K, _stream()),
          "matmul_int8")
    return c


FP8_FORMATS = {"e4m3": (0, torch.float8_e4m3fn), "e5m2": (1, torch.float8_e5m2)}


def _fp8_fmt(fmt):
    if fmt not in FP8_FORMATS:
        raise ValueError(f"unknown fp8 format {fmt!r} (expected 'e4m3' or 'e5m2')")
    return FP8_FORMATS[fmt]


def quantize_fp8(w, fmt="e4m3"):
    """bf16 -> fp8 weights (torch.float8_e4m3fn / float8_e5m2 tensor), rounded
    to nearest-even and saturating like the reference's CPU fp8_round
    (kernels/cpu/matmul_quant.cpp:130-150)."""
    code, dt = _fp8_fmt(fmt)
    _req(w, "w")
    out = torch.empty(w.shape, dtype=dt, device=w.device)
    check(lib().pkb200_quantize_fp8(_ptr(w), _ptr(out), w.numel(), code, _stream()),
          "quantize_fp8")
    return out


def dequantize_fp8(wf8):
    """fp8 weights -> bf16 (exact)."""
    fmt = {torch.float8_e4m3fn: "e4m3", torch.float8_e5m2: "e5m2"}.get(wf8.dtype)
    if fmt is None:
        raise TypeError(f"wf8: expected a float8_e4m3fn/float8_e5m2 tensor, got {wf8.dtype}")
    _req(wf8, "wf8", dtype=wf8.dtype)
    out = torch.empty(wf8.shape, dtype=BF16, device=wf8.device)
    check(lib().pkb200_dequantize_fp8(_ptr(wf8), _ptr(out), wf8.numel(), FP8_FORMATS[fmt][0],
                                      _stream()), "dequantize_fp8")
    return out


def matmul_fp8(a, wf8):
    """C = bf16(A @ fp8(W)) with the weights resident as fp8 [K, N]
    (quant_golden.matmul_fp8_sim semantics, quant_golden.py:116-125)."""
    fmt = {torch.float8_e4m3fn: "e4m3", torch.float8_e5m2: "e5m2"}.get(wf8.dtype)
    if fmt is None:
        raise TypeError(f"wf8: expected a float8_e4m3fn/float8_e5m2 tensor, got {wf8.dtype}")
    _req(a, "a")
    _req(wf8, "wf8", dtype=wf8.dtype, dims=2)
    K, N = wf8.shape
    if a.shape[-1] != K:
        raise ValueError("shape mismatch")
    M = a.numel() // max(K, 1)
    c = torch.empty(*a.shape[:-1], N, dtype=BF16, device=a.device)
    check(lib().pkb200_matmul_fp8(_ptr(a), _ptr(wf8), _ptr(c), M, N, K, FP8_FORMATS[fmt][0],
                                  _stream()), "matmul_fp8")
    return c


def matmul_fp8_sim(a, w, fmt="e4m3"):
    """The reference's simulated fp8 path (quant_golden.matmul_fp8_sim; the CPU
    `fp8sim` mode, matmul_quant.cpp:207-236): bf16 W rounded onto the fp8 grid,
    then matmul."""
    code, _ = _fp8_fmt(fmt)
    _req(a, "a")
    _req(w, "w", dims=2)
    K, N = w.shape
    if a.shape[-1] != K:
        raise ValueError("shape mismatch")
    M = a.numel() // max(K, 1)
    c = torch.empty(*a.shape[:-1], N, dtype=BF16, device=a.device)
    check(lib().pkb200_matmul_fp8_sim(_ptr(a), _ptr(w), _ptr(c), M, N, K, code, _stream()),
          "matmul_fp8_sim")
    return c


def mlp_workspace(M, d, ffn, device=None):
    n = int(lib().pkb200_mlp_block_workspace_size(M, d, ffn))
    return torch.empty(max(n, 1), dtype=torch.uint8, device=device or "cuda")


def mlp_block(x, gamma, w1, b1, w2, b2, eps=1e-6, workspace=None, out=None):
    """Y = X + (GELU(rmsnorm(X;gamma)@W1 + b1) @ W2 + b2), golden rounding."""
    _req(x, "x")
    d = x.shape[-1]
    M = x.numel() // d
    for t, n in ((gamma, "gamma"), (w1, "w1"), (b1, "b1"), (w2, "w2"), (b2, "b2")):
        _req(t, n)
    ffn = w1.shape[1]
    if w1.shape[0] != d or w2.shape != (ffn, d) or b1.numel() != ffn or b2.numel() != d:
        raise ValueError("mlp_block weight shapes do not match x")
    if workspace is None:
        workspace = mlp_workspace(M, d, ffn, x.device)
    y = torch.empty_like(x) if out is None else out
    check(lib().pkb200_mlp_block(_ptr(x), _ptr(gamma), _ptr(w1), _ptr(b1), _ptr(w2), _ptr(b2),
                                 _ptr(y), M, d, ffn, float(eps), _ptr(workspace),
                                 workspace.numel(), _stream()), "mlp_block")
    return y


def mlp_block_rmsnorm_next(x, gamma, w1, b1, w2, b2, gamma_next=None, eps=1e-6, eps_next=1e-6,
                           workspace=None):
    """(Y, Yn): Y = the MLP block (the residual stream), Yn = rmsnorm(Y;
    gamma_next) for the next layer (golden.fused_residual_rmsnorm,
    golden.py:108-112). GEMM2's epilogue emits the per-row partial sums of
    squares, so Yn costs one elementwise pass over Y."""
    _req(x, "x")
    d = x.shape[-1]
    M = x.numel() // d
    for t, n in ((gamma, "gamma"), (w1, "w1"), (b1, "b1"), (w2, "w2"), (b2, "b2")):
        _req(t, n)
    if gamma_next is not None:
        _req(gamma_next, "gamma_next")
        if gamma_next.numel() != d:
            raise ValueError("gamma_next must have d elements")
    ffn = w1.shape[1]
    if w1.shape[0] != d or w2.shape != (ffn, d) or b1.numel() != ffn or b2.numel() != d:
        raise ValueError("mlp_block weight shapes do not match x")
    nbytes = lib().pkb200_mlp_block_rmsnorm_next_workspace_size(M, d, ffn)
    if workspace is None or workspace.numel() < nbytes:
        workspace = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    y = torch.empty_like(x)
    yn = torch.empty_like(x)
    check(lib().pkb200_mlp_block_rmsnorm_next(
        _ptr(x), _ptr(gamma), _ptr(w1), _ptr(b1), _ptr(w2), _ptr(b2),
        _ptr(gamma_next) if gamma_next is not None else None, _ptr(y), _ptr(yn), M, d, ffn,
        float(eps), float(eps_next), _ptr(workspace), workspace.numel(), _stream()),
        "mlp_block_rmsnorm_next")
    return y, yn


def mlp_block_int8(x, gamma, w1q, s1, b1, w2q, s2, b2, eps=1e-6, workspace=None):
    """int8 weight-only MLP chain (quant_golden.matmul_int8 for both GEMMs)."""
    _req(x, "x")
    d = x.shape[-1]
    M = x.numel() // d
    ffn = w1q.shape[1]
    if workspace is None:
        workspace = mlp_workspace(M, d, ffn, x.device)
    y = torch.empty_like(x)
    check(lib().pkb200_mlp_block_int8(_ptr(x), _ptr(gamma), _ptr(w1q), _ptr(s1), _ptr(b1),
                                      _ptr(w2q), _ptr(s2), _ptr(b2), _ptr(y), M, d, ffn,
                                      float(eps), _ptr(workspace), workspace.numel(), _stream()),
          "mlp_block_int8")
    return y


def attention_prefill(q, k, v, causal=True, scale=None):
    """Prefill attention (launch_attention_prefill, attention_prefill.cu:169).
    q [B,H,S_q,D]; k, v [B,H,S_kv,D]."""
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _req(t, n, dims=4)
    B, H, Sq, D = q.shape
    Skv = k.shape[2]
    if k.shape != (B, H, Skv, D) or v.shape != k.shape:
        raise ValueError("q/k/v shape mismatch")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    o = torch.empty_like(q)
    check(lib().pkb200_attention_prefill(_ptr(q), _ptr(k), _ptr(v), _ptr(o), B, H, Sq, Skv, D,
                                         float(scale), int(bool(causal)), _stream()),
          "attention_prefill")
    return o


def kv_cache_update(cache, new):
    """Out-of-place concat along seq (launch_kv_cache_update, kv_cache_update.cu:67)."""
    _req(cache, "cache", dims=4)
    _req(new, "new", dims=4)
    B, H, Sc, D = cache.shape
    Sn = new.shape[2]
    if new.shape != (B, H, Sn, D):
        raise ValueError("cache/new shape mismatch")
    out = torch.empty(B, H, Sc + Sn, D, dtype=BF16, device=cache.device)
    check(lib().pkb200_kv_cache_update(_ptr(cache), _ptr(new), _ptr(out), B, H, Sc, Sn, D,
                                       _stream()), "kv_cache_update")
    return out


def attention_prefill_kv_append(q, k_new, v_new, k_cache, v_cache, s_cache, causal=True,
                                scale=None, out=None):
    """Append k_new/v_new into rows [s_cache, s_cache+S_q) of the preallocated
    caches (in place) and attend over the first s_cache+S_q rows
    (golden.fused_kv_append_attention)."""
    for t, n in ((q, "q"), (k_new, "k_new"), (v_new, "v_new"), (k_cache, "k_cache"),
                 (v_cache, "v_cache")):
        _req(t, n, dims=4)
    B, H, Sq, D = q.shape
    Smax = k_cache.shape[2]
    if k_new.shape != q.shape or v_new.shape != q.shape:
        raise ValueError("k_new/v_new must match q")
    if k_cache.shape != (B, H, Smax, D) or v_cache.shape != k_cache.shape:
        raise ValueError("cache shape mismatch")
    if s_cache < 0 or s_cache + Sq > Smax:
        raise ValueError("s_cache + S_q exceeds the cache")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    o = torch.empty_like(q) if out is None else out
    check(lib().pkb200_attention_prefill_kv_append(
        _ptr(q), _ptr(k_new), _ptr(v_new), _ptr(k_cache), _ptr(v_cache), _ptr(o), B, H, Sq,
        int(s_cache), Smax, D, float(scale), int(bool(causal)), _stream()),
        "attention_prefill_kv_append")
    return o


def fused_residual_rmsnorm(x, residual, weight=None, eps=1e-5, return_sum=False):
    """golden.fused_residual_rmsnorm: rmsnorm(bf16(x + residual)); optionally also
    the rounded sum (the new residual stream)."""
    _req(x, "x")
    _req(residual, "residual")
    if residual.shape != x.shape:
        raise ValueError("x and residual must have the same shape")
    if weight is not None:
        _req(weight, "weight")
    cols = x.shape[-1]
    out = torch.empty_like(x)
    ssum = torch.empty_like(x) if return_sum else None
    check(lib().pkb200_fused_residual_rmsnorm(_ptr(x), _ptr(residual), _ptr(weight), _ptr(out),
                                              _ptr(ssum), x.numel() // max(cols, 1), cols,
                                              float(eps), _stream()), "fused_residual_rmsnorm")
    return (out, ssum) if return_sum else out


def qkv_projection(x, w_qkv, num_heads):
    """golden.qkv_projection with Q, K, V returned in the attention layout
    [B, H, S, Dh] (x is [B, S, H*Dh])."""
    _req(x, "x", dims=3)
    _req(w_qkv, "w_qkv", dims=2)
    B, S, Dm = x.shape
    if w_qkv.shape != (Dm, 3 * Dm) or Dm % num_heads:
        raise ValueError("w_qkv must be [D, 3D] with D divisible by num_heads")
    Dh = Dm // num_heads
    q, k, v = (torch.empty(B, num_heads, S, Dh, dtype=BF16, device=x.device) for _ in range(3))
    check(lib().pkb200_qkv_projection(_ptr(x), _ptr(w_qkv), _ptr(q), _ptr(k), _ptr(v), B, S,
                                      num_heads, Dh, _stream()), "qkv_projection")
    return q, k, v
