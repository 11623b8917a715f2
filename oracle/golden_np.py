"""NumPy restatement of the reference golden for the fused MLP and prefill
attention path (test infrastructure; see oracle/__init__.py).

Rounding contract (tests/golden/golden.py:1-18 of the reference): inputs are
bf16, every reduction accumulates in fp32, every op's output is rounded to bf16
(round-to-nearest-even), and comparisons upcast the final bf16 to fp32.

bf16 values are carried here as float32 arrays whose values are exactly
representable in bf16 (``bf16()`` rounds onto that grid). ``to_bits`` /
``from_bits`` convert to/from the raw uint16 encoding the C ABI uses.
"""
from __future__ import annotations

import math

import numpy as np

try:  # scipy's erf is double precision, like math.erf
    from scipy.special import erf as _erf64
except Exception:  # pragma: no cover - scipy is in the image, fall back to libm
    _erf64 = np.vectorize(math.erf, otypes=[np.float64])

F32 = np.float32


# ------------------------------------------------------------------ bf16 grid --
def to_bits(x) -> np.ndarray:
    """fp32 -> bf16 bits, round-to-nearest-even; NaN stays a quiet NaN.

    Same rounding as the reference's float_to_bf16 (kernels/cpu/cpu_reference.h:52-61)
    and ml_dtypes.bfloat16: add 0x7FFF plus the kept LSB, then truncate.
    """
    u = np.ascontiguousarray(np.asarray(x, dtype=F32)).view(np.uint32)
    nan = (u & 0x7F800000) == 0x7F800000
    nan &= (u & 0x007FFFFF) != 0
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    if nan.any():
        r = np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)
    return r


def from_bits(b) -> np.ndarray:
    """bf16 bits -> fp32 (exact)."""
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(F32)


def bf16(x) -> np.ndarray:
    """Round onto the bf16 grid, returned as float32 (golden.py:_bf)."""
    return from_bits(to_bits(x))


# ------------------------------------------------------------ primitive ops --
def add(a, b):
    """golden.add (golden.py:48-50)."""
    return bf16(bf16(a) + bf16(b))


def bias(x, b):
    """golden.bias (golden.py:53-55): per-column add."""
    return bf16(bf16(x) + bf16(b))


def matmul(a, b, acc=F32):
    """golden.matmul (golden.py:58-60): fp32 accumulate, bf16 out.

    ``acc=np.float64`` gives the fp64-accumulated variant used to separate
    reduction-order noise from real error.
    """
    return bf16(np.matmul(bf16(a).astype(acc), bf16(b).astype(acc)).astype(F32))


def gelu(x):
    """golden.gelu (golden.py:63-66): erf evaluated in double on the fp32
    product x*(1/sqrt2), rounded to fp32, then 0.5*x*(1+erf) in fp32."""
    xf = bf16(x)
    e = _erf64((xf * F32(1.0 / math.sqrt(2.0))).astype(np.float64)).astype(F32)
    return bf16((F32(0.5) * xf) * (F32(1.0) + e))


def softmax(x):
    """golden.softmax (golden.py:75-80): fp32 exp(x - max) / sum over the last axis."""
    xf = bf16(x)
    e = np.exp(xf - np.max(xf, axis=-1, keepdims=True))
    return bf16(e / np.sum(e, axis=-1, keepdims=True))


def rmsnorm(x, weight=None, eps=1e-5):
    """golden.rmsnorm (golden.py:83-90): x / sqrt(mean(x^2)+eps) [* w], fp32."""
    xf = bf16(x)
    rms = np.sqrt(np.mean(xf * xf, axis=-1, keepdims=True, dtype=F32) + F32(eps)).astype(F32)
    out = (xf / rms).astype(F32)
    if weight is not None:
        out = out * bf16(weight)
    return bf16(out)


# -------------------------------------------------------------- fused chains --
def fused_rmsnorm_matmul(x, w, weight=None, eps=1e-5, acc=F32):
    """golden.fused_rmsnorm_matmul (golden.py:96-100)."""
    return matmul(rmsnorm(x, weight, eps), w, acc)


def fused_matmul_bias_gelu(x, w, b, acc=F32):
    """golden.fused_matmul_bias_gelu (golden.py:103-105): bias BEFORE gelu."""
    return gelu(bias(matmul(x, w, acc), b))


def mlp_block(x, gamma, w1, b1, w2, b2, eps=1e-6, acc=F32):
    """The MLP fragment composed from golden primitives:
    add(bias(matmul(gelu(bias(matmul(rmsnorm(X,g,eps),W1),b1)),W2),b2), X)
    (golden.py:48-100; the reference composes the same chain inline in
    tests/e2e/conftest.py:104-107 and examples/mlp_block.mlir, without biases)."""
    h = fused_matmul_bias_gelu(rmsnorm(x, gamma, eps), w1, b1, acc)
    return add(bias(matmul(h, w2, acc), b2), x)


def matmul_int8(a, wq, scale, acc=F32):
    """quant_golden.matmul_int8 (quant_golden.py:91-101): C = bf16(A @ (wq*scale))."""
    wdeq = np.asarray(wq).astype(F32) * np.asarray(scale, dtype=F32)[None, :]
    return bf16(np.matmul(bf16(a).astype(acc), wdeq.astype(acc)).astype(F32))


def mlp_block_int8(x, gamma, w1q, s1, b1, w2q, s2, b2, eps=1e-6, acc=F32):
    """int8 weight-only MLP chain: each matmul is quant_golden.matmul_int8, the
    rest as mlp_block."""
    h = gelu(bias(matmul_int8(rmsnorm(x, gamma, eps), w1q, s1, acc), b1))
    return add(bias(matmul_int8(h, w2q, s2, acc), b2), x)


# ------------------------------------------------------- fp8 weight path --
# (e4m3fn: 3 mantissa bits, bias 7, max finite 448, no inf; e5m2: 2 mantissa
# bits, bias 15, max finite 57344, IEEE inf/NaN.)
FP8_FORMATS = {"e4m3": (3, 7, 448.0, False), "e5m2": (2, 15, 57344.0, True)}


def fp8_round(x, fmt):
    """Round onto the fp8 grid, returned as float32 (the reference's CPU
    fp8_round, kernels/cpu/matmul_quant.cpp:130-150): NaN stays NaN, +-inf
    saturates to +-max-finite for e4m3 and stays inf for e5m2, finite
    magnitudes above max-finite saturate, the rest round to nearest-even at
    the value's own exponent (fixed smallest ulp below the normal range), and
    a result rounded past max-finite is clamped. Signed zeros are kept."""
    with np.errstate(invalid="ignore"):
        return _fp8_round(np.asarray(x, dtype=F32), *FP8_FORMATS[fmt])


def _fp8_round(x, mbits, bias_, fmax, has_inf):
    mag = np.abs(x).astype(np.float64)
    finite = np.isfinite(mag)
    m = np.where(finite, np.minimum(mag, fmax), 0.0)
    emin = 1 - bias_
    _, e = np.frexp(np.where(m > 0, m, 1.0))
    ex = np.maximum(e - 1, emin)
    ulp = np.ldexp(1.0, ex - mbits)
    r = np.minimum(np.rint(m / ulp) * ulp, fmax)
    inf_val = np.inf if has_inf else fmax
    r = np.where(np.isinf(mag), inf_val, r)
    r = np.where(np.isnan(x), np.nan, np.copysign(r, x))
    return r.astype(F32)


def fp8_bits(x, fmt):
    """fp8 encoding (uint8) of values already on the fp8 grid (fp8_round's
    output): sign, biased exponent, mantissa; NaN -> 0x7F|sign."""
    mbits, bias_, _, _ = FP8_FORMATS[fmt]
    x = np.asarray(x, dtype=F32)
    sign = np.signbit(x).astype(np.uint8) << 7
    mag = np.abs(x).astype(np.float64)
    emin = 1 - bias_
    out = np.zeros(x.shape, np.uint8)
    sub = mag < 2.0 ** emin
    out = np.where(sub, np.rint(mag / 2.0 ** (emin - mbits)), out)
    _, e = np.frexp(np.where(mag > 0, mag, 1.0))
    ex = e - 1
    frac = np.rint((mag / np.ldexp(1.0, ex) - 1.0) * (1 << mbits))
    normal = ~sub & np.isfinite(mag)
    out = np.where(normal, ((ex + bias_) << mbits) + frac, out)
    out = np.where(np.isinf(mag), (0x1F << 2) if fmt == "e5m2" else 0x7E, out)
    out = np.where(np.isnan(x), 0x7F, out)
    return out.astype(np.uint8) | sign


def fp8_decode(bits, fmt):
    """fp8 bits -> float32 (exact; every fp8 value is a bf16 value)."""
    mbits, bias_, _, has_inf = FP8_FORMATS[fmt]
    b = np.asarray(bits, dtype=np.uint8).astype(np.int64)
    s = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> mbits) & ((1 << (7 - mbits)) - 1)
    m = b & ((1 << mbits) - 1)
    emax_field = (1 << (7 - mbits)) - 1
    v = np.where(e == 0, m * 2.0 ** (1 - bias_ - mbits),
                 (1.0 + m / (1 << mbits)) * np.ldexp(1.0, e - bias_))
    if has_inf:
        v = np.where(e == emax_field, np.where(m == 0, np.inf, np.nan), v)
    else:
        v = np.where((e == emax_field) & (m == (1 << mbits) - 1), np.nan, v)
    return (s * v).astype(F32)


def matmul_fp8_sim(a, w, fmt, acc=F32):
    """quant_golden.matmul_fp8_sim (quant_golden.py:116-125): weight-only fp8,
    C = bf16(fp32(bf16(A)) @ fp8(bf16(W)))."""
    w8 = fp8_round(bf16(w), fmt)
    return bf16(np.matmul(bf16(a).astype(acc), w8.astype(acc)).astype(F32))


# ----------------------------------------------------------------- attention --
def attention_prefill(q, k, v, causal=True, scale=None, acc=F32):
    """Prefill SDPA (kernels/cpu/attention.cpp:95-163; golden.py:139-172):
    scores = q.k * scale in fp32 (scale defaults to 1/sqrt(D)), query row i sees
    key j <= S_kv - S_q + i when causal, softmax in fp32, P.V in fp32, one bf16
    rounding. A row that sees no key yields 0. With acc=np.float64 every
    intermediate is fp64 (same single bf16 rounding of O): the fp64-accumulated
    reference that separates reduction-order noise from real error."""
    qf, kf, vf = bf16(q), bf16(k), bf16(v)
    D = qf.shape[-1]
    Sq, Skv = qf.shape[-2], kf.shape[-2]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    s = np.matmul(qf.astype(acc), np.swapaxes(kf, -1, -2).astype(acc)).astype(acc) * acc(scale)
    if causal:
        i = np.arange(Sq)[:, None]
        j = np.arange(Skv)[None, :]
        s = np.where(j <= (Skv - Sq + i), s, -np.inf).astype(acc)
    m = np.max(s, axis=-1, keepdims=True) if Skv else np.zeros(s.shape[:-1] + (1,), acc)
    m = np.where(np.isfinite(m), m, acc(0))
    e = np.exp(s - m).astype(acc)
    l = np.sum(e, axis=-1, keepdims=True, dtype=acc)
    o = np.matmul(e, vf.astype(acc)).astype(acc)
    o = np.where(l > 0, o / np.where(l > 0, l, acc(1)), acc(0))
    return bf16(o)


def kv_cache_update(cache, new):
    """kernels/generated/kv_cache_update.cu:34-58: concat along the seq axis."""
    return np.concatenate([bf16(cache), bf16(new)], axis=2)


def attention_prefill_kv_append(q, k_new, v_new, k_cache, v_cache, s_cache, causal=True,
                                scale=None):
    """Fused append + attention (golden.fused_kv_append_attention,
    golden.py:139-172) on a preallocated cache: rows [s_cache, s_cache+S_q) of
    the caches receive k_new / v_new, then q attends to the first s_cache+S_q
    rows. Returns (O, K_cache', V_cache') with untouched rows preserved."""
    Sq = q.shape[-2]
    kc = bf16(k_cache).copy()
    vc = bf16(v_cache).copy()
    kc[:, :, s_cache:s_cache + Sq] = bf16(k_new)
    vc[:, :, s_cache:s_cache + Sq] = bf16(v_new)
    o = attention_prefill(q, kc[:, :, :s_cache + Sq], vc[:, :, :s_cache + Sq], causal, scale)
    return o, kc, vc


# --------------------------------------------------- next-row fragments --
def fused_residual_rmsnorm(x, residual, weight=None, eps=1e-5):
    """golden.fused_residual_rmsnorm (golden.py:108-112): rmsnorm(add(x, residual))."""
    return rmsnorm(add(x, residual), weight, eps)


def qkv_projection(x, w_qkv, num_heads):
    """golden.qkv_projection (golden.py:120-136): x @ w_qkv (bf16), split the last
    axis into Q, K, V and reshape each to [..., num_heads, head_dim]."""
    proj = matmul(x, w_qkv)
    q, k, v = np.split(proj, 3, axis=-1)
    hd = q.shape[-1] // num_heads
    shp = q.shape[:-1] + (num_heads, hd)
    return q.reshape(shp), k.reshape(shp), v.reshape(shp)
