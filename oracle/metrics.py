"""Correctness gate of the reference (tests/golden/metrics.py:20-77), restated.
Test infrastructure only (see oracle/__init__.py).

All metrics flatten and upcast to fp32. Thresholds: cosine >= 0.999,
max_rel_err <= 1e-2 (eps 1e-6), PCC >= 0.99 (metrics.py:20-23); the quantised
gate relaxes to cosine >= 0.99 / max_rel_err <= 5e-2 (quant_golden.py:46-48).
"""
from __future__ import annotations

import numpy as np

COSINE_THRESHOLD = 0.999
MAX_REL_ERR_THRESHOLD = 1e-2
PCC_THRESHOLD = 0.99
REL_ERR_EPS = 1e-6
QUANT_COSINE_THRESHOLD = 0.99
QUANT_MAX_REL_ERR_THRESHOLD = 5e-2


def _flat(x):
    return np.asarray(x, dtype=np.float64).reshape(-1)


def cosine(a, ref):
    x, y = _flat(a), _flat(ref)
    nx, ny = np.linalg.norm(x), np.linalg.norm(y)
    if nx * ny == 0.0:
        return 1.0 if (nx == 0.0 and ny == 0.0) else 0.0
    return float(np.dot(x, y) / (nx * ny))


def max_rel_err(a, ref, eps=REL_ERR_EPS):
    x, y = _flat(a), _flat(ref)
    if x.size == 0:
        return 0.0
    return float(np.max(np.abs(x - y) / (np.abs(y) + eps)))


def pcc(a, ref):
    x, y = _flat(a), _flat(ref)
    xc, yc = x - x.mean(), y - y.mean()
    d = float(np.sqrt(np.sum(xc * xc)) * np.sqrt(np.sum(yc * yc)))
    if d == 0.0:
        return 1.0 if np.array_equal(x, y) else 0.0
    return float(np.sum(xc * yc) / d)


def report(a, ref, ref64=None, small=1e-3):
    """The three gate metrics, plus (when an fp64-accumulated reference is
    given) max_rel_err against it, the count of near-zero reference elements
    that dominate max_rel_err, and the bit-exact fraction."""
    out = {"cosine": cosine(a, ref), "max_rel_err": max_rel_err(a, ref), "pcc": pcc(a, ref),
           "bit_exact": float(np.mean(_flat(a) == _flat(ref))) if np.size(ref) else 1.0,
           "near_zero": int(np.sum(np.abs(_flat(ref)) < small))}
    if ref64 is not None:
        out["max_rel_err_vs_fp64"] = max_rel_err(a, ref64)
    return out


def passes(m, quant=False):
    c_t = QUANT_COSINE_THRESHOLD if quant else COSINE_THRESHOLD
    r_t = QUANT_MAX_REL_ERR_THRESHOLD if quant else MAX_REL_ERR_THRESHOLD
    return m["cosine"] >= c_t and m["max_rel_err"] <= r_t and m["pcc"] >= PCC_THRESHOLD
