"""Shared helpers for the tests: bf16-bit <-> torch conversion and gate checks."""
from __future__ import annotations

import numpy as np

from oracle import golden_np as O
from oracle import metrics as Mx


def t_from_bits(bits, device="cuda"):
    """uint16 bf16 bits (numpy) -> torch bf16 tensor on device."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(bits).astype(np.int16)).view(torch.bfloat16)
    return t.to(device)


def bits_from_t(t):
    import torch
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def f32_from_t(t):
    return O.from_bits(bits_from_t(t))


def check_gate(out_f32, ref_f32, rel_ceiling=Mx.MAX_REL_ERR_THRESHOLD, min_exact=0.90,
               quant=False):
    """The reference's kernel check (tests/kernels/test_cuda_run.py:262-288):
    cosine and PCC gates, a bit-exact fraction floor, and a max_rel_err ceiling."""
    m = Mx.report(out_f32, ref_f32)
    c_t = Mx.QUANT_COSINE_THRESHOLD if quant else Mx.COSINE_THRESHOLD
    assert m["cosine"] >= c_t, m
    assert m["pcc"] >= Mx.PCC_THRESHOLD, m
    assert m["bit_exact"] >= min_exact, m
    assert m["max_rel_err"] <= rel_ceiling, m
    return m
