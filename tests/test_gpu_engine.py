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
