"""CPU: the C-ABI library loads and exports every symbol include/pkb200.h declares
(no compute calls: this container has no GPU)."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "pkb200.h")


def _declared():
    txt = open(HEADER).read()
    c_names = sorted(set(re.findall(r"\b(pkb200_\w+|polykernel_\w+)\s*\(", txt)))
    cpp_names = sorted(set(re.findall(r"^void (launch_\w+)\(", txt, flags=re.M)))
    return c_names, cpp_names


def test_header_declares_reference_entry_points():
    c_names, cpp_names = _declared()
    for n in ("launch_matmul", "launch_fused_rmsnorm_matmul", "launch_fused_matmul_bias_gelu",
              "launch_rmsnorm", "launch_gelu", "launch_attention_prefill",
              "launch_kv_cache_update", "launch_matmul_int8"):
        assert n in cpp_names
    assert "pkb200_mlp_block" in c_names and "pkb200_attention_prefill_kv_append" in c_names


def test_library_loads_and_exports_all_symbols():
    from polykernel_b200 import _lib
    lib = _lib.lib()
    c_names, cpp_names = _declared()
    for n in c_names:
        assert hasattr(lib, n), n
    assert set(c_names) == set(_lib.SIGNATURES), "ctypes table out of sync with the header"
    syms = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                          text=True, check=True).stdout
    for n in cpp_names:
        # reference mangling: pk_bf16 == __nv_bfloat16 (cuda_run_main.cpp:59-71)
        assert re.search(rf"_Z\d+{n}PK13__nv_bfloat16", syms), n
    assert lib.pkb200_version().startswith(b"pkb200")


def test_reference_mangled_names_exact():
    from polykernel_b200 import _lib
    syms = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                          text=True, check=True).stdout
    # The names a binary built against the reference's declarations links to.
    for m in ("_Z13launch_matmulPK13__nv_bfloat16S1_PS_iiiPv",
              "_Z27launch_fused_rmsnorm_matmulPK13__nv_bfloat16S1_PS_iiifPv",
              "_Z29launch_fused_matmul_bias_geluPK13__nv_bfloat16S1_S1_PS_iiiPv",
              "_Z24launch_attention_prefillPK13__nv_bfloat16S1_S1_PS_iiiiifiPv",
              "_Z22launch_kv_cache_updatePK13__nv_bfloat16S1_PS_iiiiiPv",
              "_Z18launch_matmul_int8PK13__nv_bfloat16PKaPKfPS_iiiPv",
              "_Z14launch_rmsnormPK13__nv_bfloat16S1_PS_iifPv",
              "_Z11launch_geluPK13__nv_bfloat16PS_iPv"):
        assert m in syms, m
    # the additive entries, in the same style
    for m in ("_Z33launch_fused_rmsnorm_matmul_gammaPK13__nv_bfloat16S1_S1_PS_iiifPv",
              "_Z16launch_mlp_blockPK13__nv_bfloat16S1_S1_S1_S1_S1_PS_iiifPv",
              "_Z21launch_mlp_block_int8PK13__nv_bfloat16S1_PKaPKfS1_S3_S5_S1_PS_iiifPv",
              "_Z34launch_attention_prefill_kv_appendPK13__nv_bfloat16S1_S1_PS_S2_S2_iiiiiifiPv"):
        assert m in syms, m


def test_workspace_size_is_host_only():
    from polykernel_b200 import _lib
    lib = _lib.lib()
    assert lib.pkb200_mlp_block_workspace_size(0, 4096, 16384) == 0
    n = lib.pkb200_mlp_block_workspace_size(2048, 4096, 16384)
    assert n >= 2048 * 4096 * 2 + 2048 * 16384 * 2


def test_ops_reject_cpu_tensors():
    torch = pytest.importorskip("torch")
    from polykernel_b200 import ops
    x = torch.zeros(4, 8, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        ops.gelu(x)
    with pytest.raises(ValueError):
        ops.matmul(x, torch.zeros(8, 8, dtype=torch.bfloat16))


def test_empty_and_negative_sizes_without_a_device():
    """Empty inputs are no-ops and negative sizes are cudaErrorInvalidValue (1),
    decided before any device work, so this runs without a GPU (the reference's
    launchers likewise return before launching for empty shapes)."""
    import ctypes
    from polykernel_b200 import _lib
    L = _lib.lib()
    P = None
    eps = ctypes.c_float(1e-5)
    zero = [L.pkb200_matmul(P, P, P, 0, 8, 8, P),
            L.pkb200_matmul(P, P, P, 8, 0, 8, P),
            L.pkb200_fused_matmul_bias_gelu(P, P, P, P, 0, 8, 8, P),
            L.pkb200_fused_rmsnorm_matmul(P, P, P, P, 0, 8, 8, eps, P),
            L.pkb200_rmsnorm(P, P, P, 0, 8, eps, P),
            L.pkb200_gelu(P, P, 0, P),
            L.pkb200_softmax(P, P, 0, 8, P),
            L.pkb200_softmax(P, P, 4, 0, P),
            L.pkb200_attention_prefill(P, P, P, P, 1, 1, 0, 0, 64, ctypes.c_float(0.125), 1, P),
            L.pkb200_kv_cache_update(P, P, P, 1, 1, 0, 0, 64, P),
            L.pkb200_matmul_int8(P, P, P, P, 0, 8, 8, P),
            L.pkb200_mlp_block(P, P, P, P, P, P, P, 0, 8, 8, ctypes.c_float(1e-6), P, 0, P),
            L.pkb200_matmul_fp8_sim(P, P, P, 0, 8, 8, 0, P),
            L.pkb200_quantize_fp8(P, P, 0, 0, P),
            L.pkb200_dequantize_fp8(P, P, 0, 1, P)]
    assert zero == [0] * len(zero)
    negative = [L.pkb200_matmul(P, P, P, -1, 8, 8, P),
                L.pkb200_softmax(P, P, -1, 8, P),
                L.pkb200_rmsnorm(P, P, P, -1, 8, eps, P),
                L.pkb200_quantize_fp8(P, P, -4, 0, P),
                L.pkb200_matmul_fp8_sim(P, P, P, 0, 8, 8, 5, P),   # unknown fp8 format
                L.pkb200_quantize_fp8(P, P, 0, 7, P)]
    assert negative == [1] * len(negative)
