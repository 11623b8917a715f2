"""ctypes binding of libpkb200.so (the C ABI declared in include/pkb200.h).

The library is built in-tree (polykernel_b200/_lib/libpkb200.so, see
polykernel_b200/build.py). There is no fallback: if the shared library is
missing or does not load, every op raises.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_float, c_int, c_longlong, c_size_t, c_void_p

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libpkb200.so")

# (name, restype, argtypes) for every symbol in include/pkb200.h's C section.
_P = c_void_p
SIGNATURES = {
    "pkb200_version": (ctypes.c_char_p, []),
    "pkb200_rmsnorm": (c_int, [_P, _P, _P, c_int, c_int, c_float, _P]),
    "pkb200_gelu": (c_int, [_P, _P, c_longlong, _P]),
    "pkb200_softmax": (c_int, [_P, _P, c_int, c_int, _P]),
    "pkb200_matmul": (c_int, [_P, _P, _P, c_int, c_int, c_int, _P]),
    "pkb200_matmul_f32out": (c_int, [_P, _P, _P, c_int, c_int, c_int, _P]),
    "pkb200_fused_rmsnorm_matmul": (c_int, [_P, _P, _P, _P, c_int, c_int, c_int, c_float, _P]),
    "pkb200_fused_rmsnorm_matmul_noalloc": (c_int, [_P, _P, _P, _P, c_int, c_int, c_int,
                                                    c_float, _P]),
    "pkb200_fused_matmul_bias_gelu": (c_int, [_P, _P, _P, _P, c_int, c_int, c_int, _P]),
    "pkb200_matmul_bias_residual": (c_int, [_P, _P, _P, _P, _P, c_int, c_int, c_int, _P]),
    "pkb200_matmul_peer_store_f32": (c_int, [_P, _P, _P, c_int, c_int, c_int, c_int, c_int, _P]),
    "pkb200_reduce_slots_bias_residual": (c_int, [_P, c_int, c_int, c_int, _P, _P, _P, _P]),
    "pkb200_bias_residual_f32": (c_int, [_P, _P, _P, _P, c_int, c_int, _P]),
    "pkb200_fused_residual_rmsnorm": (c_int, [_P, _P, _P, _P, _P, c_int, c_int, c_float, _P]),
    "pkb200_qkv_projection": (c_int, [_P, _P, _P, _P, _P, c_int, c_int, c_int, c_int, _P]),
    "pkb200_matmul_int8": (c_int, [_P, _P, _P, _P, c_int, c_int, c_int, _P]),
    "pkb200_set_gemm_schedule": (c_int, [c_int]),
    "pkb200_stream_wait_value32": (c_int, [_P, _P, ctypes.c_uint]),
    "pkb200_stream_write_value32": (c_int, [_P, _P, ctypes.c_uint]),
    "pkb200_ipc_alloc": (c_int, [c_size_t, _P, _P]),
    "pkb200_ipc_open": (c_int, [_P, _P]),
    "pkb200_ipc_close": (c_int, [_P]),
    "pkb200_free": (c_int, [_P]),
    "pkb200_copy_async": (c_int, [_P, _P, c_size_t, _P]),
    "pkb200_tp_ce_create": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, _P, _P, _P, _P, _P,
                                    _P]),
    "pkb200_tp_ce_destroy": (c_int, [_P]),
    "pkb200_tp_ce_mlp_step": (c_int, [_P, _P, _P, c_int, _P, _P, _P, ctypes.c_uint, _P]),
    "pkb200_tp_ce_mlp_block": (c_int, [_P, _P, _P, _P, _P, c_int, _P, _P, _P, _P, ctypes.c_uint,
                                       _P]),
    "pkb200_tp_ce_wait": (c_int, [_P, c_int]),
    "pkb200_tp_ce_joined_streams": (c_int, [_P, ctypes.POINTER(c_int)]),
    "pkb200_quantize_fp8": (c_int, [_P, _P, c_longlong, c_int, _P]),
    "pkb200_dequantize_fp8": (c_int, [_P, _P, c_longlong, c_int, _P]),
    "pkb200_matmul_fp8": (c_int, [_P, _P, _P, c_int, c_int, c_int, c_int, _P]),
    "pkb200_matmul_fp8_sim": (c_int, [_P, _P, _P, c_int, c_int, c_int, c_int, _P]),
    "pkb200_mlp_block_workspace_size": (c_size_t, [c_int, c_int, c_int]),
    "pkb200_mlp_block": (c_int, [_P, _P, _P, _P, _P, _P, _P, c_int, c_int, c_int, c_float,
                                 _P, c_size_t, _P]),
    "pkb200_mlp_block_int8": (c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _P, c_int, c_int, c_int,
                                      c_float, _P, c_size_t, _P]),
    "pkb200_attention_prefill": (c_int, [_P, _P, _P, _P, c_int, c_int, c_int, c_int, c_int,
                                         c_float, c_int, _P]),
    "pkb200_kv_cache_update": (c_int, [_P, _P, _P, c_int, c_int, c_int, c_int, c_int, _P]),
    "pkb200_attention_prefill_kv_append": (c_int, [_P, _P, _P, _P, _P, _P, c_int, c_int, c_int,
                                                   c_int, c_int, c_int, c_float, c_int, _P]),
    "pkb200_set_gemm_max_ctas": (c_int, [c_int]),
    "pkb200_device_arch": (c_int, [ctypes.c_char_p, c_size_t]),
    "pkb200_tuning_load": (c_int, [ctypes.c_char_p, ctypes.c_char_p, c_size_t]),
    "pkb200_tuning_clear": (c_int, []),
    "pkb200_gemm_select": (c_int, [ctypes.c_char_p, c_int, c_int, c_int, ctypes.POINTER(c_int)]),
    "pkb200_set_gemm_config": (c_int, [ctypes.POINTER(c_int)]),
    "pkb200_last_gemm_config": (c_int, [ctypes.POINTER(c_int)]),
    "pkb200_selftest_wait_timeout": (c_int, [c_longlong, ctypes.POINTER(c_int)]),
    "pkb200_engine_load_mlp": (c_int, [_P, _P, _P, _P, _P, c_int, c_int, c_float]),
    "polykernel_fused_mlp_block": (c_int, [_P, _P, c_int, c_int, c_int]),
    "pkb200_device_error": (c_int, [ctypes.POINTER(c_int)]),
    "pkb200_path_counters": (c_int, [ctypes.POINTER(c_longlong), c_int]),
    "pkb200_attention_exact_ctas": (c_int, [ctypes.POINTER(ctypes.c_ulonglong)]),
    "pkb200_mlp_block_rmsnorm_next_workspace_size": (c_size_t, [c_int, c_int, c_int]),
    "pkb200_mlp_block_rmsnorm_next": (c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _P, c_int, c_int,
                                              c_int, c_float, c_float, _P, c_size_t, _P]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Load (once) and return the library; raise if it is not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"pkb200: CUDA library not built ({LIB_PATH} missing); "
                "run `python -c 'import __graft_entry__ as g; g.build()'` or "
                "`make -C polykernel_b200/csrc`")
        h = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _lib = h
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        raise RuntimeError(f"pkb200: {what} failed with CUDA status {status}")


def path_counters() -> dict:
    buf = (c_longlong * 5)()
    n = lib().pkb200_path_counters(buf, 5)
    keys = ["gemm_tc", "gemm_simt", "attn_tc", "attn_simt", "other"]
    return {keys[i]: int(buf[i]) for i in range(n)}


def device_error() -> int:
    v = c_int(0)
    check(lib().pkb200_device_error(ctypes.byref(v)), "pkb200_device_error")
    return int(v.value)


def attention_exact_ctas() -> int:
    """CTAs of the tensor-core attention kernel that took the exact fp32 row
    path (V values outside the fp16 P.V pass's exact range), since load."""
    v = ctypes.c_ulonglong(0)
    check(lib().pkb200_attention_exact_ctas(ctypes.byref(v)), "pkb200_attention_exact_ctas")
    return int(v.value)
