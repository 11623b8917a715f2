"""Small single-kernel cases for profiling (ncu): `python -m polykernel_b200.profile_cases <case>`.

attn     attention_prefill, BASELINE config 3 (B=4, H=32, S=2048, D=128, causal)
gemm1c5  fused_matmul_bias_gelu at config-5 GEMM1 shape with M=4096 (d=8192, ffn=28672)
gemm     plain matmul 2048 x 4096 x 16384 (config-2 GEMM1 shape)
Each runs its kernel twice (profile the second launch with `-s 1 -c 1`).
"""
import sys

import torch

import polykernel_b200 as pk


def main(which):
    dev = "cuda"
    if which == "attn":
        q = torch.randn(4, 32, 2048, 128, device=dev).bfloat16()
        k, v = torch.randn_like(q), torch.randn_like(q)
        for _ in range(2):
            pk.ops.attention_prefill(q, k, v, True)
    elif which == "gemm1c5":
        a = torch.randn(4096, 8192, device=dev).bfloat16()
        b = (torch.randn(8192, 28672, device=dev) / 90).bfloat16()
        bias = (0.02 * torch.randn(28672, device=dev)).bfloat16()
        for _ in range(2):
            pk.ops.fused_matmul_bias_gelu(a, b, bias)
    elif which == "gemm":
        a = torch.randn(2048, 4096, device=dev).bfloat16()
        b = (torch.randn(4096, 16384, device=dev) / 64).bfloat16()
        for _ in range(2):
            pk.ops.matmul(a, b)
    else:
        raise SystemExit(f"unknown case {which!r}")
    torch.cuda.synchronize()
    assert pk.device_error() == 0
    print("ok", pk.path_counters())


if __name__ == "__main__":
    main(sys.argv[1])
