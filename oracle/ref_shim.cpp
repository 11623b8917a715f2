// ref_shim.cpp - extern "C" entry points over the reference's own CPU code
// (kernels/cpu/cpu_reference.cpp, compiled from the reference's sources by
// oracle/Makefile into oracle/_ref/liboracle_ref.so). TEST INFRASTRUCTURE:
// used by tests/ as a second oracle and by bench.py as the timed CPU baseline.
//
// ref_mlp_rows composes the MLP chain exactly as the reference's e2e harness
// does (tests/e2e/conftest.py:104-107): launch_rmsnorm_cpu (with gamma) ->
// launch_fused_matmul_bias_gelu_cpu -> launch_matmul_cpu, then bias and the
// residual add inline with golden.bias / golden.add rounding (golden.py:48-55).
#include <cstdint>
#include <vector>

#include "cpu_reference.h"

namespace cpu = polykernel::cpu;

extern "C" {

void ref_rmsnorm(const uint16_t* x, const uint16_t* w, uint16_t* y, int64_t rows, int64_t cols,
                 float eps) {
  cpu::launch_rmsnorm_cpu(x, w, y, rows, cols, eps);
}

void ref_gelu(const uint16_t* x, uint16_t* y, int64_t n) { cpu::launch_gelu_cpu(x, y, n); }

void ref_matmul(const uint16_t* a, const uint16_t* b, uint16_t* c, int64_t M, int64_t N,
                int64_t K) {
  cpu::launch_matmul_cpu(a, b, c, M, N, K);
}

void ref_fused_rmsnorm_matmul(const uint16_t* x, const uint16_t* w, uint16_t* y, int64_t M,
                              int64_t N, int64_t K, float eps) {
  cpu::launch_fused_rmsnorm_matmul_cpu(x, w, y, M, N, K, eps);
}

void ref_fused_matmul_bias_gelu(const uint16_t* a, const uint16_t* b, const uint16_t* bias,
                                uint16_t* y, int64_t M, int64_t N, int64_t K) {
  cpu::launch_fused_matmul_bias_gelu_cpu(a, b, bias, y, M, N, K);
}

void ref_mlp_rows(const uint16_t* x, const uint16_t* gamma, const uint16_t* w1,
                  const uint16_t* b1, const uint16_t* w2, const uint16_t* b2, uint16_t* y,
                  int64_t M, int64_t d, int64_t ffn, float eps) {
  std::vector<uint16_t> xn(static_cast<size_t>(M * d)), h(static_cast<size_t>(M * ffn)),
      t(static_cast<size_t>(M * d));
  cpu::launch_rmsnorm_cpu(x, gamma, xn.data(), M, d, eps);
  cpu::launch_fused_matmul_bias_gelu_cpu(xn.data(), w1, b1, h.data(), M, ffn, d);
  cpu::launch_matmul_cpu(h.data(), w2, t.data(), M, d, ffn);
  for (int64_t i = 0; i < M; ++i)
    for (int64_t j = 0; j < d; ++j) {
      const float u = cpu::bf16_to_float(cpu::float_to_bf16(
          cpu::bf16_to_float(t[i * d + j]) + cpu::bf16_to_float(b2[j])));
      y[i * d + j] = cpu::float_to_bf16(u + cpu::bf16_to_float(x[i * d + j]));
    }
}

}  // extern "C"
