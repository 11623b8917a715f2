// fp8.cuh - fp8 (e4m3fn / e5m2) weight storage for the weight-only GEMM.
//
// The reference only simulates fp8 weights (tests/golden/quant_golden.py:
// 107-125 rounds bf16 weights onto the fp8 grid with ml_dtypes; its CPU twin
// is kernels/cpu/matmul_quant.cpp:130-160) and has no kernel. Here the weights
// live in HBM as one byte per element and are expanded to bf16 for the
// tcgen05 bf16 GEMM. The expansion is exact (every e4m3/e5m2 value is a bf16
// value: 3/2 mantissa bits against 7, exponents inside bf16's range), so the
// GEMM's result is the golden's C = bf16(fp32(bf16(A)) @ fp8(W)). A real
// kind::f8f6f4 MMA would need A in fp8 as well, which the golden does not do.
//
// Rounding (encode) follows the reference CPU fp8_round: NaN stays NaN (code
// 0x7F|sign), +-inf stays inf for e5m2 and saturates to +-max-finite for
// e4m3, finite magnitudes above max-finite saturate, the rest round to
// nearest-even at their own exponent with a fixed smallest ulp below the
// normal range. ml_dtypes (the golden's cast) agrees on every value up to
// max-finite and differs only above it (it gives NaN/inf where the CPU code
// saturates).
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

namespace pkb200 {

enum Fp8Format : int { kFp8E4M3 = 0, kFp8E5M2 = 1 };

template <int FMT>
struct Fp8Traits;
template <>
struct Fp8Traits<kFp8E4M3> {
  static constexpr int kMbits = 3, kBias = 7;
  static constexpr bool kHasInf = false;
  static constexpr float kMax = 448.0f;
};
template <>
struct Fp8Traits<kFp8E5M2> {
  static constexpr int kMbits = 2, kBias = 15;
  static constexpr bool kHasInf = true;
  static constexpr float kMax = 57344.0f;
};

// 2^k for |k| well inside the normal float range (exact).
__device__ __forceinline__ float fp8_pow2(int k) { return __int_as_float((127 + k) << 23); }

// float (a bf16 value here) -> fp8 code.
//
// With e = max(floor(log2 |x|), emin) and q = rint(|x| * 2^(mbits - e)), the
// code is ((e + bias - 1) << mbits) + q: for a normal value q is in
// [2^mbits, 2^(mbits+1)] and this is ((e + bias) << mbits) + (q - 2^mbits),
// q = 2^(mbits+1) carrying into the next exponent; below the normal range
// e = emin = 1 - bias and the code is the subnormal mantissa q itself.
template <int FMT>
__device__ __forceinline__ uint32_t fp8_encode(float x) {
  using T = Fp8Traits<FMT>;
  const uint32_t u = __float_as_uint(x);
  const uint32_t sign = (u >> 24) & 0x80u;
  const uint32_t abs_bits = u & 0x7FFFFFFFu;
  if (abs_bits > 0x7F800000u) return 0x7Fu | sign;  // NaN
  if (abs_bits == 0x7F800000u && T::kHasInf) return sign | (0x1Fu << 2);  // e5m2 inf
  const float mag = fminf(__uint_as_float(abs_bits), T::kMax);  // saturate (inf too)
  constexpr int emin = 1 - T::kBias;
  int e = static_cast<int>((__float_as_uint(mag) >> 23) & 0xFF) - 127;
  if (e < emin) e = emin;
  const uint32_t q = static_cast<uint32_t>(rintf(mag * fp8_pow2(T::kMbits - e)));
  if (q == 0) return sign;
  return sign | ((static_cast<uint32_t>(e + T::kBias - 1) << T::kMbits) + q);
}

// fp8 code -> bf16 bits (exact).
template <int FMT>
__device__ __forceinline__ uint32_t fp8_decode_bf16_bits(uint32_t c) {
  using T = Fp8Traits<FMT>;
  constexpr uint32_t mmask = (1u << T::kMbits) - 1;
  constexpr uint32_t efmax = 0x7Fu >> T::kMbits;
  const uint32_t s = (c & 0x80u) << 8;
  const uint32_t ef = (c & 0x7Fu) >> T::kMbits;
  const uint32_t m = c & mmask;
  if (ef == efmax) {
    if (T::kHasInf) return s | (m == 0 ? 0x7F80u : 0x7FC0u);
    if (m == mmask) return s | 0x7FC0u;  // e4m3fn's only NaN
  }
  if (ef == 0) {
    if (m == 0) return s;
    const float v = static_cast<float>(m) * fp8_pow2(1 - T::kBias - T::kMbits);
    return s | (__float_as_uint(v) >> 16);  // exact: v has at most 3 significant bits
  }
  return s | ((ef - T::kBias + 127) << 7) | (m << (7 - T::kMbits));
}

__device__ __forceinline__ float bf16_bits_to_float(uint32_t h) { return __uint_as_float(h << 16); }

// bf16 [n] -> fp8 codes [n]. 8 elements per thread step (16-byte loads, 8-byte
// stores) when `vec` (both pointers 16-byte aligned), else one element per step.
template <int FMT>
__global__ void bf16_to_fp8_kernel(const __nv_bfloat16* __restrict__ w, uint8_t* __restrict__ out,
                                   long long n, bool vec) {
  if (!vec) {
    const uint16_t* wb = reinterpret_cast<const uint16_t*>(w);
    for (long long k = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
         k += static_cast<long long>(gridDim.x) * blockDim.x)
      out[k] = static_cast<uint8_t>(fp8_encode<FMT>(bf16_bits_to_float(wb[k])));
    return;
  }
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x * 8;
  long long i = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  const uint16_t* wb = reinterpret_cast<const uint16_t*>(w);
  for (; i + 8 <= n; i += stride) {
    const uint4 v = __ldcs(reinterpret_cast<const uint4*>(wb + i));
    const uint32_t in[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[2] = {0, 0};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t h = (in[j >> 1] >> ((j & 1) * 16)) & 0xFFFFu;
      o[j >> 2] |= fp8_encode<FMT>(bf16_bits_to_float(h)) << ((j & 3) * 8);
    }
    *reinterpret_cast<uint2*>(out + i) = make_uint2(o[0], o[1]);
  }
  for (; i < n; ++i) out[i] = static_cast<uint8_t>(fp8_encode<FMT>(bf16_bits_to_float(wb[i])));
}

// fp8 codes [n] -> bf16 [n].
template <int FMT>
__global__ void fp8_to_bf16_kernel(const uint8_t* __restrict__ q, __nv_bfloat16* __restrict__ out,
                                   long long n, bool vec) {
  if (!vec) {
    uint16_t* ob = reinterpret_cast<uint16_t*>(out);
    for (long long k = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
         k += static_cast<long long>(gridDim.x) * blockDim.x)
      ob[k] = static_cast<uint16_t>(fp8_decode_bf16_bits<FMT>(q[k]));
    return;
  }
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x * 8;
  long long i = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  uint16_t* ob = reinterpret_cast<uint16_t*>(out);
  for (; i + 8 <= n; i += stride) {
    const uint2 v = __ldcs(reinterpret_cast<const uint2*>(q + i));
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t word = j < 2 ? v.x : v.y;
      const int sh = (j & 1) * 16;
      o[j] = fp8_decode_bf16_bits<FMT>((word >> sh) & 0xFFu) |
             (fp8_decode_bf16_bits<FMT>((word >> (sh + 8)) & 0xFFu) << 16);
    }
    *reinterpret_cast<uint4*>(ob + i) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  for (; i < n; ++i) ob[i] = static_cast<uint16_t>(fp8_decode_bf16_bits<FMT>(q[i]));
}

// bf16 [n] -> bf16 [n] rounded onto the fp8 grid (the simulated-weight path,
// encode then decode in one pass).
template <int FMT>
__global__ void bf16_round_fp8_grid_kernel(const __nv_bfloat16* __restrict__ w,
                                           __nv_bfloat16* __restrict__ out, long long n,
                                           bool vec) {
  if (!vec) {
    const uint16_t* wb = reinterpret_cast<const uint16_t*>(w);
    uint16_t* ob = reinterpret_cast<uint16_t*>(out);
    for (long long k = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
         k += static_cast<long long>(gridDim.x) * blockDim.x)
      ob[k] = static_cast<uint16_t>(
          fp8_decode_bf16_bits<FMT>(fp8_encode<FMT>(bf16_bits_to_float(wb[k]))));
    return;
  }
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x * 8;
  long long i = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  const uint16_t* wb = reinterpret_cast<const uint16_t*>(w);
  uint16_t* ob = reinterpret_cast<uint16_t*>(out);
  for (; i + 8 <= n; i += stride) {
    const uint4 v = __ldcs(reinterpret_cast<const uint4*>(wb + i));
    const uint32_t in[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t lo = fp8_encode<FMT>(bf16_bits_to_float(in[j] & 0xFFFFu));
      const uint32_t hi = fp8_encode<FMT>(bf16_bits_to_float(in[j] >> 16));
      o[j] = fp8_decode_bf16_bits<FMT>(lo) | (fp8_decode_bf16_bits<FMT>(hi) << 16);
    }
    *reinterpret_cast<uint4*>(ob + i) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  for (; i < n; ++i)
    ob[i] = static_cast<uint16_t>(fp8_decode_bf16_bits<FMT>(fp8_encode<FMT>(bf16_bits_to_float(wb[i]))));
}

}  // namespace pkb200
