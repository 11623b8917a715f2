// simt_kernels.cuh - the memory-bound and general-shape kernels of the library:
// RMSNorm, GELU, the KV-cache copy/append, and the bounds-checked SIMT GEMM and
// attention used for shapes the TMA/tcgen05 paths cannot address (row strides
// that are not 16-byte multiples, head dims other than 64/128).
//
// All of them keep the reference's rounding contract (tests/golden/golden.py:1-18):
// fp32 compute, bf16 output of every op.
#pragma once

#include "gemm_tc.cuh"

namespace pkb200 {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Row softmax (golden.py:75-80; the reference's kernels/generated/softmax.cu):
// m = max(x), e = exp(x - m), y = bf16(e / sum(e)), all in fp32. One warp per
// row, three passes over the row (max, sum, normalise); the row stays in L1/L2
// between passes. Rows of -inf only produce NaN, as the golden does.
__global__ void softmax_rows_kernel(const __nv_bfloat16* __restrict__ x,
                                    __nv_bfloat16* __restrict__ out, long long rows, int cols) {
  const long long r = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  const __nv_bfloat16* xr = x + r * cols;
  __nv_bfloat16* yr = out + r * cols;
  float m = -INFINITY;
  for (int c = lane; c < cols; c += 32) m = fmaxf(m, __bfloat162float(xr[c]));
  m = warp_max(m);
  float sum = 0.f;
  for (int c = lane; c < cols; c += 32) sum += expf(__bfloat162float(xr[c]) - m);
  sum = warp_sum(sum);
  for (int c = lane; c < cols; c += 32)
    yr[c] = __float2bfloat16_rn(expf(__bfloat162float(xr[c]) - m) / sum);
}

// ------------------------------------------------------------------ RMSNorm --
// out[r, :] = bf16((x / sqrt(mean(x^2) + eps)) * w)   (golden.py:83-90,
// cpu_reference.cpp:16-44). One warp per row; the division is the correctly
// rounded fp32 divide the golden uses. `weight` may be null (no scale).
// When `rstd_out` is non-null the row's 1/rms is also stored (fp32).
__global__ void rmsnorm_rows_kernel(const __nv_bfloat16* __restrict__ x,
                                    const __nv_bfloat16* __restrict__ weight,
                                    __nv_bfloat16* __restrict__ out, long long rows, int cols,
                                    float eps) {
  const long long r = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  const __nv_bfloat16* xr = x + r * cols;
  __nv_bfloat16* yr = out + r * cols;
  const bool vec = (cols % 8) == 0 && (reinterpret_cast<uintptr_t>(x) % 16) == 0 &&
                   (reinterpret_cast<uintptr_t>(out) % 16) == 0 &&
                   (weight == nullptr || (reinterpret_cast<uintptr_t>(weight) % 16) == 0);
  float ss = 0.f;
  if (vec) {
    for (int c = lane * 8; c < cols; c += 256) {
      const uint4 u = *reinterpret_cast<const uint4*>(xr + c);
      const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(w4[j]);
        ss += f.x * f.x;
        ss += f.y * f.y;
      }
    }
  } else {
    for (int c = lane; c < cols; c += 32) {
      const float f = __bfloat162float(xr[c]);
      ss += f * f;
    }
  }
  ss = warp_sum(ss);
  const float rms = sqrtf(ss / static_cast<float>(cols) + eps);
  if (vec) {
    for (int c = lane * 8; c < cols; c += 256) {
      const uint4 u = *reinterpret_cast<const uint4*>(xr + c);
      const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
      uint32_t g4[4] = {0, 0, 0, 0};
      if (weight) {
        const uint4 g = *reinterpret_cast<const uint4*>(weight + c);
        g4[0] = g.x; g4[1] = g.y; g4[2] = g.z; g4[3] = g.w;
      }
      uint32_t o4[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(w4[j]);
        float a = __fdiv_rn(f.x, rms), b = __fdiv_rn(f.y, rms);
        if (weight) {
          const float2 g = unpack_bf16x2(g4[j]);
          a *= g.x;
          b *= g.y;
        }
        o4[j] = pack_bf16x2(a, b);
      }
      *reinterpret_cast<uint4*>(yr + c) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
    }
  } else {
    for (int c = lane; c < cols; c += 32) {
      float a = __fdiv_rn(__bfloat162float(xr[c]), rms);
      if (weight) a *= __bfloat162float(weight[c]);
      yr[c] = __float2bfloat16_rn(a);
    }
  }
}

// Same operation with the row held in registers: one 256-thread CTA per row,
// thread t owns 16-byte chunks t, t+256, ... (CH of them), so the row is read
// from HBM once (the warp-per-row kernel above reads it twice, and at 16 KB
// rows the second read misses L2). Requires cols % 8 == 0, cols <= 2048*CH and
// 16-byte aligned pointers.
template <int CH>
__global__ void __launch_bounds__(256) rmsnorm_rows_reg_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ weight,
    __nv_bfloat16* __restrict__ out, int cols, float eps) {
  __shared__ float red[8];
  const long long r = blockIdx.x;
  const int t = threadIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + r * cols);
  uint4* yr = reinterpret_cast<uint4*>(out + r * cols);
  const int nch = cols >> 3;
  uint4 v[CH];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const int c = t + 256 * j;
    v[j] = c < nch ? xr[c] : make_uint4(0u, 0u, 0u, 0u);
    const uint32_t w4[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = unpack_bf16x2(w4[q]);
      ss += f.x * f.x;
      ss += f.y * f.y;
    }
  }
  ss = warp_sum(ss);
  if ((t & 31) == 0) red[t >> 5] = ss;
  __syncthreads();
  if (t < 32) {
    float a = t < 8 ? red[t] : 0.f;
    a = warp_sum(a);
    if (t == 0) red[0] = a;
  }
  __syncthreads();
  const float rms = sqrtf(red[0] / static_cast<float>(cols) + eps);
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const int c = t + 256 * j;
    if (c >= nch) break;
    const uint32_t w4[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
    uint32_t g4[4] = {0, 0, 0, 0};
    if (weight) {
      const uint4 g = reinterpret_cast<const uint4*>(weight)[c];
      g4[0] = g.x; g4[1] = g.y; g4[2] = g.z; g4[3] = g.w;
    }
    uint32_t o4[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = unpack_bf16x2(w4[q]);
      float a = __fdiv_rn(f.x, rms), b = __fdiv_rn(f.y, rms);
      if (weight) {
        const float2 g = unpack_bf16x2(g4[q]);
        a *= g.x;
        b *= g.y;
      }
      o4[q] = pack_bf16x2(a, b);
    }
    yr[c] = make_uint4(o4[0], o4[1], o4[2], o4[3]);
  }
}

// Second half of the RMSNorm fused behind GEMM2 (kEpiBiasResidSS): the GEMM's
// epilogue left `parts` partial sums of squares per row in row_ss (stride
// ss_stride); out = bf16((y / sqrt(sum/cols + eps)) * w) with the partials
// summed in a fixed order (deterministic) and the golden's correctly rounded
// divide (golden.py:83-90). One 256-thread CTA per row, 16-byte vectors.
__global__ void __launch_bounds__(256) rmsnorm_apply_kernel(
    const __nv_bfloat16* __restrict__ y, const float* __restrict__ row_ss, int ss_stride,
    int parts, const __nv_bfloat16* __restrict__ weight, __nv_bfloat16* __restrict__ out,
    int cols, float eps) {
  __shared__ float rms_s;
  const long long r = blockIdx.x;
  if (threadIdx.x < 32) {
    float a = 0.f;
    for (int i = threadIdx.x; i < parts; i += 32) a += row_ss[r * ss_stride + i];
    a = warp_sum(a);
    if (threadIdx.x == 0) rms_s = sqrtf(a / static_cast<float>(cols) + eps);
  }
  __syncthreads();
  const float rms = rms_s;
  const uint4* yr = reinterpret_cast<const uint4*>(y + r * cols);
  uint4* orow = reinterpret_cast<uint4*>(out + r * cols);
  for (int c = threadIdx.x; c < (cols >> 3); c += 256) {
    const uint4 v = yr[c];
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
    uint32_t g4[4] = {0, 0, 0, 0};
    if (weight) {
      const uint4 g = reinterpret_cast<const uint4*>(weight)[c];
      g4[0] = g.x; g4[1] = g.y; g4[2] = g.z; g4[3] = g.w;
    }
    uint32_t o4[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = unpack_bf16x2(w4[q]);
      float a = __fdiv_rn(f.x, rms), b = __fdiv_rn(f.y, rms);
      if (weight) {
        const float2 g = unpack_bf16x2(g4[q]);
        a *= g.x;
        b *= g.y;
      }
      o4[q] = pack_bf16x2(a, b);
    }
    orow[c] = make_uint4(o4[0], o4[1], o4[2], o4[3]);
  }
}

// ------------------------------------------------- residual add + RMSNorm --
// t = bf16(x + resid) (golden.add), out = rmsnorm(t; weight, eps)
// (golden.fused_residual_rmsnorm, golden.py:108-112). `sum_out` (nullable)
// receives t, the new residual stream. One warp per row.
__global__ void residual_rmsnorm_rows_kernel(const __nv_bfloat16* __restrict__ x,
                                             const __nv_bfloat16* __restrict__ resid,
                                             const __nv_bfloat16* __restrict__ weight,
                                             __nv_bfloat16* __restrict__ out,
                                             __nv_bfloat16* __restrict__ sum_out, long long rows,
                                             int cols, float eps) {
  const long long r = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  const long long base = r * cols;
  float ss = 0.f;
  for (int c = lane; c < cols; c += 32) {
    const float t = bf16_round(__bfloat162float(x[base + c]) + __bfloat162float(resid[base + c]));
    ss += t * t;
    if (sum_out) sum_out[base + c] = __float2bfloat16_rn(t);
  }
  ss = warp_sum(ss);
  const float rms = sqrtf(ss / static_cast<float>(cols) + eps);
  for (int c = lane; c < cols; c += 32) {
    const float t = bf16_round(__bfloat162float(x[base + c]) + __bfloat162float(resid[base + c]));
    float a = __fdiv_rn(t, rms);
    if (weight) a *= __bfloat162float(weight[c]);
    out[base + c] = __float2bfloat16_rn(a);
  }
}

// --------------------------------------------------------------------- GELU --
// y = bf16(0.5 x (1 + erf(x/sqrt 2)))  (golden.py:63-66, gelu.cu:35-49).
__global__ void gelu_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y,
                            long long n) {
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride)
    y[i] = __float2bfloat16_rn(gelu_erf(__bfloat162float(x[i])));
}

// ------------------------------------------------------------- KV-cache copy --
// Row copy used for the KV-cache update. Copies `rows` rows of `D` bf16 from
// src (row stride src_ld rows grouped per bh) into dst. 16-byte vectors when
// the row byte length allows it.
//   dst[bh, dst_off + s, :] = src[bh, s, :]   for s < rows_per_bh
__global__ void kv_rows_copy_kernel(const __nv_bfloat16* __restrict__ src,
                                    __nv_bfloat16* __restrict__ dst, int BH, int rows_per_bh,
                                    int src_rows_total, int dst_rows_total, int dst_off, int D) {
  const long long total_vec_per_bh = static_cast<long long>(rows_per_bh) * D;
  const bool vec = (D % 8) == 0;
  const long long units = vec ? total_vec_per_bh / 8 : total_vec_per_bh;
  const long long total = units * BH;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += stride) {
    const long long bh = i / units;
    const long long e = (i - bh * units) * (vec ? 8 : 1);  // element offset within bh block
    const long long s = e / D;
    const long long d = e - s * D;
    const __nv_bfloat16* sp = src + (bh * src_rows_total + s) * D + d;
    __nv_bfloat16* dp = dst + (bh * dst_rows_total + dst_off + s) * D + d;
    if (vec)
      *reinterpret_cast<uint4*>(dp) = *reinterpret_cast<const uint4*>(sp);
    else
      *dp = *sp;
  }
}

// ------------------------------------------------------------- SIMT GEMM --
// General-shape fallback: 32x32 output tile per 256-thread block, 4 outputs per
// thread, K staged through shared memory in 32-wide slabs. fp32 accumulate and
// the same epilogue rounding as the tensor-core path.
template <int EPI>
__device__ __forceinline__ float epilogue1(float acc, const EpilogueArgs& ea, long long m, int n) {
  if constexpr (EPI == kEpiPlain) {
    return acc;
  } else if constexpr (EPI == kEpiBiasGelu) {
    return gelu_erf(bf16_round(bf16_round(acc) + __bfloat162float(ea.bias[n])));
  } else if constexpr (EPI == kEpiBiasResid || EPI == kEpiBiasResidSS) {
    return bf16_round(bf16_round(acc) + __bfloat162float(ea.bias[n])) +
           __bfloat162float(ea.resid[m * ea.ld_resid + n]);
  } else if constexpr (EPI == kEpiColScale) {
    return acc * ea.col_scale[n];
  } else if constexpr (EPI == kEpiScaleBiasGelu) {
    return gelu_erf(bf16_round(bf16_round(acc * ea.col_scale[n]) + __bfloat162float(ea.bias[n])));
  } else if constexpr (EPI == kEpiScaleBiasResid) {
    return bf16_round(bf16_round(acc * ea.col_scale[n]) + __bfloat162float(ea.bias[n])) +
           __bfloat162float(ea.resid[m * ea.ld_resid + n]);
  } else {
    return acc;
  }
}

template <int EPI, typename TB>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const __nv_bfloat16* __restrict__ A,
                                                        const TB* __restrict__ B, void* C,
                                                        long long ldc, int M, int N, int K,
                                                        EpilogueArgs ea) {
  __shared__ float As[32][33];
  __shared__ float Bs[32][33];
  const int tx = threadIdx.x & 31;   // column within tile
  const int ty = threadIdx.x >> 5;   // 0..7, rows ty, ty+8, ty+16, ty+24
  const long long m0 = static_cast<long long>(blockIdx.y) * 32;
  const int n0 = blockIdx.x * 32;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int k0 = 0; k0 < K; k0 += 32) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = ty + 8 * i;
      const long long gm = m0 + r;
      const int gk = k0 + tx;
      As[r][tx] = (gm < M && gk < K) ? __bfloat162float(A[gm * K + gk]) : 0.f;
      const int bk = k0 + r;
      const int bn = n0 + tx;
      float bv = 0.f;
      if (bk < K && bn < N) {
        if constexpr (sizeof(TB) == 1)
          bv = static_cast<float>(B[static_cast<long long>(bk) * N + bn]);
        else
          bv = __bfloat162float(B[static_cast<long long>(bk) * N + bn]);
      }
      Bs[r][tx] = bv;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < 32; ++kk) {
      const float b = Bs[kk][tx];
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] += As[ty + 8 * i][kk] * b;
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const long long m = m0 + ty + 8 * i;
    const int n = n0 + tx;
    if (m < M && n < N) {
      if constexpr (EPI == kEpiF32)
        static_cast<float*>(C)[m * ldc + n] = acc[i];
      else
        static_cast<__nv_bfloat16*>(C)[m * ldc + n] =
            __float2bfloat16_rn(epilogue1<EPI>(acc[i], ea, m, n));
    }
  }
}

// -------------------------------------------------------- SIMT attention --
// General-shape causal attention (any D <= 256): one warp per query row, keys
// in chunks of 32 (one per lane), online softmax in fp32, each lane owning
// D/32 output columns. Semantics of attention_prefill.cu:84-155 and
// golden.py:139-172: scores = q.k * scale, row i may see keys j <= S_kv - S_q + i
// when causal, softmax in fp32, O rounded to bf16 once.
//
// Keys/values come from up to two sources so the same kernel serves both the
// plain prefill (one source of S_kv rows) and the KV-append prefill (cache
// prefix of S_cache rows, then the new rows):
//   key position p <  n_a : K_a[bh, p, :]      (row stride per bh: lda_rows)
//   key position p >= n_a : K_b[bh, p - n_a, :] (row stride per bh: ldb_rows)
struct KvSources {
  const __nv_bfloat16* Ka;
  const __nv_bfloat16* Va;
  int n_a;
  int lda_rows;
  const __nv_bfloat16* Kb;
  const __nv_bfloat16* Vb;
  int n_b;
  int ldb_rows;
};

// One query row of exact prefill attention, computed by one warp: fp32 scores,
// online softmax with expf, fp32 P.V, one bf16 rounding of O (the golden's
// arithmetic, golden.py:139-172; attention_prefill.cu:84-155). Used by the
// general-shape kernel below and by the tensor-core kernel for the rows of a
// CTA whose V tiles fall outside what its fp16 P.V can carry exactly.
__device__ __forceinline__ void attention_row_exact(const __nv_bfloat16* __restrict__ Q,
                                                    __nv_bfloat16* __restrict__ O,
                                                    const KvSources& kv, int S_q, int D,
                                                    float scale, int causal, int bh, int i,
                                                    int lane) {
  const int S_kv = kv.n_a + kv.n_b;
  const int limit = causal ? (S_kv - S_q + i) : (S_kv - 1);
  const __nv_bfloat16* q = Q + (static_cast<long long>(bh) * S_q + i) * D;
  constexpr int MAXC = 8;  // D <= 256
  float o[MAXC];
#pragma unroll
  for (int c = 0; c < MAXC; ++c) o[c] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;
  const int kend = min(S_kv - 1, limit);
  for (int j0 = 0; j0 <= kend; j0 += 32) {
    const int j = j0 + lane;
    float s = -INFINITY;
    if (j <= kend) {
      const __nv_bfloat16* krow =
          (j < kv.n_a) ? kv.Ka + (static_cast<long long>(bh) * kv.lda_rows + j) * D
                       : kv.Kb + (static_cast<long long>(bh) * kv.ldb_rows + (j - kv.n_a)) * D;
      float dot = 0.f;
      for (int d = 0; d < D; ++d) dot += __bfloat162float(q[d]) * __bfloat162float(krow[d]);
      s = dot * scale;
    }
    const float cmax = warp_max(s);
    const float m_new = fmaxf(m_run, cmax);
    const float alpha = (m_run == -INFINITY) ? 0.f : expf(m_run - m_new);
    const float p = (j <= kend) ? expf(s - m_new) : 0.f;
    l_run = l_run * alpha + warp_sum(p);
#pragma unroll
    for (int c = 0; c < MAXC; ++c) o[c] *= alpha;
    const int nk = min(32, kend - j0 + 1);
    for (int t = 0; t < nk; ++t) {
      const float pt = __shfl_sync(0xffffffffu, p, t);
      const int jt = j0 + t;
      const __nv_bfloat16* vrow =
          (jt < kv.n_a) ? kv.Va + (static_cast<long long>(bh) * kv.lda_rows + jt) * D
                        : kv.Vb + (static_cast<long long>(bh) * kv.ldb_rows + (jt - kv.n_a)) * D;
#pragma unroll
      for (int c = 0; c < MAXC; ++c) {
        const int d = lane + 32 * c;
        if (d < D) o[c] += pt * __bfloat162float(vrow[d]);
      }
    }
    m_run = m_new;
  }
  __nv_bfloat16* orow = O + (static_cast<long long>(bh) * S_q + i) * D;
  const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll
  for (int c = 0; c < MAXC; ++c) {
    const int d = lane + 32 * c;
    if (d < D) orow[d] = __float2bfloat16_rn(l_run > 0.f ? o[c] * inv : 0.f);
  }
}

__global__ void attention_simt_kernel(const __nv_bfloat16* __restrict__ Q,
                                      __nv_bfloat16* __restrict__ O, KvSources kv, int S_q, int D,
                                      float scale, int causal) {
  const int warps = blockDim.x >> 5;
  const int i = blockIdx.x * warps + (threadIdx.x >> 5);
  if (i >= S_q) return;
  attention_row_exact(Q, O, kv, S_q, D, scale, causal, blockIdx.y, i, threadIdx.x & 31);
}

}  // namespace pkb200
