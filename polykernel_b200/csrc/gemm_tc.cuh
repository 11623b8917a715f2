// gemm_tc.cuh - persistent tcgen05 GEMM with fused epilogues (sm_100a).
//
//   C[M,N] = epilogue( A[M,K] @ B[K,N] )   A, B, C bf16 row-major, fp32 accumulate.
//
// This is the contraction behind every matmul-shaped entry point of the
// reference kernel library (kernels/generated/matmul.cu:78 launch_matmul,
// fused_matmul_bias_gelu.cu:104, fused_rmsnorm_matmul.cu:114,
// matmul_int8.cu:97) and of the MLP block composed in tests/e2e/conftest.py:104-107.
//
// Structure (one CTA per SM, persistent over output tiles):
//   warp 0   TMA producer: A tile 128x64 (K-major, 128B swizzle) and B tile
//            64x256 as four 64x64 N-major boxes, into a STAGES-deep ring.
//   warp 1   TMEM allocator + tcgen05.mma issuer (whole warp, one elected lane issues)
//            (M=128, N=256, K=16 per instruction, 4 per stage).
//   warps 2-9 epilogue (two per TMEM lane quarter, each owning half of the
//            columns): tcgen05.ld 32 columns at a time from the finished
//            accumulator, apply the fused epilogue with the reference's
//            rounding points, 16-byte vector stores.
//   The accumulator is double buffered in TMEM (2 x 256 fp32 columns), so the
//   epilogue of tile t overlaps the mainloop of tile t+1.
//
// Rounding contract (tests/golden/golden.py:1-18): every op rounds its output
// to bf16, so the epilogues round after the matmul, after each bias/residual
// add and after GELU, exactly where the golden composition does.
#pragma once

#include "sm100.cuh"

namespace pkb200 {

enum EpilogueKind : int {
  kEpiPlain = 0,      // C = bf16(acc)                                  (matmul.cu)
  kEpiBiasGelu = 1,   // C = bf16(gelu(bf16(bf16(acc) + bias)))         (fused_matmul_bias_gelu.cu)
  kEpiBiasResid = 2,  // C = bf16(bf16(bf16(acc) + bias) + resid)       (MLP GEMM2 + residual)
  kEpiColScale = 3,   // C = bf16(acc * scale[n])                       (matmul_int8.cu)
  kEpiF32 = 4,        // C(fp32) = acc   (tensor-parallel partial sums)
  kEpiPeerStoreF32 = 6,  // owner(m).slot[src_rank][m % rows_per_rank, n] = acc (plain stores;
                         // the owner sums the slots afterwards)
  kEpiQkvScatter = 7,    // bf16(acc) written to Q/K/V in [B, H, S, Dh] layout
  // int8 weight-only chain (quant_golden.matmul_int8, then the golden bias /
  // gelu / add, each rounded): the matmul's per-column scale, then as kinds 1/2
  kEpiScaleBiasGelu = 8,   // C = bf16(gelu(bf16(bf16(acc * s[n]) + bias)))
  kEpiScaleBiasResid = 9,  // C = bf16(bf16(bf16(acc * s[n]) + bias) + resid)
  // MLP GEMM2 feeding the next layer's RMSNorm (golden.fused_residual_rmsnorm,
  // golden.py:108-112): C as kEpiBiasResid, plus each (row, N tile, column
  // half)'s fp32 sum of squares of the rounded outputs into row_ss
  kEpiBiasResidSS = 10,
};

constexpr int kMaxPeers = 8;

// kEpiPeerStoreF32: one TMA map per owner rank over its [world*rows_per_rank, N]
// fp32 slot buffer (box 32 columns x 32 rows, 128-byte swizzle). Passed as a
// __grid_constant__ kernel parameter so the maps stay in parameter space.
struct PeerMaps {
  CUtensorMap m[kMaxPeers];
};

struct EpilogueArgs {
  const __nv_bfloat16* bias;   // [N] or null
  const __nv_bfloat16* resid;  // [M, ld_resid] or null
  const float* col_scale;      // [N] or null
  long long ld_resid;
  // kEpiPeerStoreF32: rows [r*rows_per_rank, (r+1)*rows_per_rank) of the
  // product go to peer[r] (an fp32 buffer, possibly on another GPU, reached
  // through NVLink peer mapping).
  float* peer[kMaxPeers];
  long long rows_per_rank;
  int src_rank;  // kEpiPeerStoreF32: this rank's slot index in every owner's buffer
  // kEpiQkvScatter: row m = b*seq + s, column n = which*heads*head_dim + h*head_dim + e
  __nv_bfloat16* qkv[3];
  int seq, heads, head_dim;
  // kEpiBiasResidSS: row_ss[m * ss_stride + 2 * n_tile + half]
  float* row_ss;
  int ss_stride;
};



// GELU as the golden evaluates it (tests/golden/golden.py:63-66):
//   z = fp32(x * (1/sqrt 2)); e = fp32(erf(z)) (erf in double, rounded once);
//   y = (0.5 * x) * (1 + e) in fp32.
// For z <= -0.5, e lies in (-1, -0.52] where fp32 spacing is 2^-24, so the
// golden's 1 + e equals erfc(-z) rounded to a multiple of 2^-24; computing it
// that way (erfcf is accurate relative to the small result) reproduces the
// golden's value instead of amplifying erff's absolute error by the
// cancellation in 1 + e. Elsewhere 1 + erff(z) has no cancellation.
__device__ __forceinline__ float gelu_erf(float x) {
  const float z = x * 0.70710678118654752440f;
  float one_plus_e;
  if (z <= -0.5f) {
    one_plus_e = rintf(erfcf(-z) * 16777216.0f) * (1.0f / 16777216.0f);
  } else {
    one_plus_e = 1.0f + erff(z);
  }
  return (0.5f * x) * one_plus_e;
}

// Apply epilogue `EPI` to 8 consecutive columns and return them packed as bf16.
template <int EPI>
__device__ __forceinline__ uint4 epilogue8(const float (&acc)[8], const EpilogueArgs& ea,
                                           long long m, int n) {
  float v[8];
  if constexpr (EPI == kEpiPlain) {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = acc[j];
  } else if constexpr (EPI == kEpiBiasGelu) {
    const uint4 b = __ldg(reinterpret_cast<const uint4*>(ea.bias + n));
    const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 bb = unpack_bf16x2(bw[j]);
      const float u0 = bf16_round(bf16_round(acc[2 * j]) + bb.x);
      const float u1 = bf16_round(bf16_round(acc[2 * j + 1]) + bb.y);
      v[2 * j] = gelu_erf(u0);
      v[2 * j + 1] = gelu_erf(u1);
    }
  } else if constexpr (EPI == kEpiBiasResid || EPI == kEpiBiasResidSS) {
    const uint4 b = __ldg(reinterpret_cast<const uint4*>(ea.bias + n));
    const uint4 r = *reinterpret_cast<const uint4*>(ea.resid + m * ea.ld_resid + n);
    const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
    const uint32_t rw[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 bb = unpack_bf16x2(bw[j]);
      const float2 rr = unpack_bf16x2(rw[j]);
      v[2 * j] = bf16_round(bf16_round(acc[2 * j]) + bb.x) + rr.x;
      v[2 * j + 1] = bf16_round(bf16_round(acc[2 * j + 1]) + bb.y) + rr.y;
    }
  } else if constexpr (EPI == kEpiColScale) {
    const float4 s0 = __ldg(reinterpret_cast<const float4*>(ea.col_scale + n));
    const float4 s1 = __ldg(reinterpret_cast<const float4*>(ea.col_scale + n + 4));
    v[0] = acc[0] * s0.x; v[1] = acc[1] * s0.y; v[2] = acc[2] * s0.z; v[3] = acc[3] * s0.w;
    v[4] = acc[4] * s1.x; v[5] = acc[5] * s1.y; v[6] = acc[6] * s1.z; v[7] = acc[7] * s1.w;
  } else if constexpr (EPI == kEpiScaleBiasGelu || EPI == kEpiScaleBiasResid) {
    const float4 s0 = __ldg(reinterpret_cast<const float4*>(ea.col_scale + n));
    const float4 s1 = __ldg(reinterpret_cast<const float4*>(ea.col_scale + n + 4));
    const float sc[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    const uint4 b = __ldg(reinterpret_cast<const uint4*>(ea.bias + n));
    const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
    uint32_t rw[4] = {0u, 0u, 0u, 0u};
    if constexpr (EPI == kEpiScaleBiasResid) {
      const uint4 r = *reinterpret_cast<const uint4*>(ea.resid + m * ea.ld_resid + n);
      rw[0] = r.x; rw[1] = r.y; rw[2] = r.z; rw[3] = r.w;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 bb = unpack_bf16x2(bw[j]);
      const float u0 = bf16_round(bf16_round(acc[2 * j] * sc[2 * j]) + bb.x);
      const float u1 = bf16_round(bf16_round(acc[2 * j + 1] * sc[2 * j + 1]) + bb.y);
      if constexpr (EPI == kEpiScaleBiasGelu) {
        v[2 * j] = gelu_erf(u0);
        v[2 * j + 1] = gelu_erf(u1);
      } else {
        const float2 rr = unpack_bf16x2(rw[j]);
        v[2 * j] = u0 + rr.x;
        v[2 * j + 1] = u1 + rr.y;
      }
    }
  } else {
    // kinds whose tiles never reach this packer (fp32 and peer-store outputs)
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = acc[j];
  }
  uint4 out;
  out.x = pack_bf16x2(v[0], v[1]);
  out.y = pack_bf16x2(v[2], v[3]);
  out.z = pack_bf16x2(v[4], v[5]);
  out.w = pack_bf16x2(v[6], v[7]);
  return out;
}

namespace gemm {
// Fixed by the instruction shape and the 128-byte swizzle atom.
constexpr int BM = 128;
constexpr int BK = 64;
constexpr int NUM_THREADS = 320;            // 2 control warps + 8 epilogue warps
constexpr int EPI_THREADS = 256;
constexpr int GROUP_ROWS = 2048;            // rasterisation group: output rows sharing W panels in L2
constexpr int SCHED_DEPTH = 8;              // tile ids in flight producer -> consumers
// Tunable per launch (the tuning cache's block_n / shared_memory_stages):
// tile width BN in {128, 256} and pipeline depth STAGES.
constexpr int a_bytes() { return BM * BK * 2; }
constexpr int b_bytes(int bn) { return BK * bn * 2; }
constexpr int stage_bytes(int bn) { return a_bytes() + b_bytes(bn); }
constexpr int smem_bytes(int bn, int stages) {
  return stages * stage_bytes(bn) + 1024 /*align*/ + 512 /*barriers, tile ring*/;
}
constexpr int tmem_cols(int bn) { return 2 * bn; }  // two accumulators
// Peer-store epilogue staging: 8 epilogue warps x 2 buffers x (32 x 32 fp32).
constexpr int kPeerStageBytes = 8 * 2 * 4096;
constexpr int smem_bytes_peer(int bn, int stages) {
  return stages * stage_bytes(bn) + 1024 /*barriers*/ + kPeerStageBytes + 1024 /*align*/;
}
constexpr int kMaxSmem = 232448;                    // 227 KB per CTA on sm_100
// Narrow weights (B as int8 / fp8 codes in HBM): BT selects the code type.
// Shared memory then holds three rings: A tiles and the weights' 1-byte codes
// (STAGES deep, one TMA barrier per slot, deep enough to cover load latency),
// and the bf16 B tiles the MMA reads (kBf16Stages deep), which kConvWarps
// extra warps fill by expanding the codes.
constexpr int kBtBf16 = 0, kBtInt8 = 1, kBtE4M3 = 2, kBtE5M2 = 3;
constexpr int kConvWarps = 8;
constexpr int kBf16Stages = 2;
constexpr int raw_bytes(int bn) { return BK * bn; }
constexpr int threads_for(int bt) { return NUM_THREADS + (bt ? 32 * kConvWarps : 0); }
constexpr int smem_bytes_narrow(int bn, int stages) {
  return stages * (a_bytes() + raw_bytes(bn)) + kBf16Stages * b_bytes(bn) + 1024 + 512;
}
}  // namespace gemm

// Four int8 codes -> four bf16 (exact: |q| <= 128 needs 8 bits). The byte plus
// 128 is placed in the low mantissa bits of 2^23, and 2^23 + 128 subtracted.
__device__ __forceinline__ void int8x4_to_bf16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t x = w ^ 0x80808080u;
  constexpr float kMagic = 8388736.0f;  // 2^23 + 128
  const float f0 = __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7440)) - kMagic;
  const float f1 = __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7441)) - kMagic;
  const float f2 = __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7442)) - kMagic;
  const float f3 = __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7443)) - kMagic;
  lo = __byte_perm(__float_as_uint(f0), __float_as_uint(f1), 0x7632);
  hi = __byte_perm(__float_as_uint(f2), __float_as_uint(f3), 0x7632);
}

// Two fp8 codes (low byte first) -> two bf16, through the hardware fp8 -> fp16
// conversion (exact) and fp16 -> fp32 -> bf16 (exact: an fp8 value has at most
// 4 significant bits and lies in bf16's exponent range).
template <int BT>
__device__ __forceinline__ uint32_t fp8x2_to_bf16x2(uint32_t codes16) {
  uint32_t h;
  const uint16_t c = static_cast<uint16_t>(codes16);
  if constexpr (BT == gemm::kBtE4M3)
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(c));
  else
    asm("cvt.rn.f16x2.e5m2x2 %0, %1;" : "=r"(h) : "h"(c));
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h));
  return pack_bf16x2(f.x, f.y);
}

// 16 codes -> 16 bf16 (two 16-byte chunks).
template <int BT>
__device__ __forceinline__ void codes16_to_bf16(const uint4 w, uint4& o0, uint4& o1) {
  if constexpr (BT == gemm::kBtInt8) {
    int8x4_to_bf16x4(w.x, o0.x, o0.y);
    int8x4_to_bf16x4(w.y, o0.z, o0.w);
    int8x4_to_bf16x4(w.z, o1.x, o1.y);
    int8x4_to_bf16x4(w.w, o1.z, o1.w);
  } else {
    o0.x = fp8x2_to_bf16x2<BT>(w.x & 0xFFFFu);
    o0.y = fp8x2_to_bf16x2<BT>(w.x >> 16);
    o0.z = fp8x2_to_bf16x2<BT>(w.y & 0xFFFFu);
    o0.w = fp8x2_to_bf16x2<BT>(w.y >> 16);
    o1.x = fp8x2_to_bf16x2<BT>(w.z & 0xFFFFu);
    o1.y = fp8x2_to_bf16x2<BT>(w.z >> 16);
    o1.z = fp8x2_to_bf16x2<BT>(w.w & 0xFFFFu);
    o1.w = fp8x2_to_bf16x2<BT>(w.w >> 16);
  }
}

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int group_m, int& mb,
                                            int& nb) {
  const int per_group = group_m * tiles_n;
  const int g = t / per_group;
  const int first_m = g * group_m;
  const int gm = min(group_m, tiles_m - first_m);
  const int local = t - g * per_group;
  mb = first_m + local % gm;
  nb = local / gm;
}

template <int EPI, int BN, int STAGES, int BT = gemm::kBtBf16>
__global__ void __launch_bounds__(gemm::threads_for(BT), 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a,
                   const __grid_constant__ CUtensorMap map_b, void* __restrict__ C, long long ldc,
                   int M, int N, int K, EpilogueArgs ea, int* err,
                   const __grid_constant__ PeerMaps peer_maps, int* tile_counter, int group_m) {
  using gemm::BM;
  using gemm::BK;
  using gemm::EPI_THREADS;
  constexpr int A_BYTES = gemm::a_bytes();
  constexpr int STAGE_BYTES = gemm::stage_bytes(BN);
  constexpr int B_BLOCK_BYTES = BK * 64 * 2;  // one 64-wide N block
  constexpr int TMEM_COLS = gemm::tmem_cols(BN);
  static_assert(BN == 128 || BN == 256, "tile width");
  static_assert((EPI == kEpiPeerStoreF32 ? gemm::smem_bytes_peer(BN, STAGES)
                 : BT                   ? gemm::smem_bytes_narrow(BN, STAGES)
                                        : gemm::smem_bytes(BN, STAGES)) <= gemm::kMaxSmem,
                "pipeline does not fit");
  static_assert(BT == gemm::kBtBf16 || (BN == 256 && EPI != kEpiPeerStoreF32),
                "narrow weights: 256-wide tiles, no peer-store epilogue");
  constexpr int BST = gemm::kBf16Stages;
  constexpr int RAW_BYTES = gemm::raw_bytes(BN);
  constexpr int B_BYTES = gemm::b_bytes(BN);
  constexpr int CONV_WARPS = BT ? gemm::kConvWarps : 0;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  // bf16 B: STAGES slots of [A | B]. Narrow B: [A ring][code ring][bf16 B ring].
  uint8_t* raw_ring = smem + STAGES * gemm::a_bytes();
  uint8_t* b_ring = raw_ring + STAGES * RAW_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(
      BT ? b_ring + BST * B_BYTES : smem + STAGES * STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  // tile-id ring from the producer to the MMA issuer and the epilogue warps
  uint64_t* sched_full = tempty_bar + 2;
  uint64_t* sched_empty = sched_full + gemm::SCHED_DEPTH;
  volatile int* sched_tile = reinterpret_cast<volatile int*>(sched_empty + gemm::SCHED_DEPTH);
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(const_cast<int*>(sched_tile) + gemm::SCHED_DEPTH);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);
  // narrow B: bf16 B ring barriers (after the tile ring; 8-byte aligned)
  uint64_t* bfull_bar = reinterpret_cast<uint64_t*>(tmem_base_slot + 4);
  uint64_t* bempty_bar = bfull_bar + gemm::kBf16Stages;

  const int warp = warp_id();
  const int lane = lane_id();
  const int tiles_m = (M + BM - 1) / BM;
  const int tiles_n = (N + BN - 1) / BN;
  const int num_tiles = tiles_m * tiles_n;
  const int num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      // freed by the MMA's commit (+ each converter warp, done with the codes)
      mbar_init(&empty_bar[s], 1 + CONV_WARPS);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], EPI_THREADS);
    }
    for (int i = 0; i < gemm::SCHED_DEPTH; ++i) {
      mbar_init(&sched_full[i], 1);
      // MMA issuer + one lane per epilogue warp (+ one per converter warp)
      mbar_init(&sched_empty[i], 1 + EPI_THREADS / 32 + CONV_WARPS);
    }
    if (BT) {
      for (int i = 0; i < BST; ++i) {
        mbar_init(&bfull_bar[i], CONV_WARPS);
        mbar_init(&bempty_bar[i], 1);
      }
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  if (warp == 0) {
    {
      // ---------------------------------------------------------- producer --
      // The whole warp runs the loop (warp-uniform values, waits agreed by a
      // vote); one elected lane issues each TMA load and barrier arrival.
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu,
                          mbar_wait(bar, parity, err, abort_flag, kErrTimeoutProducer));
      };
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int slot = 0;
      uint32_t sphase = 0;
      // First tile by CTA index, the rest from the launch's counter when one
      // is given (CTAs that start late, e.g. behind a collective holding some
      // SMs, then take fewer tiles), else by stride.
      int t = blockIdx.x;
      while (ok) {
        if (!wait(&sched_empty[slot], sphase ^ 1)) break;
        if (lane == 0) {
          sched_tile[slot] = t < num_tiles ? t : -1;
          mbar_arrive(&sched_full[slot]);
        }
        __syncwarp();
        if (++slot == gemm::SCHED_DEPTH) {
          slot = 0;
          sphase ^= 1;
        }
        if (t >= num_tiles) break;
        int next = 0;
        if (lane == 0)
          next = tile_counter ? static_cast<int>(gridDim.x) + atomicAdd(tile_counter, 1)
                              : t + static_cast<int>(gridDim.x);
        next = __shfl_sync(0xffffffffu, next, 0);
        int mb, nb;
        tile_coords(t, tiles_m, tiles_n, group_m, mb, nb);
        t = next;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!wait(&empty_bar[stage], phase ^ 1)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          if constexpr (BT == gemm::kBtBf16) {
            mbar_arrive_expect_tx_warp(&full_bar[stage], STAGE_BYTES);
            tma_load_2d_warp(sa, &map_a, &full_bar[stage], kb * BK, mb * BM);
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d_warp(sb + j * B_BLOCK_BYTES, &map_b, &full_bar[stage],
                               nb * BN + j * 64, kb * BK);
          } else {
            // A and the B codes of this k-block, both on the slot's barrier;
            // the converter warps expand the codes into the bf16 B ring
            uint8_t* ra = smem + stage * gemm::a_bytes();
            uint8_t* sr = raw_ring + stage * RAW_BYTES;
            mbar_arrive_expect_tx_warp(&full_bar[stage], gemm::a_bytes() + RAW_BYTES);
            tma_load_2d_warp(ra, &map_a, &full_bar[stage], kb * BK, mb * BM);
#pragma unroll
            for (int j = 0; j < BN / 128; ++j)
              tma_load_2d_warp(sr + j * (BK * 128), &map_b, &full_bar[stage], nb * BN + j * 128,
                               kb * BK);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    {
      // ------------------------------------------------------- MMA issuer --
      // The whole warp runs the loop with warp-uniform values and one elected
      // lane issues each MMA and commit (a single diverged thread issuing
      // MMAs back to back is slower than the tensor core). Every wait is
      // taken by all lanes and agreed with a vote, so the warp stays converged.
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, err, abort_flag, kErrTimeoutMma));
      };
      constexpr uint32_t idesc = make_idesc_bf16(BM, BN, false, true);
      int stage = 0;
      uint32_t phase = 0;
      int bstage = 0;  // narrow B: bf16 B ring
      uint32_t bphase = 0;
      int local = 0;
      bool ok = true;
      int slot = 0;
      uint32_t sphase = 0;
      for (;; ++local) {
        if (!wait(&sched_full[slot], sphase)) break;
        const int t = sched_tile[slot];
        __syncwarp();
        if (lane == 0) mbar_arrive(&sched_empty[slot]);
        __syncwarp();
        if (++slot == gemm::SCHED_DEPTH) {
          slot = 0;
          sphase ^= 1;
        }
        if (t < 0 || !ok) break;
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!wait(&tempty_bar[acc], acc_phase ^ 1)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!wait(&full_bar[stage], phase) ||
              (BT != gemm::kBtBf16 && !wait(&bfull_bar[bstage], bphase))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = BT ? smem_u32(smem + stage * A_BYTES)
                                     : smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t b_addr = BT ? smem_u32(b_ring + bstage * B_BYTES) : a_addr + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t adesc = make_sw128_desc(a_addr + kk * 32, 16, 1024);
            const uint64_t bdesc = make_sw128_desc(b_addr + kk * 2048, B_BLOCK_BYTES, 1024);
            tc_mma_f16_warp(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0);
          }
          tc_commit_warp(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
          if constexpr (BT != gemm::kBtBf16) {
            tc_commit_warp(&bempty_bar[bstage]);
            if (++bstage == BST) {
              bstage = 0;
              bphase ^= 1;
            }
          }
        }
        if (ok) tc_commit_warp(&tfull_bar[acc]);
      }
    }
  } else if (BT != gemm::kBtBf16 && warp >= 2 + EPI_THREADS / 32) {
    // --------------------------------------------------------- converters --
    // Each k-block's codes (BK rows x BN codes, two 128-byte swizzled boxes)
    // are expanded to bf16 into the next bf16 B slot (four 128-byte swizzled
    // boxes of 64 columns), in the order the producer loaded them; the tile
    // ring only tells how many k-blocks follow.
    const int ct = static_cast<int>(threadIdx.x) - 32 * (2 + EPI_THREADS / 32);
    auto wait = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, err, abort_flag, kErrTimeoutEpilogue));
    };
    int stage = 0, bstage = 0, slot = 0;
    uint32_t phase = 0, bphase = 0, sphase = 0;
    bool ok = true;
    while (ok) {
      if (!wait(&sched_full[slot], sphase)) break;
      const int t = sched_tile[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sched_empty[slot]);
      __syncwarp();
      if (++slot == gemm::SCHED_DEPTH) {
        slot = 0;
        sphase ^= 1;
      }
      if (t < 0) break;
      for (int kb = 0; kb < num_kb; ++kb) {
        // the codes have landed, and the MMA is done with this bf16 B slot
        if (!wait(&full_bar[stage], phase) || !wait(&bempty_bar[bstage], bphase ^ 1)) {
          ok = false;
          break;
        }
        const uint8_t* sr = raw_ring + stage * RAW_BYTES;
        uint8_t* sb = b_ring + bstage * B_BYTES;
#pragma unroll 2
        for (int u = ct; u < RAW_BYTES / 16; u += 32 * CONV_WARPS) {
          const int box = u >> 9;           // 128-code box (512 chunks each)
          const int k = (u >> 3) & 63;      // row (k)
          const int c8 = u & 7;             // 16-code chunk within the row
          const uint4 w =
              *reinterpret_cast<const uint4*>(sr + box * (BK * 128) + k * 128 + ((c8 ^ (k & 7)) << 4));
          uint4 o0, o1;
          codes16_to_bf16<BT>(w, o0, o1);
          uint8_t* row = sb + (2 * box + (c8 >> 2)) * B_BLOCK_BYTES + k * 128;
          const int cb = 2 * (c8 & 3);
          *reinterpret_cast<uint4*>(row + ((cb ^ (k & 7)) << 4)) = o0;
          *reinterpret_cast<uint4*>(row + (((cb + 1) ^ (k & 7)) << 4)) = o1;
        }
        fence_proxy_async_smem();  // the MMA reads the slot through the async proxy
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&bfull_bar[bstage]);
          mbar_arrive(&empty_bar[stage]);  // done with the codes
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
        if (++bstage == BST) {
          bstage = 0;
          bphase ^= 1;
        }
      }
    }
  } else {
    // ---------------------------------------------------------- epilogue --
    const int q = warp & 3;           // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;  // which 128-column half of the tile
    const int row = q * 32 + lane;
    int local = 0;
    int peer_issue = 0;  // TMA stores issued by this warp (peer-store epilogue)
    int slot = 0;
    uint32_t sphase = 0;
    for (;; ++local) {
      if (!mbar_wait(&sched_full[slot], sphase, err, abort_flag, kErrTimeoutEpilogue)) break;
      const int t = sched_tile[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sched_empty[slot]);
      if (++slot == gemm::SCHED_DEPTH) {
        slot = 0;
        sphase ^= 1;
      }
      if (t < 0) break;
      int mb, nb;
      tile_coords(t, tiles_m, tiles_n, group_m, mb, nb);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull_bar[acc], acc_phase, err, abort_flag, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      const long long m = static_cast<long long>(mb) * BM + row;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      float ss_row = 0.f;  // kEpiBiasResidSS: this thread's share of the row's sum of squares
#pragma unroll 1
      for (int cc = 0; cc < BN / 64; ++cc) {
        const int c = half * (BN / 64) + cc;
        uint32_t r[32];
        tmem_ld32(t_row + c * 32, r);
        tmem_ld_wait();
        const int n0 = nb * BN + c * 32;
        if constexpr (EPI == kEpiPeerStoreF32) {
          // Stage this warp's 32 rows x 32 columns (128-byte swizzled rows) and
          // send them to the owner rank's slot buffer with one TMA store: full
          // 128-byte lines over NVLink instead of per-thread 16-byte stores.
          const long long m0 = static_cast<long long>(mb) * BM + q * 32;
          const int owner = static_cast<int>(m0 / ea.rows_per_rank);
          uint8_t* buf = smem + STAGES * STAGE_BYTES + 1024 + (warp - 2) * 8192 + (peer_issue & 1) * 4096;
          if (lane == 0 && peer_issue >= 2) bulk_wait_group_read1();
          __syncwarp();
#pragma unroll
          for (int k = 0; k < 8; ++k)
            *reinterpret_cast<uint4*>(buf + lane * 128 + ((k ^ (lane & 7)) << 4)) =
                make_uint4(r[4 * k], r[4 * k + 1], r[4 * k + 2], r[4 * k + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && m0 < M && n0 < N) {
            const int y = static_cast<int>(ea.src_rank * ea.rows_per_rank + (m0 - owner * ea.rows_per_rank));
            tma_store_2d(&peer_maps.m[owner], buf, n0, y);
            bulk_commit_group();
          }
          ++peer_issue;
          continue;
        }
        if (m < M) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int n = n0 + g * 8;
            if (n < N) {
              float a8[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) a8[j] = __uint_as_float(r[g * 8 + j]);
              if constexpr (EPI == kEpiQkvScatter) {
                const int hd = ea.head_dim, width = ea.heads * hd;
                const int which = n / width, rem = n - which * width;
                const int hh = rem / hd, e = rem - hh * hd;
                const long long b = m / ea.seq, sq = m - b * ea.seq;
                __nv_bfloat16* dst =
                    ea.qkv[which] + ((b * ea.heads + hh) * ea.seq + sq) * hd + e;
                *reinterpret_cast<uint4*>(dst) = epilogue8<kEpiPlain>(a8, ea, m, n);
              } else if constexpr (EPI == kEpiF32) {
                float* cp = static_cast<float*>(C) + m * ldc + n;
                reinterpret_cast<float4*>(cp)[0] = make_float4(a8[0], a8[1], a8[2], a8[3]);
                reinterpret_cast<float4*>(cp)[1] = make_float4(a8[4], a8[5], a8[6], a8[7]);
              } else {
                const uint4 o = epilogue8<EPI>(a8, ea, m, n);
                *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(C) + m * ldc + n) = o;
                if constexpr (EPI == kEpiBiasResidSS) {
                  const uint32_t ow[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
                  for (int k = 0; k < 4; ++k) {
                    const float2 f = unpack_bf16x2(ow[k]);
                    ss_row = fmaf(f.x, f.x, ss_row);
                    ss_row = fmaf(f.y, f.y, ss_row);
                  }
                }
              }
            }
          }
        }
      }
      if constexpr (EPI == kEpiBiasResidSS) {
        if (m < M) ea.row_ss[m * ea.ss_stride + 2 * nb + half] = ss_row;
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);
    }
    if constexpr (EPI == kEpiPeerStoreF32) {
      if (lane == 0) bulk_wait_group0();  // every store has landed before the kernel ends
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace pkb200
