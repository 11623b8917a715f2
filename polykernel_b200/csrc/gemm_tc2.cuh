// gemm_tc2.cuh - the persistent tcgen05 GEMM on CTA pairs (cta_group::2).
//
//   C[M,N] = epilogue( A[M,K] @ B[K,N] )   A, B, C bf16 row-major, fp32 accumulate.
//
// Same contraction, epilogues and rounding as gemm_tc.cuh; the difference is
// the MMA: a cluster of two CTAs on two SMs computes a 256 x 256 output tile
// with tcgen05.mma.cta_group::2 (M=256, N=256, K=16). Each CTA holds its own
// 128 rows of A and its own 128 columns of B per stage (the instruction reads
// both halves), so an SM stages 32 KB per K-block instead of 48 KB for a
// 128 x 256 single-SM tile: less shared-memory traffic per MMA and six stages
// of look-ahead in the same space. Each CTA's TMEM holds its 128 rows x 256
// columns of the accumulator (two buffers, 512 columns).
//
// Roles (320 threads per CTA):
//   warp 0   TMA producer in both CTAs: its A half (128 x 64, K-major) and B
//            half (two 64 x 64 N-major boxes); the loads' byte counts land on
//            the leader CTA's full barrier (cta_group::2 loads, no multicast).
//   warp 1   TMEM allocator in both CTAs (cta_group::2); in the leader, the
//            MMA issuer (whole warp, one elected lane issues). Its commits
//            arrive on both CTAs' barriers (tcgen05.commit multicast).
//   warps 2-9 epilogue in both CTAs: drain the CTA's own accumulator rows.
// Tiles are statically assigned (cluster c takes tiles c, c + clusters, ...),
// so the pair needs no shared schedule. Every mbarrier wait is bounded as in
// gemm_tc.cuh; the two cluster barriers (after set-up, before TMEM release)
// are reached by every thread on every path.
#pragma once

#include "gemm_tc.cuh"

namespace pkb200 {
namespace gemm2 {
constexpr int BM = 128;       // rows per CTA (256 per pair)
constexpr int BN = 256;       // columns per pair tile (128 per CTA's B half)
constexpr int BK = 64;
constexpr int NUM_THREADS = 320;
constexpr int EPI_WARPS = 8;
constexpr int A_BYTES = BM * BK * 2;             // 16 KB
constexpr int B_BYTES = BK * (BN / 2) * 2;       // 16 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;   // 32 KB
constexpr int smem_bytes(int stages) { return stages * STAGE_BYTES + 1024 + 512; }
constexpr int kTmemCols = 2 * BN;
}  // namespace gemm2

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}

// Shared-memory address of the same variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

// TMA tile load whose completion (byte count) lands on the pair leader's
// barrier: `bar_leader` is the barrier's address in the leader CTA.
// Issued by a whole converged warp; one elected lane runs the instruction.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map,
                                                 uint32_t bar_leader, int c0, int c1) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];\n\t}" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_leader), "r"(c0), "r"(c1)
      : "memory");
}

// Issued by a whole converged warp; one elected lane runs the instruction.
__device__ __forceinline__ void tc_mma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` (same offset) in both CTAs of the pair when the MMAs
// issued so far have completed. Issued by a whole converged warp; one elected
// lane runs the instruction.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar) {
  const uint16_t mask = 0x3;
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;\n\t}" ::"r"(smem_u32(bar)), "h"(mask)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

template <int EPI, int STAGES>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(gemm2::NUM_THREADS, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap map_a,
                    const __grid_constant__ CUtensorMap map_b, void* __restrict__ C,
                    long long ldc, int M, int N, int K, EpilogueArgs ea, int* err,
                    int group_m) {
  using namespace gemm2;
  static_assert(EPI != kEpiPeerStoreF32 && EPI != kEpiQkvScatter, "single-SM kernel only");
  static_assert(smem_bytes(STAGES) <= gemm::kMaxSmem, "pipeline does not fit");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);  // leader's
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;  // leader's: both CTAs' epilogue warps arrive
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t cta = cluster_ctarank();
  const int cluster = static_cast<int>(blockIdx.x) >> 1;
  const int clusters = static_cast<int>(gridDim.x) >> 1;
  const int tiles_m = (M + 2 * BM - 1) / (2 * BM);
  const int tiles_n = (N + BN - 1) / BN;
  const int num_tiles = tiles_m * tiles_n;
  const int num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 2 * EPI_WARPS);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers exist before any cross-CTA arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    {
      // ---------------------------------------------------------- producer --
      // whole warp, warp-uniform values, one elected lane issues
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = cluster; t < num_tiles && ok; t += clusters) {
        int mb, nb;
        tile_coords(t, tiles_m, tiles_n, group_m, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!__all_sync(0xffffffffu, mbar_wait(&empty_bar[stage], phase ^ 1, err, abort_flag,
                                                 kErrTimeoutProducer))) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          const uint32_t bar = map_to_rank(smem_u32(&full_bar[stage]), 0);
          if (cta == 0) mbar_arrive_expect_tx_warp(&full_bar[stage], 2 * STAGE_BYTES);
          tma_load_2d_pair(sa, &map_a, bar, kb * BK, mb * 2 * BM + static_cast<int>(cta) * BM);
#pragma unroll
          for (int j = 0; j < 2; ++j)
            tma_load_2d_pair(sb + j * (BK * 128), &map_b, bar,
                             nb * BN + static_cast<int>(cta) * (BN / 2) + j * 64, kb * BK);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (cta == 0) {
      // ---------------------------------------------- MMA issuer (leader) --
      // The whole warp runs the loop (warp-uniform values, every wait agreed
      // by a vote); one elected lane issues each MMA and commit.
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, err, abort_flag, kErrTimeoutMma));
      };
      constexpr uint32_t idesc = make_idesc_bf16(2 * BM, BN, false, true);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = cluster; t < num_tiles && ok; t += clusters, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!wait(&tempty_bar[acc], acc_phase ^ 1)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!wait(&full_bar[stage], phase)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = make_sw128_desc(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = make_sw128_desc(b_addr + kk * 2048, BK * 128, 1024);
            tc_mma_pair(d_tmem, ad, bd, idesc, (kb | kk) != 0);
          }
          tc_commit_pair(&empty_bar[stage]);  // both CTAs may refill this stage
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) tc_commit_pair(&tfull_bar[acc]);  // both CTAs' accumulator halves ready
      }
    }
  } else {
    // ---------------------------------------------------------- epilogue --
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;  // which 128-column half of the tile
    const int row = q * 32 + lane;
    const uint32_t tempty_leader0 = map_to_rank(smem_u32(&tempty_bar[0]), 0);
    int local = 0;
    for (int t = cluster; t < num_tiles; t += clusters, ++local) {
      int mb, nb;
      tile_coords(t, tiles_m, tiles_n, group_m, mb, nb);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull_bar[acc], acc_phase, err, abort_flag, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      const long long m = static_cast<long long>(mb) * 2 * BM + static_cast<long long>(cta) * BM + row;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      float ss_row = 0.f;  // kEpiBiasResidSS: this thread's share of the row's sum of squares
#pragma unroll 1
      for (int cc = 0; cc < BN / 64; ++cc) {
        const int c = half * (BN / 64) + cc;
        uint32_t r[32];
        tmem_ld32(t_row + c * 32, r);
        tmem_ld_wait();
        const int n0 = nb * BN + c * 32;
        if (m < M) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int n = n0 + g * 8;
            if (n < N) {
              float a8[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) a8[j] = __uint_as_float(r[g * 8 + j]);
              if constexpr (EPI == kEpiF32) {
                float* cp = static_cast<float*>(C) + m * ldc + n;
                reinterpret_cast<float4*>(cp)[0] = make_float4(a8[0], a8[1], a8[2], a8[3]);
                reinterpret_cast<float4*>(cp)[1] = make_float4(a8[4], a8[5], a8[6], a8[7]);
              } else {
                const uint4 o = epilogue8<EPI>(a8, ea, m, n);
                *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(C) + m * ldc + n) = o;
                if constexpr (EPI == kEpiBiasResidSS) {
                  const uint32_t ow[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
                  for (int k2 = 0; k2 < 4; ++k2) {
                    const float2 f = unpack_bf16x2(ow[k2]);
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
        // two 128-column halves per 256-wide tile: the same (row, 2*nb+half)
        // slots a 256-wide single-SM tile writes
        if (m < M) ea.row_ss[m * ea.ss_stride + 2 * nb + half] = ss_row;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader0 + acc * 8);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no CTA releases TMEM or exits while its pair may still signal it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

}  // namespace pkb200
