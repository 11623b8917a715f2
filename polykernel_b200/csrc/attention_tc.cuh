// attention_tc.cuh - causal prefill attention with fused KV-cache append on
// tcgen05 tensor cores (sm_100a), head_dim 64 or 128.
//
// Semantics follow the reference's kernels/generated/attention_prefill.cu:84-155
// and the golden tests/golden/golden.py:139-172: scores = (q . k) * scale in
// fp32, query row i (of S_q) sees key positions p <= S_kv - S_q + i when
// causal (attention_prefill.cu:103), softmax in fp32, P.V accumulated in fp32,
// one bf16 rounding of O. Rows that see no key produce 0 (attention_prefill.cu:154).
//
// One CTA per (pair of 128-query tiles A and B, batch*head). Roles (320 threads):
//   warps 0-3  softmax for tile A, warps 4-7 softmax for tile B. Thread r of a
//              group owns query row r (= TMEM lane r). It reads its S row with
//              tcgen05.ld, keeps the running max/sum in the exp2 domain, and
//              writes P (bf16 pairs) back into the same TMEM columns with
//              tcgen05.st, where the P.V MMA reads it as its A operand. O is
//              rescaled in TMEM only when the row max grew by more than 2^8
//              (exact: every P and the final sum use the same stale max). At
//              the end the group normalises O and stores it.
//   warp 8     TMA producer: Q tiles once; K and V tiles (128 keys) through two
//              2-deep rings shared by both query tiles. For the append entry
//              point, the CTA whose query tiles match a tile of new rows also
//              writes those K/V tiles from shared memory into the cache with
//              TMA stores, so the append costs no extra HBM read.
//   warp 9     TMEM owner + single-thread MMA issuer. Order per key tile j:
//              PV_A(j); S_A(j+1); PV_B(j); S_B(j+1). S_X(j+1) overwrites the TMEM
//              columns that held P_X(j), so the issuer waits for PV_X(j) to
//              complete first (PV_B(j) is queued meanwhile, keeping the tensor
//              pipe busy). The two groups interleave: while one waits for its
//              MMAs the other runs its exponentials.
// TMEM (512 columns): S/P_A [0,128), S/P_B [128,256), O_A [256,256+D), O_B [384,384+D).
//
// Key positions come from two sources (KvSources): A (rows [0, n_a), the
// cache prefix or the whole K/V of the plain entry point) and B (the new
// rows, positions n_a + r). Key tiles never straddle the two: a source's last
// tile may be partial, and the keys past its end are masked.
#pragma once

#include "simt_kernels.cuh"

namespace pkb200 {
namespace attn {
constexpr int BM = 128;       // query rows per tile (two tiles per CTA)
constexpr int BN = 128;       // keys per tile
constexpr int NUM_THREADS = 320;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

template <int D>
struct Layout {
  static constexpr int DBOX = D / 64;                 // 64-column boxes per row
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int OFF_Q = 0;                      // Q_A, Q_B
  static constexpr int OFF_K = OFF_Q + 2 * Q_BYTES;    // 2 stages
  static constexpr int OFF_V = OFF_K + 2 * KV_BYTES;   // 2 stages
  static constexpr int OFF_BAR = OFF_V + 2 * KV_BYTES;
  static constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;
};
}  // namespace attn

struct AttnTcParams {
  int BH;
  int S_q;
  int n_a;        // rows in source A
  int n_b;        // rows in source B (0 if none)
  int tiles_a;    // ceil(n_a / BN)
  int tiles_b;    // ceil(n_b / BN)
  float scale_log2;  // scale * log2(e)
  int causal;
  int append;     // 1: write source-B tiles into the cache maps
  int num_qtiles;
  int num_pairs;
  __nv_bfloat16* O;
  int* err;
};

// Number of key tiles query tile `qt` visits (0 if the tile is past S_q).
__device__ __forceinline__ int attn_tiles_for(const AttnTcParams& p, int qt) {
  if (qt * attn::BM >= p.S_q) return 0;
  const int S_kv = p.n_a + p.n_b;
  const int last_row = min(qt * attn::BM + attn::BM - 1, p.S_q - 1);
  const int limit_last = p.causal ? (S_kv - p.S_q + last_row) : (S_kv - 1);
  int n = 0;
  for (int j = 0; j < p.tiles_a + p.tiles_b; ++j) {
    const int p0 = j < p.tiles_a ? j * attn::BN : p.n_a + (j - p.tiles_a) * attn::BN;
    if (p0 <= limit_last) n = j + 1;
  }
  return n;
}

template <int D>
__global__ void __launch_bounds__(attn::NUM_THREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap map_q,
                        const __grid_constant__ CUtensorMap map_ka,
                        const __grid_constant__ CUtensorMap map_va,
                        const __grid_constant__ CUtensorMap map_kb,
                        const __grid_constant__ CUtensorMap map_vb,
                        const __grid_constant__ CUtensorMap map_kc_store,
                        const __grid_constant__ CUtensorMap map_vc_store, AttnTcParams p) {
  using namespace attn;
  using L = Layout<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* k_empty = bars + 3;   // [2]
  uint64_t* v_full = bars + 5;    // [2]
  uint64_t* v_empty = bars + 7;   // [2]
  uint64_t* s_full = bars + 9;    // [2]  per query tile (A, B)
  uint64_t* p_full = bars + 11;   // [2]
  uint64_t* pv_done = bars + 13;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const int bh = blockIdx.y;
  const int pair = p.num_pairs - 1 - static_cast<int>(blockIdx.x);  // heavy pairs first
  const int qt_a = 2 * pair, qt_b = 2 * pair + 1;
  const int n_tile0 = attn_tiles_for(p, qt_a);
  const int n_tile1 = attn_tiles_for(p, qt_b);
  const int nmax = max(n_tile0, n_tile1);
  const bool valid_b = qt_b * BM < p.S_q;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&pv_done[i], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    if (lane == 0 && nmax > 0) {
      // -------------------------------------------------------- producer --
      tma_prefetch_desc(&map_q);
      mbar_arrive_expect_tx(q_full, (valid_b ? 2 : 1) * L::Q_BYTES);
#pragma unroll
      for (int c = 0; c < L::DBOX; ++c) {
        tma_load_3d(smem + L::OFF_Q + c * (BM * 128), &map_q, q_full, c * 64, qt_a * BM, bh);
        if (valid_b)
          tma_load_3d(smem + L::OFF_Q + L::Q_BYTES + c * (BM * 128), &map_q, q_full, c * 64,
                      qt_b * BM, bh);
      }
      for (int j = 0; j < nmax; ++j) {
        const bool from_a = j < p.tiles_a;
        const int row0 = from_a ? j * BN : (j - p.tiles_a) * BN;
        const CUtensorMap* mk = from_a ? &map_ka : &map_kb;
        const CUtensorMap* mv = from_a ? &map_va : &map_vb;
        const int new_tile = row0 / BN;
        const bool do_append = p.append && !from_a && (new_tile == qt_a || new_tile == qt_b);
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        uint8_t* sk = smem + L::OFF_K + st * L::KV_BYTES;
        uint8_t* sv = smem + L::OFF_V + st * L::KV_BYTES;
        if (!mbar_wait(&k_empty[st], ph ^ 1, p.err, abort_flag, kErrTimeoutProducer)) break;
        mbar_arrive_expect_tx(&k_full[st], L::KV_BYTES);
#pragma unroll
        for (int c = 0; c < L::DBOX; ++c)
          tma_load_3d(sk + c * (BN * 128), mk, &k_full[st], c * 64, row0, bh);
        if (!mbar_wait(&v_empty[st], ph ^ 1, p.err, abort_flag, kErrTimeoutProducer)) break;
        mbar_arrive_expect_tx(&v_full[st], L::KV_BYTES);
#pragma unroll
        for (int c = 0; c < L::DBOX; ++c)
          tma_load_3d(sv + c * (BN * 128), mv, &v_full[st], c * 64, row0, bh);
        if (do_append) {
          // Write this tile of new rows into the cache (rows n_a + row0 ...).
          if (!mbar_wait(&k_full[st], ph, p.err, abort_flag, kErrTimeoutProducer)) break;
#pragma unroll
          for (int c = 0; c < L::DBOX; ++c)
            tma_store_3d(&map_kc_store, sk + c * (BN * 128), c * 64, p.n_a + row0, bh);
          if (!mbar_wait(&v_full[st], ph, p.err, abort_flag, kErrTimeoutProducer)) break;
#pragma unroll
          for (int c = 0; c < L::DBOX; ++c)
            tma_store_3d(&map_vc_store, sv + c * (BN * 128), c * 64, p.n_a + row0, bh);
          bulk_commit_group();
          bulk_wait_group_read0();
        }
      }
      bulk_wait_group0();
    }
  } else if (warp == 9) {
    if (lane == 0 && nmax > 0) {
      // ------------------------------------------------------ MMA issuer --
      constexpr uint32_t idesc_s = make_idesc_bf16(BM, BN, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16(BM, D, false, true);
      bool ok = mbar_wait(q_full, 0, p.err, abort_flag, kErrTimeoutMma);
      auto issue_s = [&](int x, int j) {
        const uint32_t q_addr = smem_u32(smem + L::OFF_Q + x * L::Q_BYTES);
        const uint32_t k_addr = smem_u32(smem + L::OFF_K + (j & 1) * L::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          const uint64_t ad = make_sw128_desc(q_addr + off, 16, 1024);
          const uint64_t bd = make_sw128_desc(k_addr + off, 16, 1024);
          tc_mma_f16(tmem + x * BN, ad, bd, idesc_s, kk != 0);
        }
        tc_commit(&s_full[x]);
      };
      auto issue_pv = [&](int x, int j) {
        const uint32_t v_addr = smem_u32(smem + L::OFF_V + (j & 1) * L::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t bd = make_sw128_desc(v_addr + kk * 2048, BN * 128, 1024);
          tc_mma_f16_tmem_a(tmem + 256 + x * 128, tmem + x * BN + kk * 8, bd, idesc_o,
                            (j | kk) != 0);
        }
        tc_commit(&pv_done[x]);
      };
      // prologue: S for key tile 0
      if (ok) ok = mbar_wait(&k_full[0], 0, p.err, abort_flag, kErrTimeoutMma);
      if (ok) {
        tc_fence_after();
        if (n_tile0 > 0) issue_s(0, 0);
        if (n_tile1 > 0) issue_s(1, 0);
        tc_commit(&k_empty[0]);
      }
      for (int j = 0; j < nmax && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        const int jn = j + 1;
        bool v_ready = false, k_next_ready = false;
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          const int nt = x == 0 ? n_tile0 : n_tile1;
          if (!ok || j >= nt) continue;
          if (!v_ready) {
            ok = mbar_wait(&v_full[st], ph, p.err, abort_flag, kErrTimeoutMma);
            v_ready = true;
          }
          if (ok) ok = mbar_wait(&p_full[x], j & 1, p.err, abort_flag, kErrTimeoutMma);
          if (!ok) break;
          tc_fence_after();
          issue_pv(x, j);
          if (jn < nt) {
            if (!k_next_ready) {
              ok = mbar_wait(&k_full[jn & 1], (jn >> 1) & 1, p.err, abort_flag, kErrTimeoutMma);
              k_next_ready = true;
            }
            // S_X(j+1) reuses the TMEM columns P_X(j) occupies: wait for PV_X(j).
            if (ok) ok = mbar_wait(&pv_done[x], j & 1, p.err, abort_flag, kErrTimeoutMma);
            if (!ok) break;
            tc_fence_after();
            issue_s(x, jn);
          }
        }
        if (!ok) break;
        tc_commit(&v_empty[st]);
        if (k_next_ready) tc_commit(&k_empty[jn & 1]);
      }
    }
  } else {
    // ----------------------------------------------------------- softmax --
    const int x = warp >> 2;        // query tile A (0) or B (1)
    const int qw = warp & 3;        // TMEM lane quarter
    const int r = qw * 32 + lane;   // query row within the tile == TMEM lane
    const int qt = x == 0 ? qt_a : qt_b;
    const int qi = qt * BM + r;
    const int ntiles = x == 0 ? n_tile0 : n_tile1;
    const int S_kv = p.n_a + p.n_b;
    const int limit = p.causal ? (S_kv - p.S_q + qi) : (S_kv - 1);
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(qw * 32) << 16);
    const uint32_t s_col = x * BN;
    const uint32_t o_col = 256 + x * 128;
    float m_run = -INFINITY;
    float l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const bool from_a = j < p.tiles_a;
      const int p0 = from_a ? j * BN : p.n_a + (j - p.tiles_a) * BN;
      const int cnt = from_a ? min(BN, p.n_a - j * BN) : min(BN, p.n_b - (j - p.tiles_a) * BN);
      const int nvalid = max(0, min(cnt, limit - p0 + 1));
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[x], j & 1, p.err, abort_flag,
                                             kErrTimeoutSoftmax));
      if (!ok) break;
      tc_fence_after();
      const bool full = __all_sync(0xffffffffu, nvalid == BN);
      // The tile is processed in two halves of 64 keys. Half h reads S
      // columns [64h, 64h+64) and writes its P (32 columns of bf16 pairs) to
      // columns [32h, 32h+32), which the first half has already consumed.
      // When the running max is known and the tile is fully visible, the
      // exponentials use it straight away while the half's max is computed
      // alongside; only if that max exceeds the running one by more than the
      // rescale threshold is the half redone (rare). Otherwise the max comes
      // first. When the max grows, O, the row sum, and (in the second half)
      // the first half's P are rescaled, so P and the sum always share one max.
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        uint32_t sv[64];
        tmem_ld32(lane_base + s_col + h * 64, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
        tmem_ld32(lane_base + s_col + h * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
        tmem_ld_wait();
        if (!full) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (h * 64 + c >= nvalid) sv[c] = __float_as_uint(-INFINITY);
        }
        uint32_t pk[32];
        float ls4[4] = {0.f, 0.f, 0.f, 0.f};
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        const bool optimistic = full && m_run != -INFINITY;
        if (optimistic) {
          const float neg_m = -m_run;
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            const float s0 = __uint_as_float(sv[2 * k]), s1 = __uint_as_float(sv[2 * k + 1]);
            mx4[k & 3] = fmax3(mx4[k & 3], s0, s1);
            const float e0 = fast_exp2(fmaf(s0, p.scale_log2, neg_m));
            const float e1 = fast_exp2(fmaf(s1, p.scale_log2, neg_m));
            ls4[(2 * k) & 3] += e0;
            ls4[(2 * k + 1) & 3] += e1;
            pk[k] = pack_bf16x2(e0, e1);
          }
        } else {
#pragma unroll
          for (int k = 0; k < 32; ++k)
            mx4[k & 3] = fmax3(mx4[k & 3], __uint_as_float(sv[2 * k]), __uint_as_float(sv[2 * k + 1]));
        }
        const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * p.scale_log2;
        const float m_new = fmaxf(m_run, mx);
        const bool grow = m_new > m_run + kRescaleThreshold || (m_run == -INFINITY && m_new > -INFINITY);
        const bool any_grow = __any_sync(0xffffffffu, grow);
        if (!optimistic || any_grow) {
          const float alpha = grow ? (m_run == -INFINITY ? 0.f : fast_exp2(m_run - m_new)) : 1.f;
          if (grow) m_run = m_new;
          if (any_grow && j > 0) {
            // O_X holds P_0..P_{j-1} V and is complete: S_X(j) was issued only
            // after PV_X(j-1) finished, and S_X(j) has completed.
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
              uint32_t o[32];
              tmem_ld32(lane_base + o_col + c * 32, o);
              tmem_ld_wait();
#pragma unroll
              for (int k = 0; k < 32; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
              tmem_st32(lane_base + o_col + c * 32, o);
            }
          }
          if (any_grow && h == 1) {
            // the first half's P was made with the old max
            uint32_t q[32];
            tmem_ld32(lane_base + s_col, q);
            tmem_ld_wait();
#pragma unroll
            for (int k = 0; k < 32; ++k) {
              const float2 f = unpack_bf16x2(q[k]);
              q[k] = pack_bf16x2(f.x * alpha, f.y * alpha);
            }
            tmem_st32(lane_base + s_col, q);
          }
          l_run *= alpha;
          const float neg_m = (m_run == -INFINITY) ? 0.f : -m_run;
#pragma unroll
          for (int q = 0; q < 4; ++q) ls4[q] = 0.f;
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            const float e0 = fast_exp2(fmaf(__uint_as_float(sv[2 * k]), p.scale_log2, neg_m));
            const float e1 = fast_exp2(fmaf(__uint_as_float(sv[2 * k + 1]), p.scale_log2, neg_m));
            ls4[(2 * k) & 3] += e0;
            ls4[(2 * k + 1) & 3] += e1;
            pk[k] = pack_bf16x2(e0, e1);
          }
        }
        tmem_st32(lane_base + s_col + h * 32, pk);
        l_run += (ls4[0] + ls4[1]) + (ls4[2] + ls4[3]);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[x]);
    }
    // ------------------------------------------------------- epilogue --
    if (x == 0 || valid_b) {
      __nv_bfloat16* orow = p.O + (static_cast<long long>(bh) * p.S_q + qi) * D;
      if (ntiles > 0 && ok) {
        ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[x], (ntiles - 1) & 1, p.err, abort_flag,
                                               kErrTimeoutSoftmax));
      }
      if (ok) {
        tc_fence_after();
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          if (ntiles > 0) {
            tmem_ld32(lane_base + o_col + c * 32, o);
            tmem_ld_wait();
          } else {
#pragma unroll
            for (int k = 0; k < 32; ++k) o[k] = 0u;
          }
          if (qi < p.S_q) {
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              uint4 v;
              v.x = pack_bf16x2(__uint_as_float(o[g * 8 + 0]) * inv, __uint_as_float(o[g * 8 + 1]) * inv);
              v.y = pack_bf16x2(__uint_as_float(o[g * 8 + 2]) * inv, __uint_as_float(o[g * 8 + 3]) * inv);
              v.z = pack_bf16x2(__uint_as_float(o[g * 8 + 4]) * inv, __uint_as_float(o[g * 8 + 5]) * inv);
              v.w = pack_bf16x2(__uint_as_float(o[g * 8 + 6]) * inv, __uint_as_float(o[g * 8 + 7]) * inv);
              *reinterpret_cast<uint4*>(orow + c * 32 + g * 8) = v;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------- host side --
inline bool attention_tc_supported(const KvSources& kv, int S_q, int D, const void* Q,
                                   const void* O) {
  auto al = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
  if (!(D == 64 || D == 128)) return false;
  if (S_q <= 0) return false;
  if (kv.n_a < 0 || kv.n_b < 0) return false;
  if (!al(Q) || !al(O)) return false;
  if (kv.n_a > 0 && (!al(kv.Ka) || !al(kv.Va))) return false;
  if (kv.n_b > 0 && (!al(kv.Kb) || !al(kv.Vb))) return false;
  return true;
}

}  // namespace pkb200
