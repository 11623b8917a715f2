// attention_tc.cuh - causal prefill attention with fused KV-cache append on
// tcgen05 tensor cores (sm_100a), head_dim 64 or 128.
//
// Semantics follow the reference's kernels/generated/attention_prefill.cu:84-155
// and the golden tests/golden/golden.py:139-172: scores = (q . k) * scale in
// fp32, query row i (of S_q) sees key positions p <= S_kv - S_q + i when
// causal (attention_prefill.cu:103), softmax in fp32, P.V accumulated in fp32,
// one bf16 rounding of O. Rows that see no key produce 0 (attention_prefill.cu:154).
//
// One CTA per (128-query tile, batch*head). Roles:
//   warps 0-3  softmax: thread r owns query row r (= TMEM lane r). Reads the
//              S row with tcgen05.ld, online max/sum in the exp2 domain,
//              writes P (bf16) into shared memory in the 128B-swizzled K-major
//              layout the PV MMA reads, rescales O in TMEM only when the row
//              max grew by more than 2^8 (the result is exact either way:
//              every P and the final sum use the same stale max), and at the
//              end normalises O and stores it.
//   warp 4     TMA producer: Q once; K and V tiles (128 keys) through two
//              2-deep rings. For the append entry point, the CTA whose query
//              tile matches a tile of new rows also writes those K/V tiles
//              from shared memory into the cache with TMA stores, so the
//              append costs no extra HBM read.
//   warp 5     TMEM owner + single-thread MMA issuer. S_j = Q K_j^T into one of
//              two TMEM S buffers; O += P_{j-1} V_{j-1} is issued after S_j so
//              the tensor cores work on S_j while the softmax warps handle S_{j-1}.
// TMEM: S0 cols [0,128), S1 [128,256), O [256, 256+D).
//
// Key positions come from two sources (KvSources): A (rows [0, n_a), the
// cache prefix or the whole K/V of the plain entry point) and B (the new
// rows, positions n_a + r). Tiles never straddle the two: a source's last tile
// may be partial, and the keys past its end are masked.
#pragma once

#include "simt_kernels.cuh"

namespace pkb200 {
namespace attn {
constexpr int BM = 128;       // query rows per CTA
constexpr int BN = 128;       // keys per tile
constexpr int NUM_THREADS = 192;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

template <int D>
struct Layout {
  static constexpr int DBOX = D / 64;                 // 64-column boxes per row
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int P_BYTES = BM * BN * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + 2 * KV_BYTES;
  static constexpr int OFF_P = OFF_V + 2 * KV_BYTES;
  static constexpr int OFF_BAR = OFF_P + 2 * P_BYTES;
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
  __nv_bfloat16* O;
  int* err;
};

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
  uint64_t* s_full = bars + 9;    // [2]
  uint64_t* s_free = bars + 11;   // [2]
  uint64_t* p_full = bars + 13;   // [2]
  uint64_t* pv_done = bars + 15;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const int bh = blockIdx.x;
  const int qt = p.num_qtiles - 1 - static_cast<int>(blockIdx.y);  // heavy tiles first
  const int q0 = qt * BM;
  const int S_kv = p.n_a + p.n_b;
  // Last key position any row of this tile may see.
  const int last_row = min(q0 + BM - 1, p.S_q - 1);
  const int limit_last = p.causal ? (S_kv - p.S_q + last_row) : (S_kv - 1);
  // Number of key tiles this CTA visits (tile start positions are increasing).
  int ntiles = 0;
  for (int j = 0; j < p.tiles_a + p.tiles_b; ++j) {
    const int p0 = j < p.tiles_a ? j * BN : p.n_a + (j - p.tiles_a) * BN;
    if (p0 <= limit_last) ntiles = j + 1;
  }

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&pv_done[i], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    if (lane == 0 && ntiles > 0) {
      // -------------------------------------------------------- producer --
      tma_prefetch_desc(&map_q);
      mbar_arrive_expect_tx(q_full, L::Q_BYTES);
#pragma unroll
      for (int c = 0; c < L::DBOX; ++c)
        tma_load_3d(smem + L::OFF_Q + c * (BM * 128), &map_q, q_full, c * 64, q0, bh);
      for (int j = 0; j < ntiles; ++j) {
        const bool from_a = j < p.tiles_a;
        const int row0 = from_a ? j * BN : (j - p.tiles_a) * BN;
        const CUtensorMap* mk = from_a ? &map_ka : &map_kb;
        const CUtensorMap* mv = from_a ? &map_va : &map_vb;
        const bool do_append = p.append && !from_a && (row0 / BN) == qt;
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
  } else if (warp == 5) {
    if (lane == 0 && ntiles > 0) {
      // ------------------------------------------------------ MMA issuer --
      constexpr uint32_t idesc_s = make_idesc_bf16(BM, BN, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16(BM, D, false, true);
      const uint32_t q_addr = smem_u32(smem + L::OFF_Q);
      const uint32_t o_tmem = tmem + 256;
      bool ok = mbar_wait(q_full, 0, p.err, abort_flag, kErrTimeoutMma);
      auto issue_pv = [&](int i) -> bool {
        const int st = i & 1;
        const uint32_t ph = (i >> 1) & 1;
        if (!mbar_wait(&v_full[st], ph, p.err, abort_flag, kErrTimeoutMma)) return false;
        if (!mbar_wait(&p_full[st], ph, p.err, abort_flag, kErrTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t p_addr = smem_u32(smem + L::OFF_P + st * L::P_BYTES);
        const uint32_t v_addr = smem_u32(smem + L::OFF_V + st * L::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t ad = make_sw128_desc(p_addr + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = make_sw128_desc(v_addr + kk * 2048, BN * 128, 1024);
          tc_mma_f16(o_tmem, ad, bd, idesc_o, (i | kk) != 0);
        }
        tc_commit(&v_empty[st]);
        tc_commit(&pv_done[st]);
        return true;
      };
      for (int j = 0; j < ntiles && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&k_full[st], ph, p.err, abort_flag, kErrTimeoutMma)) { ok = false; break; }
        if (!mbar_wait(&s_free[st], ph ^ 1, p.err, abort_flag, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + L::OFF_K + st * L::KV_BYTES);
        const uint32_t s_tmem = tmem + st * BN;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          const uint64_t ad = make_sw128_desc(q_addr + off, 16, 1024);
          const uint64_t bd = make_sw128_desc(k_addr + (kk >> 2) * (BN * 128) + (kk & 3) * 32, 16, 1024);
          tc_mma_f16(s_tmem, ad, bd, idesc_s, kk != 0);
        }
        tc_commit(&k_empty[st]);
        tc_commit(&s_full[st]);
        if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok) issue_pv(ntiles - 1);
    }
  } else {
    // ----------------------------------------------------------- softmax --
    const int r = warp * 32 + lane;  // query row within the tile == TMEM lane
    const int qi = q0 + r;
    const int limit = p.causal ? (S_kv - p.S_q + qi) : (S_kv - 1);
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    float m_run = -INFINITY;
    float l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int st = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      const bool from_a = j < p.tiles_a;
      const int p0 = from_a ? j * BN : p.n_a + (j - p.tiles_a) * BN;
      const int cnt = from_a ? min(BN, p.n_a - j * BN) : min(BN, p.n_b - (j - p.tiles_a) * BN);
      const int nvalid = max(0, min(cnt, limit - p0 + 1));
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[st], ph, p.err, abort_flag, kErrTimeoutSoftmax));
      if (!ok) break;
      tc_fence_after();
      uint32_t s[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c)
        tmem_ld32(lane_base + st * BN + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&s[c * 32]));
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&s_free[st]);

      // Row max over the valid keys (raw scores; scale > 0 so the max commutes).
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < BN; ++c) {
        const float v = c < nvalid ? __uint_as_float(s[c]) : -INFINITY;
        s[c] = __float_as_uint(v);
        mx4[c & 3] = fmaxf(mx4[c & 3], v);
      }
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * p.scale_log2;
      const float m_new = fmaxf(m_run, mx);
      const bool grow = m_new > m_run + kRescaleThreshold || (m_run == -INFINITY && m_new > -INFINITY);
      const float alpha = grow ? (m_run == -INFINITY ? 0.f : fast_exp2(m_run - m_new)) : 1.f;
      if (grow) m_run = m_new;
      const bool any_grow = __any_sync(0xffffffffu, grow) && j > 0;
      if (any_grow) {
        // O holds P_0..P_{j-1} V; wait for the last of them, then rescale.
        const int pj = j - 1;
        ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[pj & 1], (pj >> 1) & 1, p.err, abort_flag,
                                               kErrTimeoutSoftmax));
        if (!ok) break;
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(lane_base + 256 + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int k = 0; k < 32; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
          tmem_st32(lane_base + 256 + c * 32, o);
        }
        tmem_st_wait();
      }
      l_run *= alpha;
      // P buffer `st` is free once PV_{j-2} finished.
      if (j >= 2) {
        const int pj = j - 2;
        ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[pj & 1], (pj >> 1) & 1, p.err, abort_flag,
                                               kErrTimeoutSoftmax));
        if (!ok) break;
      }
      uint8_t* pbuf = smem + L::OFF_P + st * L::P_BYTES;
      // p = 2^(s * scale*log2e - m): one FFMA + one SFU op per score.
      const float neg_m = (m_run == -INFINITY) ? 0.f : -m_run;
      float ls4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c8 = 0; c8 < BN / 8; ++c8) {
        float e[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          e[k] = fast_exp2(fmaf(__uint_as_float(s[c8 * 8 + k]), p.scale_log2, neg_m));
          ls4[k & 3] += e[k];
        }
        uint4 pk;
        pk.x = pack_bf16x2(e[0], e[1]);
        pk.y = pack_bf16x2(e[2], e[3]);
        pk.z = pack_bf16x2(e[4], e[5]);
        pk.w = pack_bf16x2(e[6], e[7]);
        const int sub = c8 >> 3;          // which 64-key half
        const int chunk = c8 & 7;         // 16-byte chunk within the 128-byte row
        uint8_t* dst = pbuf + sub * (BM * 128) + r * 128 + ((chunk ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) = pk;
      }
      const float lsum = (ls4[0] + ls4[1]) + (ls4[2] + ls4[3]);
      l_run += lsum;
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[st]);
    }
    // ------------------------------------------------------- epilogue --
    __nv_bfloat16* orow = p.O + (static_cast<long long>(bh) * p.S_q + qi) * D;
    if (ntiles > 0 && ok) {
      const int pj = ntiles - 1;
      ok = mbar_wait(&pv_done[pj & 1], (pj >> 1) & 1, p.err, abort_flag, kErrTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        if (ntiles > 0) {
          tmem_ld32(lane_base + 256 + c * 32, o);
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

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
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
  if (!al(Q) || !al(O)) return false;
  if (kv.n_a > 0 && (!al(kv.Ka) || !al(kv.Va))) return false;
  if (kv.n_b > 0 && (!al(kv.Kb) || !al(kv.Vb))) return false;
  return true;
}

}  // namespace pkb200
