// attention_tc.cuh - causal prefill attention with fused KV-cache append on
// tcgen05 tensor cores (sm_100a), head_dim 64 or 128.
//
// Semantics follow the reference's kernels/generated/attention_prefill.cu:84-155
// and the golden tests/golden/golden.py:139-172: scores = (q . k) * scale in
// fp32, query row i (of S_q) sees key positions p <= S_kv - S_q + i when
// causal (attention_prefill.cu:103), softmax in fp32, P.V accumulated in fp32,
// one bf16 rounding of O. Rows that see no key produce 0 (attention_prefill.cu:154).
//
// One CTA per (128-query tile, batch*head); blocks run in groups of heads,
// longest tiles first within a group. Roles (448 threads):
//   warps 0-7  softmax. Warp w of group h (warps 4h..4h+3) handles key half h
//              (64 keys) of every key tile for the query rows of TMEM lane
//              quarter w%4; thread r owns query row r (= TMEM lane r). It
//              reads its S values with tcgen05.ld, agrees on the tile's max
//              with the thread holding the other half of the row (shared
//              memory + an mbarrier per lane quarter), keeps the running max
//              and its half of the row sum in the exp2 domain, and writes P
//              back over the same TMEM columns as an fp16 pair per probability
//              (P = P_hi + P_lo, ~21 significant bits, built with FMA/ALU
//              arithmetic so the SFU pipe only runs exp2), where the P.V MMAs
//              read it as their A operand. Per key tile group 0 hands the row's
//              rescale factor (2^(m_old - m_new)) to the correction warps.
//   warps 8-11 correction and V conversion. Each key tile's P.V lands in a
//              fresh TMEM accumulator Ot (16 MMA steps deep); thread r folds
//              it into the running O of row r with fp32 FMAs,
//              O = O * alpha + Ot, in TMEM. While the tensor core runs P.V(j)
//              these warps rewrite V(j+1) in place in shared memory from bf16
//              to fp16 (same layout, same swizzle) for the next P.V. Every
//              bf16 value in [2^-17, 65280] is exactly an fp16 value. A tile
//              that holds a value of magnitude >= 2^16 (or inf), or a warp's
//              share of a tile whose values are all below 2^-6 (where values
//              below 2^-17 would lose bits), marks the CTA; such a CTA
//              recomputes its query rows with the exact SIMT row routine after
//              the tensor-core pass, so the result never depends on fp16 range.
//              At the end they normalise O by the row sum and store it.
//   warp 12    TMA producer: the Q tile once; K tiles (128 keys) through a
//              2-deep ring and V tiles through a 3-deep ring, each load issued
//              as soon as its slot frees. For the append entry point, the CTA
//              whose query tile matches a tile of new rows also writes those
//              K/V tiles from shared memory into the cache with TMA stores, so
//              the append costs no extra HBM read.
//   warp 13    TMEM owner + MMA issuer (the whole warp runs the loop; one
//              elected lane issues). Per key tile j: S(j+1) into the other S
//              buffer (once P.V(j-1) has read it), then
//              P.V(j) = P_hi.V + P_lo.V into Ot (once pv_ready(j) says P(j),
//              fp16 V(j) and a drained Ot are in place). So the tensor core
//              computes S(j+1) while the softmax works on S(j), and P.V(j)
//              while the softmax works on S(j+1).
//
// Numerics: scores are fp32 (bf16 Q.K on tensor cores), P is fp32 from the
// SFU exp2 and enters P.V as fp16 hi+lo (relative error ~2^-21), V enters as
// exact fp16, each key tile's P.V accumulates in fp32 on the tensor core over
// only 128 keys, and the tiles are summed with round-to-nearest fp32 FMAs.
// Tensor-core accumulation truncates; summing a 2048-key row in one tensor-core
// accumulator would put its rounding well above the golden's fp32 sum, which
// the per-tile accumulator avoids. This is the golden's arithmetic (fp32 P,
// golden.py:139-172; attention_prefill.cu:127-147) to within fp32 summation
// order.
// TMEM (512 columns): S/P buffers [0,128) and [128,256), Ot [256,256+D),
// O [384,384+D). Within an S/P buffer, the P of keys [64h, 64h+64) sits in
// columns [64h, 64h+32) (hi) and [64h+32, 64h+64) (lo), one fp16 pair per
// column.
//
// Key positions come from two sources (KvSources): A (rows [0, n_a), the
// cache prefix or the whole K/V of the plain entry point) and B (the new
// rows, positions n_a + r). Key tiles never straddle the two: a source's last
// tile may be partial, and the keys past its end are masked.
#pragma once

#include "simt_kernels.cuh"

namespace pkb200 {
namespace attn {
constexpr int BM = 128;           // query rows per tile (one tile per CTA)
constexpr int BN = 128;           // keys per tile
constexpr int KST = 2;            // K pipeline stages
constexpr int VST = 3;            // V pipeline stages (TMA, then fp16 conversion)
constexpr int NUM_THREADS = 512;
constexpr int kConvThreads = 128;  // the correction warps 8-11 convert V
constexpr int kWarpProducer = 12, kWarpMma = 13;  // warps 14-15 idle
// Registers per thread by warpgroup (launch: 512 x 128): softmax warpgroups 0
// and 1 keep 128; the correction warpgroup holds its rows' O (D fp32) in
// registers; warpgroup 3 (producer, MMA issuer) needs few.
// 2 x 128 + kRegsCorrection + kRegsControl = 4 x 128.
constexpr int kRegsCorrection = 176;
constexpr int kRegsControl = 80;
static_assert(kRegsCorrection + kRegsControl == 2 * 128, "register split must fit the launch");
constexpr float kRescaleThreshold = 8.0f;  // log2 units
// Probabilities are formed as 2^7 * p: with the stale-max threshold p <= 2^8,
// so 2^7 * p <= 2^15 stays inside fp16's range while the values that would
// fall into fp16's subnormal range shrink by 2^7. The row sum carries the same
// factor, so O = sum(P.V) / sum(P) is unchanged.
constexpr float kPScaleLog2 = 7.0f;
constexpr uint32_t kColOt = 256;  // per-key-tile P.V accumulators Ot[j & 1]: 256, 384

template <int D>
struct Layout {
  static constexpr int DBOX = D / 64;                   // 64-column boxes per row
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;          // KST stages
  static constexpr int OFF_V = OFF_K + KST * KV_BYTES;   // VST stages
  static constexpr int OFF_ALPHA = OFF_V + VST * KV_BYTES;  // float[2][BM]
  static constexpr int OFF_L = OFF_ALPHA + 2 * BM * 4;     // float[2][BM] (per key half)
  static constexpr int OFF_HMAX = OFF_L + 2 * BM * 4;      // float[2][2][BM]
  static constexpr int OFF_BAR = OFF_HMAX + 4 * BM * 4;
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
  int head_group;  // heads per scheduling group (block order below)
  __nv_bfloat16* O;
  int* err;
  // exact fallback (rows of CTAs whose V tiles fp16 cannot carry exactly)
  const __nv_bfloat16* Q;
  KvSources kv;
  float scale;
  unsigned long long* exact_ctas;  // count of CTAs that took the fallback
};

// Key tile j of query tile qt is a tile of new rows that this CTA appends.
__device__ __forceinline__ bool attn_append_tile(const AttnTcParams& p, int j, int qt) {
  return p.append && j >= p.tiles_a && j - p.tiles_a == qt;
}

// Rewrites one 32-bit word (two bf16) as two fp16 and folds |v| into amax
// (one three-input max).
__device__ __forceinline__ uint32_t attn_bf16x2_to_f16x2(uint32_t w, float& amax) {
  const float f0 = __uint_as_float(w << 16), f1 = __uint_as_float(w & 0xffff0000u);
  amax = fmax3(amax, fabsf(f0), fabsf(f1));
  return pack_f16x2(f0, f1);
}

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
  float* alpha_s = reinterpret_cast<float*>(smem + L::OFF_ALPHA);
  float* l_s = reinterpret_cast<float*>(smem + L::OFF_L);
  float* hmax_s = reinterpret_cast<float*>(smem + L::OFF_HMAX);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;            // [KST]
  uint64_t* k_empty = k_full + KST;       // [KST]
  uint64_t* v_full = k_empty + KST;       // [VST] TMA landed (bf16)
  uint64_t* v_empty = v_full + VST;       // [VST]
  // pv_ready[j % VST]: everything P.V(j) reads is in place: P(j) written
  // over S(j) (softmax warps), V(j) converted to fp16 and Ot drained of
  // P.V(j-1) (correction warps). One barrier, so the MMA warp polls once.
  // No role can arrive for tile j+VST before tile j's phase completes: each
  // such arrival needs P.V(j+1) or later issued.
  uint64_t* pv_ready = v_empty + VST;     // [VST]
  uint64_t* s_full = pv_ready + VST;      // [2]  S(j) in S/P buffer j&1
  uint64_t* alpha_full = s_full + 2;      // [2]  rescale factors of tile j
  uint64_t* alpha_empty = alpha_full + 2; // [2]
  uint64_t* pv_done = alpha_empty + 2;    // [2]  P.V(j) in Ot[j&1]
  uint64_t* l_ready = pv_done + 2;        // row sums in l_s
  uint64_t* v_stored = l_ready + 1;       // appended V tile read out of smem
  uint64_t* pair_bar = v_stored + 1;      // [4] the two softmax warps of a lane quarter
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pair_bar + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* needs_exact = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = warp_id();
  const int lane = lane_id();
  // One-dimensional grid in groups of head_group heads; within a group the
  // longest query tiles come first across its heads, so the block scheduler
  // fills the SMs longest-job-first while the CTAs in flight share the K/V
  // of a few heads in L2.
  int bh, qt;
  {
    const int blk = static_cast<int>(blockIdx.x);
    const int per_group = p.head_group * p.num_qtiles;
    const int g = blk / per_group;
    const int gsize = min(p.head_group, p.BH - g * p.head_group);
    const int r = blk - g * per_group;
    bh = g * p.head_group + r % gsize;
    qt = p.num_qtiles - 1 - r / gsize;
  }
  const int nt = attn_tiles_for(p, qt);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < KST; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < VST; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&pv_ready[i], 2 * BM + BM);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&alpha_full[i], BM);
      mbar_init(&alpha_empty[i], BM);
    }
    mbar_init(&pv_done[0], 1);
    mbar_init(&pv_done[1], 1);
    mbar_init(l_ready, 2 * BM);
    mbar_init(v_stored, 1);
    for (int i = 0; i < 4; ++i) mbar_init(&pair_bar[i], 64);
    *abort_flag = 0;
    *needs_exact = 0;
    fence_barrier_init();
  }
  if (warp == kWarpMma) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= kWarpProducer) {
    setmaxnreg_dec<kRegsControl>();
    if (warp == kWarpProducer) {
      if (lane == 0 && nt > 0) {
        // -------------------------------------------------------- producer --
        tma_prefetch_desc(&map_q);
        mbar_arrive_expect_tx(q_full, L::Q_BYTES);
#pragma unroll
        for (int c = 0; c < L::DBOX; ++c)
          tma_load_3d(smem + L::OFF_Q + c * (BM * 128), &map_q, q_full, c * 64, qt * BM, bh);
        // K and V tiles are issued independently, each as soon as its ring
        // slot is released (a K slot frees when S(j) completes, a V slot when
        // P.V(j) does), so a K load never queues behind a V slot. V(j) is
        // issued only after K(j).
        int jk = 0, jv = 0;
        bool ok = true;
        long long t_idle = clock64();
        while (ok && jv < nt) {
          bool progressed = false;
          if (jk < nt && mbar_test_wait(&k_empty[jk % KST], ((jk / KST) & 1) ^ 1)) {
            const int row0 = jk < p.tiles_a ? jk * BN : (jk - p.tiles_a) * BN;
            uint8_t* sk = smem + L::OFF_K + (jk % KST) * L::KV_BYTES;
            mbar_arrive_expect_tx(&k_full[jk % KST], L::KV_BYTES);
#pragma unroll
            for (int c = 0; c < L::DBOX; ++c)
              tma_load_3d(sk + c * (BN * 128), jk < p.tiles_a ? &map_ka : &map_kb, &k_full[jk % KST],
                          c * 64, row0, bh);
            if (attn_append_tile(p, jk, qt)) {
              // Write this tile of new rows into the cache (rows n_a + row0 ...)
              // before the slot can be reused.
              if (!mbar_wait(&k_full[jk % KST], (jk / KST) & 1, p.err, abort_flag,
                             kErrTimeoutProducer))
                break;
#pragma unroll
              for (int c = 0; c < L::DBOX; ++c)
                tma_store_3d(&map_kc_store, sk + c * (BN * 128), c * 64, p.n_a + row0, bh);
              bulk_commit_group();
              bulk_wait_group_read0();
            }
            ++jk;
            progressed = true;
          }
          if (jv < jk && mbar_test_wait(&v_empty[jv % VST], ((jv / VST) & 1) ^ 1)) {
            const int j = jv;
            const int row0 = j < p.tiles_a ? j * BN : (j - p.tiles_a) * BN;
            const int vs = j % VST;
            uint8_t* sv = smem + L::OFF_V + vs * L::KV_BYTES;
            mbar_arrive_expect_tx(&v_full[vs], L::KV_BYTES);
#pragma unroll
            for (int c = 0; c < L::DBOX; ++c)
              tma_load_3d(sv + c * (BN * 128), j < p.tiles_a ? &map_va : &map_vb, &v_full[vs], c * 64,
                          row0, bh);
            if (attn_append_tile(p, j, qt)) {
              // The appended V tile goes to the cache before the correction
              // warps rewrite it as fp16 (they wait for v_stored).
              if (!mbar_wait(&v_full[vs], (j / VST) & 1, p.err, abort_flag, kErrTimeoutProducer)) break;
#pragma unroll
              for (int c = 0; c < L::DBOX; ++c)
                tma_store_3d(&map_vc_store, sv + c * (BN * 128), c * 64, p.n_a + row0, bh);
              bulk_commit_group();
              bulk_wait_group_read0();
              mbar_arrive(v_stored);
            }
            ++jv;
            progressed = true;
          }
          if (progressed) {
            t_idle = clock64();
          } else if (*abort_flag) {
            ok = false;
          } else if (clock64() - t_idle > kSpinLimitCycles) {
            atomicCAS(p.err, 0, kErrTimeoutProducer);
            *abort_flag = 1;
            ok = false;
          } else {
            // nothing to issue yet: sleep briefly instead of spinning, so the
            // softmax warps sharing this SM sub-partition keep its issue slots
            __nanosleep(64);
          }
        }
        bulk_wait_group0();
      }
    } else if (warp == kWarpMma) {
      if (nt > 0) {
        // ------------------------------------------------------ MMA issuer --
        // The whole warp runs this loop (warp-uniform values); one elected lane
        // issues each MMA and commit.
        constexpr uint32_t idesc_s = make_idesc_bf16(BM, BN, false, false);
        constexpr uint32_t idesc_o = make_idesc_f16(BM, D, false, true);
        const uint32_t q_addr = smem_u32(smem + L::OFF_Q);
        auto issue_s = [&](int j) {
          const uint32_t k_addr = smem_u32(smem + L::OFF_K + (j % KST) * L::KV_BYTES);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
            const uint64_t ad = make_sw128_desc(q_addr + off, 16, 1024);
            const uint64_t bd = make_sw128_desc(k_addr + off, 16, 1024);
            tc_mma_f16_warp(tmem + (j & 1) * BN, ad, bd, idesc_s, kk != 0);
          }
          tc_commit_warp(&k_empty[j % KST]);
          tc_commit_warp(&s_full[j & 1]);
        };
        auto issue_pv = [&](int j) {
          const uint32_t v_addr = smem_u32(smem + L::OFF_V + (j % VST) * L::KV_BYTES);
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const uint64_t bd = make_sw128_desc(v_addr + kk * 2048, BN * 128, 1024);
            const uint32_t a_hi = tmem + (j & 1) * BN + (kk >> 2) * 64 + (kk & 3) * 8;
            tc_mma_f16_tmem_a_warp(tmem + kColOt + (j & 1) * 128, a_hi, bd, idesc_o, kk != 0);
            tc_mma_f16_tmem_a_warp(tmem + kColOt + (j & 1) * 128, a_hi + 32, bd, idesc_o, 1);
          }
          tc_commit_warp(&v_empty[j % VST]);
          tc_commit_warp(&pv_done[j & 1]);
        };
        // every wait is taken by the whole warp, so the warp stays converged
        auto wait = [&](uint64_t* bar, uint32_t parity) {
          return __all_sync(0xffffffffu, mbar_wait(bar, parity, p.err, abort_flag, kErrTimeoutMma));
        };
        bool ok = wait(q_full, 0) && wait(&k_full[0], 0);
        if (ok) {
          tc_fence_after();
          issue_s(0);
        }
        for (int j = 0; j < nt && ok; ++j) {
          if (j + 1 < nt) {
            // S(j+1) goes into the buffer that held P(j-1): P.V(j-1) must be done.
            ok = wait(&k_full[(j + 1) % KST], ((j + 1) / KST) & 1) &&
                 (j < 1 || wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1));
            if (!ok) break;
            tc_fence_after();
            issue_s(j + 1);
          }
          ok = wait(&pv_ready[j % VST], (j / VST) & 1);
          if (!ok) break;
          tc_fence_after();
          issue_pv(j);
        }
      }
    }
  } else if (warp < 8) {
    // ----------------------------------------------------------- softmax --
    // Warp w of group h (warps 4h..4h+3) owns key half h of every tile for
    // TMEM lanes 32(w%4)..: thread r handles keys [64h, 64h+64) of query row r.
    // The two threads of a row agree on the tile's max through shared memory
    // (pair_bar: the two warps of a lane quarter), so both form P with the
    // same running max.
    const int hk = warp >> 2;                     // key half
    const int r = static_cast<int>(threadIdx.x) & (BM - 1);
    const int qi = qt * BM + r;
    const int S_kv = p.n_a + p.n_b;
    const int limit = p.causal ? (S_kv - p.S_q + qi) : (S_kv - 1);
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    uint64_t* pbar = &pair_bar[warp & 3];
    float m_run = -INFINITY;
    float l_run = 0.f;  // this thread's half of the row sum
    for (int j = 0; j < nt; ++j) {
      const int b = j & 1;
      const bool from_a = j < p.tiles_a;
      const int p0 = from_a ? j * BN : p.n_a + (j - p.tiles_a) * BN;
      const int cnt = from_a ? min(BN, p.n_a - j * BN) : min(BN, p.n_b - (j - p.tiles_a) * BN);
      const int nvalid = max(0, min(cnt, limit - p0 + 1)) - hk * 64;  // keys of this half
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[b], (j >> 1) & 1, p.err, abort_flag,
                                             kErrTimeoutSoftmax)))
        break;
      tc_fence_after();
      const uint32_t s_half = lane_base + b * BN + hk * 64;
      uint32_t sv[64];
      tmem_ld32(s_half, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
      tmem_ld32(s_half + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
      tmem_ld_wait();
      if (__any_sync(0xffffffffu, nvalid < 64)) {
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (c >= nvalid) sv[c] = __float_as_uint(-INFINITY);
      }
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int k = 0; k < 32; ++k)
        mx4[k & 3] = fmax3(mx4[k & 3], __uint_as_float(sv[2 * k]), __uint_as_float(sv[2 * k + 1]));
      const float mx_half = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * p.scale_log2;
      hmax_s[(b * 2 + hk) * BM + r] = mx_half;
      mbar_arrive(pbar);
      if (!__all_sync(0xffffffffu, mbar_wait(pbar, j & 1, p.err, abort_flag, kErrTimeoutSoftmax)))
        break;
      const float mx = fmaxf(mx_half, hmax_s[(b * 2 + (hk ^ 1)) * BM + r]);
      // The running max moves only when the tile's max exceeds it by more
      // than the rescale threshold (both threads of the row decide alike).
      const float m_prev = m_run;
      const float m_new = fmaxf(m_run, mx);
      if (m_new > m_run + kRescaleThreshold || (m_run == -INFINITY && m_new > -INFINITY)) {
        l_run *= (m_run == -INFINITY) ? 0.f : fast_exp2(m_run - m_new);
        m_run = m_new;
      }
      const float neg_m = (m_run == -INFINITY) ? 0.f : kPScaleLog2 - m_run;
      // pairs of columns on the packed fp32x2 pipe: one FMA and one add per pair
      const uint64_t sc2 = f2_pack(p.scale_log2, p.scale_log2);
      const uint64_t nm2 = f2_pack(neg_m, neg_m);
      uint64_t ls2[2] = {f2_pack(0.f, 0.f), f2_pack(0.f, 0.f)};
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        uint32_t phi[16], plo[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const int kk = q * 16 + k;
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(__uint_as_float(sv[2 * kk]), __uint_as_float(sv[2 * kk + 1])),
                           sc2, nm2),
                    x0, x1);
          const float e0 = fast_exp2(x0);
          const float e1 = fast_exp2(x1);
          ls2[k & 1] = f2_add(ls2[k & 1], f2_pack(e0, e1));
          split_f16x2(e0, e1, phi[k], plo[k]);
        }
        tmem_st16(s_half + q * 16, phi);
        tmem_st16(s_half + 32 + q * 16, plo);
      }
      {
        float a0, a1, b0, b1;
        f2_unpack(ls2[0], a0, a1);
        f2_unpack(ls2[1], b0, b1);
        l_run += (a0 + b0) + (a1 + b1);
      }
      if (hk == 0) {
        // hand the tile's O rescale factor to the correction warps
        const float tile_alpha =
            m_run == m_prev ? 1.f : (m_prev == -INFINITY ? 0.f : fast_exp2(m_prev - m_run));
        if (!__all_sync(0xffffffffu, mbar_wait(&alpha_empty[b], ((j >> 1) & 1) ^ 1, p.err,
                                               abort_flag, kErrTimeoutSoftmax)))
          break;
        alpha_s[b * BM + r] = tile_alpha;
        mbar_arrive(&alpha_full[b]);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&pv_ready[j % VST]);
    }
    l_s[hk * BM + r] = l_run;
    mbar_arrive(l_ready);
  } else {
    // -------------------------------------------------------- correction --
    setmaxnreg_inc<kRegsCorrection>();
    const int r = static_cast<int>(threadIdx.x) - 2 * BM;
    const int qi = qt * BM + r;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    // V(j) is rewritten from bf16 to fp16 in place in shared memory (same
    // layout, same swizzle) before P.V(j) reads it; every bf16 value in
    // [2^-17, 65280] is exactly an fp16 value. Per tile j these warps convert
    // V(j+1) and arrive on pv_ready(j+1) (V(j+1) in fp16, and Ot[(j+1)&1]
    // drained of P.V(j-1) in the previous step), then fold P.V(j) from
    // Ot[j&1] into the row's O, which lives in registers.
    const int ct = static_cast<int>(threadIdx.x) - 2 * BM;  // 0..127
    int appended = 0;
    auto convert_v = [&](int j) -> bool {
      const int st = j % VST;
      bool okc = __all_sync(0xffffffffu, mbar_wait(&v_full[st], (j / VST) & 1, p.err, abort_flag,
                                                   kErrTimeoutConvert));
      if (okc && attn_append_tile(p, j, qt)) {
        okc = __all_sync(0xffffffffu, mbar_wait(v_stored, appended & 1, p.err, abort_flag,
                                                kErrTimeoutConvert));
        ++appended;
      }
      if (!okc) return false;
      uint4* tile = reinterpret_cast<uint4*>(smem + L::OFF_V + st * L::KV_BYTES);
      float amax = 0.f;
#pragma unroll 4
      for (int i = ct; i < L::KV_BYTES / 16; i += kConvThreads) {
        uint4 w = tile[i];
        w.x = attn_bf16x2_to_f16x2(w.x, amax);
        w.y = attn_bf16x2_to_f16x2(w.y, amax);
        w.z = attn_bf16x2_to_f16x2(w.z, amax);
        w.w = attn_bf16x2_to_f16x2(w.w, amax);
        tile[i] = w;
      }
      fence_proxy_async_smem();
      // Range check per warp share of the tile: a value of magnitude >= 2^16
      // (inf included), or a share whose largest magnitude is below 2^-6,
      // where values below 2^-17 would lose bits in fp16. (A NaN in V
      // propagates to O as it does in fp32.)
      const float wmax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(amax)));
      if (lane == 0 && (!(wmax < 65536.f) || (wmax != 0.f && wmax < 0.015625f))) *needs_exact = 1;
      return true;
    };
    float o[D];
#pragma unroll
    for (int k = 0; k < D; ++k) o[k] = 0.f;
    // (a tile whose rows see no key has nt == 0 and still stores its zero rows)
    bool ok = nt == 0 || convert_v(0);
    if (ok && nt > 0) mbar_arrive(&pv_ready[0]);  // V(0) converted; Ot[0] holds nothing yet
    for (int j = 0; j < nt && ok; ++j) {
      const int b = j & 1;
      if (j + 1 < nt) {
        if (!convert_v(j + 1)) {
          ok = false;
          break;
        }
        mbar_arrive(&pv_ready[(j + 1) % VST]);
      }
      ok = __all_sync(0xffffffffu, mbar_wait(&alpha_full[b], (j >> 1) & 1, p.err, abort_flag,
                                             kErrTimeoutSoftmax));
      if (!ok) break;
      const float a = alpha_s[b * BM + r];
      mbar_arrive(&alpha_empty[b]);
      ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[b], (j >> 1) & 1, p.err, abort_flag,
                                             kErrTimeoutSoftmax));
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t t[32];
        tmem_ld32(lane_base + kColOt + b * 128 + c * 32, t);
        tmem_ld_wait();
#pragma unroll
        for (int k = 0; k < 32; ++k) o[c * 32 + k] = fmaf(o[c * 32 + k], a, __uint_as_float(t[k]));
      }
      // Ot[b] is read out: P.V(j+2) may overwrite it once pv_ready(j+2) says so
      tc_fence_before();
    }
    // ------------------------------------------------------- epilogue --
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(l_ready, 0, p.err, abort_flag,
                                                   kErrTimeoutSoftmax));
    if (ok && qi < p.S_q) {
      const float l = l_s[r] + l_s[BM + r];
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = p.O + (static_cast<long long>(bh) * p.S_q + qi) * D;
#pragma unroll
      for (int g = 0; g < D / 8; ++g) {
        uint4 v;
        v.x = pack_bf16x2(o[g * 8 + 0] * inv, o[g * 8 + 1] * inv);
        v.y = pack_bf16x2(o[g * 8 + 2] * inv, o[g * 8 + 3] * inv);
        v.z = pack_bf16x2(o[g * 8 + 4] * inv, o[g * 8 + 5] * inv);
        v.w = pack_bf16x2(o[g * 8 + 6] * inv, o[g * 8 + 7] * inv);
        *reinterpret_cast<uint4*>(orow + g * 8) = v;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  // Back to 128 registers everywhere for the common tail. Warpgroup 3 takes
  // its registers back only after warpgroup 2 has returned them: were it to
  // run ahead, it could take registers warpgroup 2's first increase waits for.
  if (warp >= 8 && warp < 12) setmaxnreg_dec<128>();
  __syncthreads();
  if (warp >= kWarpProducer) setmaxnreg_inc<128>();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  // Exact fallback: a V tile fp16 cannot carry exactly was seen, so every row
  // of this CTA is recomputed from global memory with fp32 arithmetic (the
  // appended cache rows were already written by the TMA stores above and are
  // not touched).
  if (*needs_exact && !*abort_flag) {
    if (threadIdx.x == 0) atomicAdd(p.exact_ctas, 1ull);
    for (int rr = warp; rr < BM; rr += NUM_THREADS / 32) {
      const int i = qt * BM + rr;
      if (i < p.S_q) attention_row_exact(p.Q, p.O, p.kv, p.S_q, D, p.scale, p.causal, bh, i, lane);
    }
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
