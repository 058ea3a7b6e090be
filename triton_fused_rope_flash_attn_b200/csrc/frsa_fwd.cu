// Forward kernel: O = softmax(R(Q) R(K)^T * scale) V with 2D RoPE fused.
//
// Restates the computation of _attn_fwd (fa_rope_full .py:91-315) as a
// persistent, warp-specialised tcgen05 kernel. A unit is a pair of 128-query
// tiles of one (batch*head) (the whole head when N <= 256); each CTA walks
// its units (see fwd_grid for the order) and, per unit, the keys in 128-key
// tiles with an online softmax in base 2. The two query tiles share every
// K/V load and K rotation, and the K/V stream runs on across units: the next
// unit's query tiles load and rotate while this unit's last tile is in its
// softmax and epilogue.
//
//   warp 0      TMA producer: each unit's query tiles, then K and V tiles into
//               rings of KS stages (K and V released separately: K once the
//               score products have read it, V once the P V products have)
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..3  no role (they complete warpgroup 0 for the register split)
//   warps 12..15  rotation warps: apply RoPE in shared memory to the Q
//               tiles and to every K tile as soon as TMA has landed it
//   warps 4..11 two compute warpgroups, warpgroup g owns query tile g of the
//               pair: it reads S from TMEM (thread = query row), writes P as
//               packed 16-bit pairs back over the scores it has read, and
//               writes O and the log-sum-exp. O accumulates in TMEM; the
//               softmax base is raised (and O rescaled in TMEM) only when a
//               tile's maximum exceeds it by more than 2^8. P V reads P from
//               TMEM (A operand) and V from shared memory, so P never touches
//               shared memory. The MMA issue order (P_0 V, S_0 next, P_1 V,
//               S_1 next) lets one group's products run while the other
//               group is in its softmax.
//
// TMEM columns: warpgroup g uses [256 g, 256 g + 128) for S (P packed in
// the first 64) and [256 g + 128, 256 g + 128 + DP) for O.
#include "frsa_internal.h"
#include "frsa_ptx.cuh"
#include "frsa_rope.cuh"

#undef FRSA_STAMP_TID
#define FRSA_STAMP_TID 128  // first compute thread of this kernel

namespace frsa {

namespace {

constexpr int kFwdCompute = 256;                // two warpgroups
constexpr int kFwdThreads = 128 + kFwdCompute + 128;  // + producer/MMA warpgroup, rotation warpgroup
// Registers per thread after the per-warpgroup split (launch: 128 each, 512
// threads; 96 + 96 + 2 x 160 = 4 x 128).
constexpr uint32_t kFwdRegsCtl = 96, kFwdRegsRot = 96, kFwdRegsCompute = 160;
constexpr uint32_t kTmemColsFwd = 512;
constexpr float kFwdSlack = 8.f;
constexpr int kFwdMaxWaves = 12;   // chunk-size levels of the guided schedule   // log2 headroom of the softmax base

template <int NCH>
struct FwdSmem {
  // K and V ring stages: the P tiles live in TMEM, so shared memory holds
  // only the two query tiles and the K/V ring.
  static constexpr int KS = (NCH == 1) ? 4 : 2;
  uint8_t q[2][NCH][kChunkBytes];      // query tile of warpgroup g
  uint8_t k[KS][NCH][kChunkBytes];     // key ring
  uint8_t v[KS][NCH][kChunkBytes];     // value ring
  uint64_t q_full[2], q_ready[2], q_empty[2];
  uint64_t k_full[KS], k_ready[KS], k_empty[KS];
  uint64_t v_full[KS], v_empty[KS];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_full[2];                  // the last P V of a unit has completed
  uint32_t tmem_base;
  int abort_flag;
};

struct FwdParams {
  const float* cosp;
  const float* sinp;
  void* o;
  float* lse;
  int H, N, D, nqt, npair, nkv, has_cls;
  int nunits;  // BH * npair
  float c2;    // scale * log2(e)
  // Guided schedule (fwd_schedule): wave w holds CTAs [wcta[w], wcta[w+1])
  // and gives each a run of wchunk[w] consecutive units starting at wunit[w].
  int nwaves;
  int wcta[kFwdMaxWaves + 1];
  int wunit[kFwdMaxWaves];
  int wchunk[kFwdMaxWaves];
};

// Units [begin, end) of this CTA.
__device__ __forceinline__ void fwd_range(const FwdParams& prm, int& begin, int& end) {
  const int b = static_cast<int>(blockIdx.x);
  int w = 0;
  while (w + 1 < prm.nwaves && b >= prm.wcta[w + 1]) ++w;
  begin = prm.wunit[w] + (b - prm.wcta[w]) * prm.wchunk[w];
  end = min(begin + prm.wchunk[w], prm.nunits);
}

// Unit u -> (head bh, pair pr, active query tiles of the pair: 1 or 2).
struct FwdUnit {
  int bh, pr, nact;
};
__device__ __forceinline__ FwdUnit fwd_unit(const FwdParams& prm, int u) {
  FwdUnit x;
  x.bh = u / prm.npair;
  x.pr = u - x.bh * prm.npair;
  x.nact = min(2, prm.nqt - 2 * x.pr);
  return x;
}

template <typename T, int NCH>
__global__ void __launch_bounds__(kFwdThreads, 1)
    fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
               const __grid_constant__ CUtensorMap tm_v, const FwdParams prm) {
  using Sm = FwdSmem<NCH>;
  constexpr int KS = Sm::KS;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Sm* smp = aligned_smem<Sm>(smem_raw);
  if (smp == nullptr) return;
  Sm& sm = *smp;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int N = prm.N, D = prm.D;
  const int nkv = prm.nkv;
  const int DP = (D + 15) & ~15;   // MMA N for P V
  const int ksteps = DP >> 4;      // MMA K steps over the head dim
  // D <= 64 and at least two key tiles: O alternates between two 64-column
  // TMEM buffers per unit, and a unit's O epilogue is deferred into the next
  // unit (after that unit's first P is published, while its second scores
  // are computed), so the softmax warps neither wait for the unit's last P V
  // nor stall the next unit on the O read-out.
  const bool two_o = NCH == 1 && nkv >= 2;
  volatile int* abort_flag = &sm.abort_flag;
  int ubeg, uend;
  fwd_range(prm, ubeg, uend);

  if (threadIdx.x == 0) {
    sm.abort_flag = 0;
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.q_full[s], 1);
      mbar_init(&sm.q_ready[s], 1);
      mbar_init(&sm.q_empty[s], 1);
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.p_full[s], 1);
      mbar_init(&sm.o_full[s], 1);
    }
    for (int s = 0; s < KS; ++s) {
      mbar_init(&sm.k_full[s], 1);
      mbar_init(&sm.k_ready[s], 1);
      mbar_init(&sm.k_empty[s], 1);
      mbar_init(&sm.v_full[s], 1);
      mbar_init(&sm.v_empty[s], 1);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, kTmemColsFwd);
    tmem_relinquish();
  }
  FRSA_STAMP(31);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  // Barrier phases. Query-tile buffer g is filled once per unit in which
  // query tile g of the pair exists (fill f: parity f & 1); the K/V tiles
  // form one running sequence t over the CTA's units (stage t % KS, parity
  // (t / KS) & 1); warpgroup g's S and P barriers count the key tiles it has
  // processed, its O barrier the units.
  if (warp < 4) {
  setmaxnreg_dec<kFwdRegsCtl>();
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      int qf[2] = {0, 0};
      int t = 0;
      for (int u = ubeg; u < uend; ++u) {
        const FwdUnit x = fwd_unit(prm, u);
        for (int g = 0; g < x.nact; ++g) {
          mbar_wait(&sm.q_empty[g], (qf[g] & 1) ^ 1, abort_flag);
          mbar_arrive_expect_tx(&sm.q_full[g], NCH * kChunkBytes);
          for (int c = 0; c < NCH; ++c)
            tma_load_bh(sm.q[g][c], &tm_q, &sm.q_full[g], c * kChunkCols, (2 * x.pr + g) * kTile,
                        x.bh, prm.H);
          ++qf[g];
        }
        for (int j = 0; j < nkv; ++j, ++t) {
          const int s = t % KS;
          const uint32_t ph = ((t / KS) & 1) ^ 1;
          mbar_wait(&sm.k_empty[s], ph, abort_flag);
          mbar_arrive_expect_tx(&sm.k_full[s], NCH * kChunkBytes);
          for (int c = 0; c < NCH; ++c)
            tma_load_bh(sm.k[s][c], &tm_k, &sm.k_full[s], c * kChunkCols, j * kTile, x.bh, prm.H);
          mbar_wait(&sm.v_empty[s], ph, abort_flag);
          mbar_arrive_expect_tx(&sm.v_full[s], NCH * kChunkBytes);
          for (int c = 0; c < NCH; ++c)
            tma_load_bh(sm.v[s][c], &tm_v, &sm.v_full[s], c * kChunkCols, j * kTile, x.bh, prm.H);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && ubeg < uend) {
      constexpr bool kBf = Elt<T>::kBf16;
      const uint32_t idS = idesc_f16(kBf, 128, 128, false, false);
      const uint32_t idO = idesc_f16(kBf, 128, DP, false, true);
      // S_g = Q^_g K^T : A = Q^ [q][d] K-major, B = K^ [kv][d] K-major.
      auto issue_s = [&](int g, int s) {
        const uint32_t tS = tmem + 256 * g;
        for (int ks = 0; ks < ksteps; ++ks) {
          const int c = ks >> 2;
          const uint32_t koff = (ks & 3) * 32;
          mma_ss(tS, sw128_desc(smem_u32(sm.q[g][c]) + koff, 16, 1024),
                 sw128_desc(smem_u32(sm.k[s][c]) + koff, 16, 1024), idS, ks > 0);
        }
        mma_commit(&sm.s_full[g]);
      };
      // O_g (+)= P_g V : A = P [q][kv] from TMEM (packed 16-bit pairs over
      // the scores: keys [16 ks, 16 ks + 16) in columns [8 ks, 8 ks + 8)),
      // B = V [kv][d] MN-major. O accumulates over a unit's key tiles.
      auto issue_pv = [&](int g, int s, bool acc, uint32_t ocol) {
        const uint32_t tS = tmem + 256 * g;
        const uint32_t tO = tS + ocol;
        for (int ks = 0; ks < kTile / 16; ++ks)
          mma_ts(tO, tS + 8 * ks, sw128_desc(smem_u32(sm.v[s][0]) + ks * 2048, kChunkBytes, 1024),
                 idO, acc || ks > 0);
      };
      int qf[2] = {0, 0};   // query-tile fill of the current unit, per warpgroup
      int tg[2] = {0, 0};   // key tiles processed, per warpgroup
      int ug[2] = {0, 0};   // units finished, per warpgroup (selects the O buffer)
      int t = 0;            // running K/V tile
      int u = ubeg;
      FwdUnit x = fwd_unit(prm, u);
      // Prologue: the first unit's scores against its first key tile.
      mbar_wait(&sm.k_ready[0], 0, abort_flag);
      for (int g = 0; g < x.nact; ++g) {
        mbar_wait(&sm.q_ready[g], 0, abort_flag);
        tc_fence_after();
        issue_s(g, 0);
        if (nkv == 1) mma_commit(&sm.q_empty[g]);
      }
      mma_commit(&sm.k_empty[0]);
      for (;;) {
        const int un = u + 1;
        const bool has_next = un < uend;
        const FwdUnit xn = fwd_unit(prm, has_next ? un : u);
        for (int j = 0; j < nkv; ++j, ++t) {
          const int s = t % KS;
          const bool more = j + 1 < nkv;
          const int t1 = t + 1, s1 = t1 % KS;
          bool k_waited = false, v_waited = false;
          bool any_s = false;
          auto wait_k = [&]() {
            if (!k_waited) {
              mbar_wait(&sm.k_ready[s1], (t1 / KS) & 1, abort_flag);
              k_waited = true;
            }
          };
          // Per group: P_g V of this key tile, then (P overwritten only
          // after the P V that reads it, by this thread's in-order issue)
          // S_g of the next key tile. The two groups alternate, so the
          // tensor core works on one group's products while the other group
          // is in its softmax.
          for (int g = 0; g < x.nact; ++g) {
            mbar_wait(&sm.p_full[g], tg[g] & 1, abort_flag);
            if (!v_waited) {
              mbar_wait(&sm.v_full[s], (t / KS) & 1, abort_flag);
              v_waited = true;
            }
            tc_fence_after();
            issue_pv(g, s, j > 0, 128 + (two_o ? 64 * (ug[g] & 1) : 0));
            ++tg[g];
            if (!more) {
              mma_commit(&sm.o_full[g]);
              ++ug[g];
            } else {
              wait_k();
              tc_fence_after();
              issue_s(g, s1);
              // The last score product of a query tile frees its buffer.
              if (j + 2 == nkv) mma_commit(&sm.q_empty[g]);
              any_s = true;
            }
          }
          if (!more && has_next) {
            // The next unit's first scores (its query tiles have landed and
            // rotated meanwhile).
            for (int g = 0; g < xn.nact; ++g) {
              wait_k();
              mbar_wait(&sm.q_ready[g], (qf[g] + (g < x.nact ? 1 : 0)) & 1, abort_flag);
              tc_fence_after();
              issue_s(g, s1);
              if (nkv == 1) mma_commit(&sm.q_empty[g]);
              any_s = true;
            }
          }
          if (any_s) mma_commit(&sm.k_empty[s1]);
          mma_commit(&sm.v_empty[s]);
        }
        for (int g = 0; g < x.nact; ++g) ++qf[g];
        if (!has_next) break;
        u = un;
        x = xn;
      }
    }
  }   // warps 2 and 3 have no role
  } else if (warp >= 12) {
    setmaxnreg_dec<kFwdRegsRot>();
    // ------------------------------------------------------------ rotation warps
    // Warps 12..15; each rotates a quarter of every tile, 16 rows (8
    // when D > 64) at a time with the table values loaded before the tile's
    // TMA wait.
    constexpr int kRows = 16 / NCH;
    const int rwp = warp - 12;
    auto rotate_tile = [&](uint8_t* tile, int tok0, uint64_t* full, uint32_t parity) {
#pragma unroll 1
      for (int blk = 0; blk < 32 / kRows; ++blk) {
        const int r0 = rwp * 32 + blk * kRows;
        RopeQ<NCH, kRows> rope;
        load_rope_q<NCH, kRows>(rope, r0, tok0, N, prm.has_cls, D, prm.cosp, prm.sinp, lane);
        if (blk == 0) mbar_wait(full, parity, abort_flag);
        if (prm.has_cls >= 0) apply_rope_q<T, NCH, kRows>(tile, r0, D, rope, lane);
      }
    };
    int qf[2] = {0, 0};
    int t = 0;
    for (int u = ubeg; u < uend; ++u) {
      const FwdUnit x = fwd_unit(prm, u);
      for (int g = 0; g < x.nact; ++g) {
        rotate_tile(&sm.q[g][0][0], (2 * x.pr + g) * kTile, &sm.q_full[g], qf[g] & 1);
        ++qf[g];
        fence_proxy_async_smem();
        named_bar(1, 128);
        if (threadIdx.x == 384) mbar_arrive(&sm.q_ready[g]);
      }
      for (int j = 0; j < nkv; ++j, ++t) {
        const int s = t % KS;
        rotate_tile(&sm.k[s][0][0], j * kTile, &sm.k_full[s], (t / KS) & 1);
        fence_proxy_async_smem();
        named_bar(1, 128);
        if (threadIdx.x == 384) mbar_arrive(&sm.k_ready[s]);
      }
    }
  } else {
    setmaxnreg_inc<kFwdRegsCompute>();
    // ------------------------------------------------------------ compute warpgroups
    const int cw = warp - 4;
    const int g = cw >> 2;                 // warpgroup = query tile of the pair
    const int wq = warp & 3;               // TMEM lane quarter
    const int r = wq * 32 + lane;          // query row in the tile == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const bool leader = threadIdx.x == 128 + 128 * g;
    const float c2 = prm.c2;
    const uint32_t tS = tmem + 256 * g + lane_off;
    const uint32_t tO = tmem + 256 * g + 128 + lane_off;
    int tg0 = 0;   // key tiles this warpgroup processed in earlier units
    int uo = 0;    // unit epilogues this warpgroup has waited for (o_full phase)
    int uc = 0;    // units this warpgroup has started (O buffer with two_o)
    // O / l of a finished unit, read from O buffer `tob` once its last P V
    // has completed, stored from registers (thread = query row; tcgen05.ld
    // is warp-collective, so the loads run in every lane of an active warp
    // and the stores only for rows that hold tokens).
    auto o_epilogue = [&](int bh_, int qrow_, float l_, bool active_, uint32_t tob) {
      mbar_wait(&sm.o_full[g], uo & 1, abort_flag);
      tc_fence_after();
      ++uo;
      if (active_) {
        const float inv_l = 1.f / l_;
        uint4* orow = reinterpret_cast<uint4*>(reinterpret_cast<T*>(prm.o) +
                                               (static_cast<size_t>(bh_) * N + qrow_) * D);
#pragma unroll 1
        for (int c16 = 0; c16 < 8; ++c16) {
          if (c16 * 16 < DP) {
            float v[16];
            tmem_ld16(tob + c16 * 16, v);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] *= inv_l;
            uint4 w0, w1;
            w0.x = Elt<T>::pack(v[0], v[1]);
            w0.y = Elt<T>::pack(v[2], v[3]);
            w0.z = Elt<T>::pack(v[4], v[5]);
            w0.w = Elt<T>::pack(v[6], v[7]);
            w1.x = Elt<T>::pack(v[8], v[9]);
            w1.y = Elt<T>::pack(v[10], v[11]);
            w1.z = Elt<T>::pack(v[12], v[13]);
            w1.w = Elt<T>::pack(v[14], v[15]);
            if (qrow_ < N) {
              orow[2 * c16] = w0;
              if (c16 * 16 + 8 < D) orow[2 * c16 + 1] = w1;
            }
          }
        }
      }
      // The O columns have been read: the P V that next overwrites them
      // follows this group's next p_full arrival.
      tc_fence_before();
    };
    // The deferred epilogue (two_o): unit, row, l, activity and O buffer.
    bool pend = false;
    int pend_bh = 0, pend_row = 0;
    float pend_l = 0.f;
    bool pend_active = false;
    uint32_t pend_tob = 0;
#ifdef FRSA_TRACE
    int tr_i = 0;
#define FWD_TR(ev, jj)                                                                   \
  do {                                                                                   \
    if (leader && blockIdx.x < 2048 && tr_i < 512) {                                     \
      g_trace_it[blockIdx.x * 1024 + g * 512 + tr_i] = globaltimer();                    \
      g_trace_fl[blockIdx.x * 1024 + g * 512 + tr_i] = (ev) | ((jj) << 8) | (x.nact << 16); \
      ++tr_i;                                                                            \
    }                                                                                    \
  } while (0)
#else
#define FWD_TR(ev, jj) \
  do {                 \
  } while (0)
#endif

#pragma unroll 1
    for (int u = ubeg; u < uend; ++u) {
      const FwdUnit x = fwd_unit(prm, u);
      if (g >= x.nact) continue;
      const int bh = x.bh;
      const int q0 = (2 * x.pr + g) * kTile;
      const int qrow = q0 + r;
      const uint32_t tOc = tO + (two_o ? 64u * static_cast<uint32_t>(uc & 1) : 0u);   // this unit's O
      ++uc;
      float m2 = -INFINITY, l = 0.f;
      // A warp whose 32 query rows are all padding skips the softmax math: its
      // P rows only ever reach O rows that are not stored.
      const bool warp_active = (q0 + wq * 32) < N;

      for (int j = 0; j < nkv; ++j) {
        const int tg = tg0 + j;
        const int nvalid = min(kTile, N - j * kTile);
        FWD_TR(0, j);
        // S of tile tg has landed; its commit also orders the P V of tile
        // tg - 1 (issued before it), so P and O are free to touch.
        mbar_wait(&sm.s_full[g], tg & 1, abort_flag);
        tc_fence_after();
        FWD_TR(1, j);
        if (warp_active) {
          // One pass over the scores, 64 columns at a time: the half's row
          // maximum, then P = exp2(S c2 - m2) and the row sum; 16-bit P is
          // packed in pairs into TMEM columns [32 h, 32 h + 32) for the keys
          // [64 h, 64 h + 64) (columns this thread has already read: the
          // write front trails the read front). The exponent base m2 is
          // raised only when a half's maximum exceeds it by more than
          // kFwdSlack (log2 units; P stays <= 2^kFwdSlack): then l, the
          // partial sums, the O accumulated in TMEM so far (the previous
          // tile's P V has completed: the commit of this tile's S follows
          // it) and, for the second half, the first half's P are rescaled.
          float sp[4] = {0.f, 0.f, 0.f, 0.f};
          // (not unrolled: one copy of the body, with its rarely taken
          // rescale code, keeps the loop small in the instruction cache)
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            if (h * 64 >= nvalid) {   // only padding keys: P = 0
              uint32_t z[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) z[i] = 0u;
              tmem_st16(tS + h * 32, z);
              tmem_st16(tS + h * 32 + 16, z);
              continue;
            }
            float sv[2][32];
            tmem_ld32(tS + h * 64, sv[0]);
            tmem_ld32(tS + h * 64 + 32, sv[1]);
            tmem_wait_ld();
            if (h * 64 + 64 > nvalid) {
#pragma unroll
              for (int uu = 0; uu < 2; ++uu)
#pragma unroll
                for (int i = 0; i < 32; ++i)
                  if (h * 64 + uu * 32 + i >= nvalid) sv[uu][i] = -INFINITY;
            }
            float mxp[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) mxp[i] = fmaxf(sv[0][i], sv[0][i + 8]);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              mxp[i] = fmaxf(fmaxf(mxp[i], sv[0][i + 16]), sv[0][i + 24]);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              mxp[i] = fmaxf(fmaxf(mxp[i], sv[1][i]), fmaxf(sv[1][i + 8], sv[1][i + 16]));
#pragma unroll
            for (int i = 0; i < 8; ++i) mxp[i] = fmaxf(mxp[i], sv[1][i + 24]);
            const float hm = fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                                   fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])));
            const bool up = hm * c2 > m2 + kFwdSlack;
            if (__any_sync(0xffffffffu, up)) {
              const float m_new = up ? hm * c2 : m2;
              const float alpha = ex2(m2 - m_new);   // 0 while m2 is -inf
              l *= alpha;
#pragma unroll
              for (int i = 0; i < 4; ++i) sp[i] *= alpha;
              if (j > 0) {
#pragma unroll 1
                for (int c16 = 0; c16 < 4 * NCH; ++c16) {
                  if (c16 * 16 < DP) {
                    float ov[16];
                    tmem_ld16(tOc + c16 * 16, ov);
                    tmem_wait_ld();
                    uint32_t w[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) w[i] = __float_as_uint(ov[i] * alpha);
                    tmem_st16(tOc + c16 * 16, w);
                  }
                }
              }
              if (h == 1) {
                tmem_wait_st();
#pragma unroll 1
                for (int c16 = 0; c16 < 2; ++c16) {
                  float pw[16];
                  tmem_ld16(tS + c16 * 16, pw);
                  tmem_wait_ld();
                  uint32_t w[16];
#pragma unroll
                  for (int i = 0; i < 16; ++i) {
                    const float2 pp = Elt<T>::unpack(__float_as_uint(pw[i]));
                    w[i] = Elt<T>::pack(pp.x * alpha, pp.y * alpha);
                  }
                  tmem_st16(tS + c16 * 16, w);
                }
              }
              m2 = m_new;
            }
#pragma unroll
            for (int uu = 0; uu < 2; ++uu) {
              uint32_t pk[16];
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                sv[uu][i] = ex2(fmaf(sv[uu][i], c2, -m2));
                sp[i & 3] += sv[uu][i];
              }
#pragma unroll
              for (int i = 0; i < 16; ++i) pk[i] = Elt<T>::pack(sv[uu][2 * i], sv[uu][2 * i + 1]);
              tmem_st16(tS + h * 32 + uu * 16, pk);
            }
          }
          l += (sp[0] + sp[1]) + (sp[2] + sp[3]);
          tmem_wait_st();
        }
        tc_fence_before();
        named_bar(2 + g, 128);
        if (leader) mbar_arrive(&sm.p_full[g]);
        FWD_TR(2, j);
        if (pend && j == 0) {   // the previous unit's O, while this unit's next scores run
          o_epilogue(pend_bh, pend_row, pend_l, pend_active, pend_tob);
          pend = false;
        }
      }

      // epilogue: lse = (m + log2 l) ln 2 now; O / l once the unit's last P V
      // has completed (deferred into the next unit with two_o).
      if (qrow < N)
        prm.lse[static_cast<size_t>(bh) * N + qrow] = (m2 + lg2(l)) * 0.69314718055994531f;
      tg0 += nkv;
      if (two_o) {
        pend = true;
        pend_bh = bh;
        pend_row = qrow;
        pend_l = l;
        pend_active = warp_active;
        pend_tob = tOc;
      } else {
        o_epilogue(bh, qrow, l, warp_active, tOc);
      }
      FWD_TR(4, 0);
    }
    if (pend) o_epilogue(pend_bh, pend_row, pend_l, pend_active, pend_tob);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemColsFwd);
  }
}

// Guided schedule: one CTA per SM at a time (the shared-memory footprint
// allows no second one), each CTA working a run of consecutive units so that
// one unit's softmax tail and epilogue overlap the next unit's loads and
// first scores. SMs do not run at the same speed (CTAs with identical work
// finish up to 30 % apart on a B200), so the runs shrink from wave to wave:
// wave w gives each of nsm CTAs about a 1/(2 nsm) share of the units still
// left, and the last units go one per CTA. The hardware dispatches CTAs in
// index order as SMs free up, which balances the tail dynamically without
// any counter in global memory. Returns the grid size.
int fwd_schedule(FwdParams& p, int nsm) {
  const int nunits = p.nunits;
  int rem = nunits, unit = 0, cta = 0, w = 0;
  while (rem > 0 && w < kFwdMaxWaves - 1) {
    const int c = rem / (2 * nsm);
    if (c < 2) break;
    p.wcta[w] = cta;
    p.wunit[w] = unit;
    p.wchunk[w] = c;
    cta += nsm;
    unit += nsm * c;
    rem -= nsm * c;
    ++w;
  }
  if (rem > 0) {   // (runs longer than 1 only for inputs beyond the wave limit)
    const int c = rem / (8 * nsm) > 1 ? rem / (8 * nsm) : 1;
    p.wcta[w] = cta;
    p.wunit[w] = unit;
    p.wchunk[w] = c;
    cta += (rem + c - 1) / c;
    ++w;
  }
  p.nwaves = w;
  p.wcta[w] = cta;
  return cta;
}

template <typename T, int NCH>
cudaError_t launch_fwd_t(const LaunchShape& s, const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                         const CUtensorMap& tm_v, const float* cosp, const float* sinp, void* o,
                         float* lse, cudaStream_t stream) {
  FwdParams p;
  p.cosp = cosp;
  p.sinp = sinp;
  p.o = o;
  p.lse = lse;
  p.H = s.H;
  p.N = s.N;
  p.D = s.D;
  p.nqt = (s.N + kTile - 1) / kTile;
  p.npair = (p.nqt + 1) / 2;
  p.nkv = p.nqt;
  p.has_cls = s.has_cls;
  p.c2 = s.scale * 1.4426950408889634f;
  const long long units = static_cast<long long>(s.BH) * p.npair;
  if (units > 0x7fffffffLL) return cudaErrorInvalidValue;
  p.nunits = static_cast<int>(units);
  const size_t smem = sizeof(FwdSmem<NCH>) + 1024;
  auto kern = fwd_kernel<T, NCH>;
  cudaError_t e = set_max_dynamic_smem_once(kern, smem);
  if (e != cudaSuccess) return e;
  if (p.nunits == 0) return cudaSuccess;
  const int grid = fwd_schedule(p, device_sm_count());
  kern<<<grid, kFwdThreads, smem, stream>>>(tm_q, tm_k, tm_v, p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_fwd(const LaunchShape& s, const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                       const CUtensorMap& tm_v, const CUtensorMap& tm_o, const float* cosp,
                       const float* sinp, void* o, float* lse, cudaStream_t stream) {
  if (fwd_small_applies(s)) return launch_fwd_small(s, tm_q, tm_k, tm_v, cosp, sinp, o, lse, stream);
  const bool two = s.D > 64;
  if (s.bf16) {
    return two ? launch_fwd_t<__nv_bfloat16, 2>(s, tm_q, tm_k, tm_v, cosp, sinp, o, lse, stream)
               : launch_fwd_t<__nv_bfloat16, 1>(s, tm_q, tm_k, tm_v, cosp, sinp, o, lse, stream);
  }
  return two ? launch_fwd_t<__half, 2>(s, tm_q, tm_k, tm_v, cosp, sinp, o, lse, stream)
             : launch_fwd_t<__half, 1>(s, tm_q, tm_k, tm_v, cosp, sinp, o, lse, stream);
}

}  // namespace frsa
