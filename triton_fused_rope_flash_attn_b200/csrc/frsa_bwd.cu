// Backward kernels: dQ, dK, dV of softmax(R(Q) R(K)^T * scale) V.
//
// Restates _attn_bwd_preprocess, _attn_bwd_dk_dv_rope and _attn_bwd_dq_rope
// (fa_rope_full .py:325-357, 374-691, 708-1009) as:
//
//   bwd_kernel    key-major tcgen05 kernel. When a query tile arrives the row
//                 warpgroup first forms Delta = rowsum(dO * O) in f32 from the
//                 dO tile in shared memory and the O row in global memory
//                 (fa_rope_full .py:352-357), so no separate preprocess launch. A CTA owns 128-key tiles of one
//                 (batch*head) and loops over all 128-query tiles:
//                   S^T  = K^ Q^T            (TMEM, f32)
//                   dP^T = V dO^T            (TMEM, f32)
//                   P    = exp2(S^T c2 - lse2_q),  dS = P (dP - Delta_q)  (registers)
//                   dV  += P dO,  dK^ += dS Q^  (TMEM accumulators)
//                   dQ^ += dS^T K^           (TMEM)
//                 P and dS are written once to shared memory as [key][query]
//                 tiles; the dQ product reads the same dS tile query-major.
//                 "Resident" mode (N <= 256, D <= 64): one CTA per head walks
//                 every key tile and keeps both dQ^ tiles in TMEM, so dQ is
//                 finished on chip with no atomics (deterministic).
//                 "Atomic" mode (any N): one CTA per (head, key tile); each
//                 dQ^ partial is scaled and added into an f32 workspace.
//   dq_finalize   (atomic mode) dQ = R^T dQ^ rounded to the I/O type.
//
// Compared with the reference, S and dP are computed once per (key tile,
// query tile) pair instead of twice, and no separate dQ pass recomputes them.
//
// Warp roles in bwd_kernel: warp 0 TMA producer, warp 1 TMEM allocator + MMA
// issuer, warps 2..5 the row warpgroup (thread = key row of the tile; for dQ
// read-back thread = query row).
//
// TMEM columns: [0,128) S^T, [128,256) dP^T (atomic mode: reused for the dQ^
// partial), [256, 256+DP) dV, [256+DP, 256+2DP) dK^, resident mode:
// [384 + 64 i, 448 + 64 i) dQ^ of query tile i.
#include "frsa_internal.h"
#include "frsa_ptx.cuh"
#include "frsa_rope.cuh"

#undef FRSA_STAMP_TID
#define FRSA_STAMP_TID 128  // first compute thread of this kernel

namespace frsa {

namespace {

constexpr int kComputeThreads = 256;                  // two warpgroups (warps 4..11)
constexpr int kBwdThreads = 128 + kComputeThreads;    // + warpgroup 0: producer, MMA, 2 idle
// Registers: launched at 168 per thread (384 x 168 = 64512); warpgroup 0 then
// drops to 96 and the two compute warpgroups rise to 200: 128*96 + 256*200 = 63488.
constexpr uint32_t kRegsCtl = 96, kRegsCompute = 200;
constexpr int kRowsPerWarp = kTile / (kComputeThreads / 32);  // 16
constexpr uint32_t kTmemColsBwd = 512;

template <int NCH>
struct BwdSmem {
  static constexpr int KVS = (NCH == 1) ? 2 : 1;  // key/value tile stages
  static constexpr int QS = (NCH == 1) ? 2 : 1;   // query/dO tile stages
  uint8_t k[KVS][NCH][kChunkBytes];
  uint8_t v[KVS][NCH][kChunkBytes];
  uint8_t q[QS][NCH][kChunkBytes];
  uint8_t dO[QS][NCH][kChunkBytes];
  uint8_t p[2][kChunkBytes];   // P  [128 key][128 query], two 64-column chunks
  uint8_t ds[2][kChunkBytes];  // dS [128 key][128 query]
  float lse2[QS][kTile];       // lse * log2(e) of the query tile
  float delta[QS][kTile];
  uint64_t kv_full[KVS], kv_empty[KVS];
  uint64_t q_full[QS], q_empty[QS];
  uint64_t kq_ready, st_full, ds_full, mm_done, tm_free, acc_free, dq_free;
  uint32_t tmem_base;
  int abort_flag;
};

struct BwdParams {
  const float* cosp;
  const float* sinp;
  const float* lse;
  const void* o;
  float* delta_out;  // optional: receives Delta when non-null
  // Optional (atomic mode): Delta of every row, computed by delta_rows_kernel
  // before this kernel; when null the kernel forms Delta itself.
  const float* delta_in = nullptr;
  void* dq;
  void* dk;
  void* dv;
  float* dq_accum;
  int BH, N, D, nqt, nkv, has_cls;
  float c2;     // scale * log2(e)
  float scale;
};

template <typename T, int NCH, bool RESIDENT>
__global__ void __launch_bounds__(kBwdThreads, 1)
    bwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
               const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
               const __grid_constant__ CUtensorMap tm_o, const BwdParams prm) {
  using Sm = BwdSmem<NCH>;
  constexpr int KVS = Sm::KVS;
  constexpr int QS = Sm::QS;
  static_assert(!RESIDENT || NCH == 1, "resident mode keeps two dQ tiles of <= 64 columns");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Sm* smp = aligned_smem<Sm>(smem_raw);
  if (smp == nullptr) return;
  Sm& sm = *smp;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int N = prm.N, D = prm.D;
  const int DP = (D + 15) & ~15;
  const int ksteps = DP >> 4;
  const int nqt = prm.nqt;
  // Work units: resident mode = one head (all key tiles), walked persistently
  // (unit = blockIdx.x, blockIdx.x + gridDim.x, ...); atomic mode = one
  // (head, key tile) per CTA.
  const int nunits = RESIDENT ? prm.BH : prm.BH * prm.nkv;
  const int nj = RESIDENT ? prm.nkv : 1;
  auto unit_head = [&](int u) { return RESIDENT ? u : u / prm.nkv; };
  auto unit_j0 = [&](int u) { return RESIDENT ? 0 : u - (u / prm.nkv) * prm.nkv; };
  volatile int* abort_flag = &sm.abort_flag;

  if (threadIdx.x == 0) {
    sm.abort_flag = 0;
    for (int s = 0; s < KVS; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
    }
    for (int s = 0; s < QS; ++s) {
      mbar_init(&sm.q_full[s], 1);
      mbar_init(&sm.q_empty[s], 1);
    }
    mbar_init(&sm.kq_ready, 1);
    mbar_init(&sm.st_full, 1);
    mbar_init(&sm.ds_full, 1);
    mbar_init(&sm.mm_done, 1);
    mbar_init(&sm.tm_free, 1);
    mbar_init(&sm.acc_free, 1);
    mbar_init(&sm.dq_free, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, kTmemColsBwd);
    tmem_relinquish();
  }
  FRSA_STAMP(31);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const uint32_t tST = tmem, tDPT = tmem + 128, tDV = tmem + 256, tDK = tmem + 256 + DP;

  if (warp < 4) {
  setmaxnreg_dec<kRegsCtl>();
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      tma_prefetch_desc(&tm_o);
      int qi = 0, kvi = 0;
      for (int u = blockIdx.x; u < nunits; u += gridDim.x) {
        const int bh = unit_head(u), j0 = unit_j0(u);
        if (RESIDENT) {
          // O rows feed Delta in the compute warps: pull this head's and the
          // next head's O into L2 ahead of those loads.
          for (int i = 0; i < nqt; ++i) {
            for (int c = 0; c < NCH; ++c) {
              if (u == (int)blockIdx.x) tma_prefetch_l2_3d(&tm_o, c * kChunkCols, i * kTile, bh);
              if (u + (int)gridDim.x < nunits)
                tma_prefetch_l2_3d(&tm_o, c * kChunkCols, i * kTile, unit_head(u + gridDim.x));
            }
          }
        }
        for (int jj = 0; jj < nj; ++jj, ++kvi) {
          const int j = j0 + jj, ks = kvi % KVS;
          mbar_wait(&sm.kv_empty[ks], ((kvi / KVS) & 1) ^ 1, abort_flag);
          mbar_arrive_expect_tx(&sm.kv_full[ks], 2 * NCH * kChunkBytes);
          for (int c = 0; c < NCH; ++c) {
            tma_load_3d(sm.k[ks][c], &tm_k, &sm.kv_full[ks], c * kChunkCols, j * kTile, bh);
            tma_load_3d(sm.v[ks][c], &tm_v, &sm.kv_full[ks], c * kChunkCols, j * kTile, bh);
          }
          for (int i = 0; i < nqt; ++i) {
            if (RESIDENT && jj > 0) continue;
            const int qs = qi % QS;
            mbar_wait(&sm.q_empty[qs], ((qi / QS) & 1) ^ 1, abort_flag);
            mbar_arrive_expect_tx(&sm.q_full[qs], 2 * NCH * kChunkBytes);
            for (int c = 0; c < NCH; ++c) {
              tma_load_3d(sm.q[qs][c], &tm_q, &sm.q_full[qs], c * kChunkCols, i * kTile, bh);
              tma_load_3d(sm.dO[qs][c], &tm_do, &sm.q_full[qs], c * kChunkCols, i * kTile, bh);
            }
            ++qi;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr bool kBf = Elt<T>::kBf16;
      const uint32_t idS = idesc_f16(kBf, 128, 128, false, false);   // S^T, dP^T
      const uint32_t idKV = idesc_f16(kBf, 128, DP, false, true);    // dV, dK^
      const uint32_t idQ = idesc_f16(kBf, 128, DP, true, true);      // dQ^
      int it = 0, qi = 0, kvi = 0, hl = 0;
      for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++hl) {
        const int qbase = qi;
        for (int jj = 0; jj < nj; ++jj, ++kvi) {
          const int ks = kvi % KVS;
          for (int i = 0; i < nqt; ++i) {
            const bool fresh = !(RESIDENT && jj > 0);
            const int qs = RESIDENT ? (qbase + i) % QS : qi % QS;
            mbar_wait(&sm.kq_ready, it & 1, abort_flag);
            tc_fence_after();
            if (it > 0) {
              mbar_wait(&sm.tm_free, (it - 1) & 1, abort_flag);
              tc_fence_after();
            }
            for (int kk = 0; kk < ksteps; ++kk) {
              const int c = kk >> 2;
              const uint32_t koff = (kk & 3) * 32;
              mma_ss(tST, sw128_desc(smem_u32(sm.k[ks][c]) + koff, 16, 1024),
                     sw128_desc(smem_u32(sm.q[qs][c]) + koff, 16, 1024), idS, kk > 0);
            }
            for (int kk = 0; kk < ksteps; ++kk) {
              const int c = kk >> 2;
              const uint32_t koff = (kk & 3) * 32;
              mma_ss(tDPT, sw128_desc(smem_u32(sm.v[ks][c]) + koff, 16, 1024),
                     sw128_desc(smem_u32(sm.dO[qs][c]) + koff, 16, 1024), idS, kk > 0);
            }
            mma_commit(&sm.st_full);
            mbar_wait(&sm.ds_full, it & 1, abort_flag);
            tc_fence_after();
            if (i == 0 && kvi > 0) {
              // dV/dK of the previous key tile have been read out.
              mbar_wait(&sm.acc_free, (kvi - 1) & 1, abort_flag);
              tc_fence_after();
            }
            if (RESIDENT && jj == 0 && i == 0 && hl > 0) {
              // dQ of the previous head has been read out.
              mbar_wait(&sm.dq_free, (hl - 1) & 1, abort_flag);
              tc_fence_after();
            }
            for (int kk = 0; kk < kTile / 16; ++kk) {
              const uint32_t aoff = (kk & 3) * 32;
              const uint32_t acc = (i == 0 && kk == 0) ? 0u : 1u;
              // dV += P dO : A = P [key][query] K-major, B = dO [query][d] MN-major.
              mma_ss(tDV, sw128_desc(smem_u32(sm.p[kk >> 2]) + aoff, 16, 1024),
                     sw128_desc(smem_u32(sm.dO[qs][0]) + kk * 2048, kChunkBytes, 1024), idKV,
                     acc);
              // dK^ += dS Q^ : B = Q^ [query][d] MN-major.
              mma_ss(tDK, sw128_desc(smem_u32(sm.ds[kk >> 2]) + aoff, 16, 1024),
                     sw128_desc(smem_u32(sm.q[qs][0]) + kk * 2048, kChunkBytes, 1024), idKV,
                     acc);
            }
            // dQ^ (+)= dS^T K^ : A = dS read query-major (MN-major), B = K^ [key][d] MN-major.
            const uint32_t tDQ = RESIDENT ? (tmem + 384 + 64 * i) : tDPT;
            for (int kk = 0; kk < kTile / 16; ++kk) {
              const uint32_t acc =
                  RESIDENT ? ((jj == 0 && kk == 0) ? 0u : 1u) : (kk > 0 ? 1u : 0u);
              mma_ss(tDQ, sw128_desc(smem_u32(sm.ds[0]) + kk * 2048, kChunkBytes, 1024),
                     sw128_desc(smem_u32(sm.k[ks][0]) + kk * 2048, kChunkBytes, 1024), idQ, acc);
            }
            mma_commit(&sm.mm_done);
            if (!RESIDENT || jj == nj - 1) mma_commit(&sm.q_empty[qs]);
            if (i == nqt - 1) mma_commit(&sm.kv_empty[ks]);
            ++it;
            if (fresh) ++qi;
          }
        }
      }
    }
  }
  } else {
    setmaxnreg_inc<kRegsCompute>();
    // ------------------------------------------------------------ compute warps
    // Two warpgroups (warps 4..11). For TMEM reads a thread owns row r (its
    // lane quarter wq); warpgroup g takes S/dP columns [64g, 64g + 64) and
    // every other 16-column block of the epilogue tiles. Warp-per-row phases
    // (rotation, Delta, drains) give each of the 8 warps 16 rows.
    constexpr int RW = kRowsPerWarp;
    const int cw = warp - 4;                       // compute warp 0..7
    const int g = cw >> 2;                         // warpgroup 0..1
    const int wq = warp & 3;                       // TMEM lane quarter
    const int r = wq * 32 + lane;
    const int rw0 = cw * RW;                       // first row of this warp's row slice
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const bool leader = threadIdx.x == 128;
    const float c2 = prm.c2;
    int bh = 0, j0 = 0;          // current unit (set at the top of the unit loop)
    int it = 0, qi = 0, kvi = 0, hl = 0;  // running iteration / load / unit counters
    size_t head_row0 = 0;

    // Resident mode: this warp always handles the same 16-row slices of token
    // tiles 0 and 1, so its table values are the same for every head; they
    // are loaded once and kept in registers for the kernel's lifetime.
    RopeQ<NCH, RW> tab[RESIDENT ? 2 : 1];
    if (RESIDENT) {
#pragma unroll
      for (int t = 0; t < (RESIDENT ? 2 : 1); ++t)
        load_rope_q<NCH, RW>(tab[t], rw0, t * kTile, N, prm.has_cls, D, prm.cosp, prm.sinp,
                             lane);
    }

    // Rotate key tile j_ (the kvi_-th key/value load) in its stage.
    auto prep_k = [&](int j_, int kvi_) {
      if (RESIDENT) {
        mbar_wait(&sm.kv_full[kvi_ % KVS], (kvi_ / KVS) & 1, abort_flag);
        if (j_ & 1) apply_rope_q<T, NCH, RW>(&sm.k[kvi_ % KVS][0][0], rw0, D, tab[RESIDENT ? 1 : 0], lane);
        else apply_rope_q<T, NCH, RW>(&sm.k[kvi_ % KVS][0][0], rw0, D, tab[0], lane);
      } else {
        RopeQ<NCH, RW> rope;
        load_rope_q<NCH, RW>(rope, rw0, j_ * kTile, N, prm.has_cls, D, prm.cosp, prm.sinp, lane);
        mbar_wait(&sm.kv_full[kvi_ % KVS], (kvi_ / KVS) & 1, abort_flag);
        apply_rope_q<T, NCH, RW>(&sm.k[kvi_ % KVS][0][0], rw0, D, rope, lane);
      }
    };
    // Prepare query tile i_ in stage qs_ (the qi_-th query load): lse2 (+inf
    // for padded rows, so their P is exactly 0), rotation of Q, and Delta.
    auto prep_q = [&](int i_, int qs_, int qi_) {
      const int q0_ = i_ * kTile;
      if (g == 0) {
        const bool qv = (q0_ + r) < N;
        sm.lse2[qs_][r] = qv ? prm.lse[head_row0 + q0_ + r] * 1.4426950408889634f : INFINITY;
      }
      // O granules of this warp's query rows (quad layout), read before the
      // tile wait so the load overlaps it.
      const bool dpre = !RESIDENT && prm.delta_in != nullptr;
      if (dpre && g == 0)
        sm.delta[qs_][r] = (q0_ + r) < N ? prm.delta_in[head_row0 + q0_ + r] : 0.f;
      const int rq = lane >> 3, gl = lane & 7;
      uint4 og[NCH][RW / 4];
#pragma unroll
      for (int k = 0; k < RW / 4; ++k)
#pragma unroll
        for (int h = 0; h < NCH; ++h) {
          const int tok = q0_ + rw0 + 4 * k + rq, gg = gl + 8 * h;
          og[h][k] = (!dpre && tok < N && 8 * gg < D)
                         ? __ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(prm.o) +
                                                                (head_row0 + tok) * D) + gg)
                         : make_uint4(0u, 0u, 0u, 0u);
        }
      if (RESIDENT) {
        if (hl == 1 && i_ == 0) FRSA_STAMP(18);
        mbar_wait(&sm.q_full[qs_], (qi_ / QS) & 1, abort_flag);
        if (hl == 1 && i_ == 0) FRSA_STAMP(19);
        if (i_ & 1) apply_rope_q<T, NCH, RW>(&sm.q[qs_][0][0], rw0, D, tab[RESIDENT ? 1 : 0], lane);
        else apply_rope_q<T, NCH, RW>(&sm.q[qs_][0][0], rw0, D, tab[0], lane);
      } else {
        RopeQ<NCH, RW> rope;
        load_rope_q<NCH, RW>(rope, rw0, q0_, N, prm.has_cls, D, prm.cosp, prm.sinp, lane);
        mbar_wait(&sm.q_full[qs_], (qi_ / QS) & 1, abort_flag);
        apply_rope_q<T, NCH, RW>(&sm.q[qs_][0][0], rw0, D, rope, lane);
      }
      if (hl == 1 && i_ == 0) FRSA_STAMP(20);
      // Delta = sum_d O dO per query row: each lane dots its granule of O with
      // the same granule of the (unrotated) dO tile; 8 lanes share a row.
      const uint32_t dob = smem_u32(&sm.dO[qs_][0][0]);
#pragma unroll
      for (int k = 0; k < (dpre ? 0 : RW / 4); ++k) {
        float dl = 0.f;
#pragma unroll
        for (int h = 0; h < NCH; ++h) {
          if (8 * (gl + 8 * h) < D) {
            const uint4 b = lds_u4(dob + h * 16384 + sw128_off(rw0 + 4 * k + rq, gl));
            const uint32_t aw[4] = {og[h][k].x, og[h][k].y, og[h][k].z, og[h][k].w};
            const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 x = Elt<T>::unpack(aw[e]), y = Elt<T>::unpack(bw[e]);
              dl = fmaf(x.x, y.x, fmaf(x.y, y.y, dl));
            }
          }
        }
        dl += __shfl_xor_sync(0xffffffffu, dl, 1);
        dl += __shfl_xor_sync(0xffffffffu, dl, 2);
        dl += __shfl_xor_sync(0xffffffffu, dl, 4);
        if (gl == 0) {
          const int rr = rw0 + 4 * k + rq;
          sm.delta[qs_][rr] = dl;
          if (prm.delta_out != nullptr && j0 == 0 && q0_ + rr < N)
            prm.delta_out[head_row0 + q0_ + rr] = dl;
        }
      }
      if (hl == 1 && i_ == 0) FRSA_STAMP(21);
    };

    // Per unit: the first iteration's operands, then one iteration of
    // look-ahead: the next key/query tile is prepared while the tensor core
    // computes S^T and dP^T.
    for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++hl) {
    bh = unit_head(u);
    j0 = unit_j0(u);
    head_row0 = static_cast<size_t>(bh) * N;
    const int qbase = qi, kvbase = kvi, itbase = it;
    (void)itbase;  // used by trace stamps only
    if (hl == 1) FRSA_STAMP(16);
    prep_k(j0, kvbase);
    if (hl == 1) FRSA_STAMP(17);
    prep_q(0, qi % QS, qi);
    ++qi;
    int cur_qs = qbase % QS;
    fence_proxy_async_smem();
    named_bar(1, kComputeThreads);
    if (leader) mbar_arrive(&sm.kq_ready);
    for (int jj = 0; jj < nj; ++jj) {
      const int j = j0 + jj;
      const int kv0 = j * kTile;
      for (int i = 0; i < nqt; ++i) {
        const int q0 = i * kTile;
        const int qs = cur_qs;
        const bool has_next = (i + 1 < nqt) || (jj + 1 < nj);
        // Look-ahead needs the next query tile in a different stage: with one
        // stage it can only arrive after this iteration's MMAs, so it is
        // prepared after them instead (prep_late).
        auto prep_next = [&]() {
          const int nj_ = (i + 1 < nqt) ? jj : jj + 1;
          const int ni = (i + 1 < nqt) ? i + 1 : 0;
          if (ni == 0) prep_k(j0 + nj_, kvbase + nj_);
          const bool nfresh = !(RESIDENT && nj_ > 0);
          const int nqs = RESIDENT ? (qbase + ni) % QS : qi % QS;
          if (nfresh) {
            prep_q(ni, nqs, qi);
            ++qi;
          }
          cur_qs = nqs;
        };
        const bool prep_late = has_next && (QS == 1 || KVS == 1);
        if (has_next && !prep_late) prep_next();
        if (hl == 0) FRSA_STAMP(hl * 15 + (it - itbase) * 3 + 0);

        mbar_wait(&sm.st_full, it & 1, abort_flag);
        if (hl == 0) FRSA_STAMP(hl * 15 + (it - itbase) * 3 + 1);
        tc_fence_after();
        if (it > 0) mbar_wait(&sm.mm_done, (it - 1) & 1, abort_flag);  // P/dS tiles free
        {
          // This warpgroup's 64 columns: S^T and dP^T loaded at once. Padded
          // query columns have lse2 = +inf (P = 0, dS = 0); padded key rows
          // only reach dV/dK rows that are never stored and dQ through zero
          // K^ rows, so no per-element masking is needed.
          float sv[2][32], dp[2][32];
          tmem_ld32(tST + lane_off + g * 64, sv[0]);
          tmem_ld32(tST + lane_off + g * 64 + 32, sv[1]);
          tmem_ld32(tDPT + lane_off + g * 64, dp[0]);
          tmem_ld32(tDPT + lane_off + g * 64 + 32, dp[1]);
          tmem_wait_ld();
          const uint32_t pbase = smem_u32(sm.p[g]), dbase = smem_u32(sm.ds[g]);
          const uint32_t lbase = smem_u32(&sm.lse2[qs][g * 64]);
          const uint32_t ebase = smem_u32(&sm.delta[qs][g * 64]);
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
            for (int c4 = 0; c4 < 8; ++c4) {
              const float4 l4 = lds_f4(lbase + (hh * 32 + c4 * 4) * 4);
              const float4 d4 = lds_f4(ebase + (hh * 32 + c4 * 4) * 4);
              const float lv[4] = {l4.x, l4.y, l4.z, l4.w}, dv4[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int c = c4 * 4 + e;
                const float pv = ex2(fmaf(sv[hh][c], c2, -lv[e]));
                sv[hh][c] = pv;
                dp[hh][c] = pv * (dp[hh][c] - dv4[e]);
              }
            }
#pragma unroll
            for (int g4 = 0; g4 < 4; ++g4) {
              const uint32_t off = sw128_off(r, hh * 4 + g4);
              uint4 w;
              w.x = Elt<T>::pack(sv[hh][g4 * 8 + 0], sv[hh][g4 * 8 + 1]);
              w.y = Elt<T>::pack(sv[hh][g4 * 8 + 2], sv[hh][g4 * 8 + 3]);
              w.z = Elt<T>::pack(sv[hh][g4 * 8 + 4], sv[hh][g4 * 8 + 5]);
              w.w = Elt<T>::pack(sv[hh][g4 * 8 + 6], sv[hh][g4 * 8 + 7]);
              sts_u4(pbase + off, w);
              w.x = Elt<T>::pack(dp[hh][g4 * 8 + 0], dp[hh][g4 * 8 + 1]);
              w.y = Elt<T>::pack(dp[hh][g4 * 8 + 2], dp[hh][g4 * 8 + 3]);
              w.z = Elt<T>::pack(dp[hh][g4 * 8 + 4], dp[hh][g4 * 8 + 5]);
              w.w = Elt<T>::pack(dp[hh][g4 * 8 + 6], dp[hh][g4 * 8 + 7]);
              sts_u4(dbase + off, w);
            }
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        named_bar(1, kComputeThreads);
        if (leader) {
          mbar_arrive(&sm.ds_full);
          if (RESIDENT) {
            mbar_arrive(&sm.tm_free);
            if (has_next && !prep_late) mbar_arrive(&sm.kq_ready);
          }
        }
        if (hl == 0) FRSA_STAMP(hl * 15 + (it - itbase) * 3 + 2);
        if (!RESIDENT) {
          // dQ^ partial of this (key tile, query tile): scale and add into the workspace.
          mbar_wait(&sm.mm_done, it & 1, abort_flag);
          tc_fence_after();
          uint8_t* stage = &sm.p[0][0];  // P/dS tiles are free until the next iteration
#pragma unroll 1
          for (int c16 = g; c16 < 4 * NCH; c16 += 2) {
            if (c16 * 16 < DP) {
              float v[16];
              tmem_ld16(tDPT + lane_off + c16 * 16, v);
              tmem_wait_ld();
              stage_write16<NCH>(stage, r, c16, v);
            }
          }
          named_bar(1, kComputeThreads);
          {
            const uint32_t sbase = smem_u32(stage);
            const int rq = lane >> 3, gl = lane & 7;
#pragma unroll
            for (int k = 0; k < RW / 4; ++k) {
              const int rr = rw0 + 4 * k + rq, tok = q0 + rr;
#pragma unroll
              for (int h = 0; h < NCH; ++h) {
                const int gg = gl + 8 * h;
                if (tok < N && 8 * gg < D) {
                  float v[8];
                  stage_read8<NCH>(sbase, rr, gg, prm.scale, v);
                  float4* dst = reinterpret_cast<float4*>(prm.dq_accum + (head_row0 + tok) * D + 8 * gg);
                  atomicAdd(dst, make_float4(v[0], v[1], v[2], v[3]));
                  atomicAdd(dst + 1, make_float4(v[4], v[5], v[6], v[7]));
                }
              }
            }
          }
          tc_fence_before();
          named_bar(1, kComputeThreads);
          if (leader) {
            mbar_arrive(&sm.tm_free);
            if (has_next && !prep_late) mbar_arrive(&sm.kq_ready);
          }
        }
        if (prep_late) {
          prep_next();
          fence_proxy_async_smem();
          named_bar(1, kComputeThreads);
          if (leader) mbar_arrive(&sm.kq_ready);
        }
        ++it;
      }
      // dV, dK epilogue of key tile j
      RopeQ<NCH, RW> rope_k;
      if (!RESIDENT) load_rope_q<NCH, RW>(rope_k, rw0, kv0, N, prm.has_cls, D, prm.cosp, prm.sinp, lane);
      mbar_wait(&sm.mm_done, (it - 1) & 1, abort_flag);
      tc_fence_after();
      {
        // TMEM rows -> f32 staging (P/dS tiles, free now) -> warp-per-row drain.
        uint8_t* stage_v = &sm.p[0][0];
        uint8_t* stage_k = (NCH == 1) ? &sm.ds[0][0] : &sm.p[0][0];
        T* dv_head = reinterpret_cast<T*>(prm.dv) + head_row0 * D;
        T* dk_head = reinterpret_cast<T*>(prm.dk) + head_row0 * D;
#pragma unroll 1
        for (int c16 = g; c16 < 4 * NCH; c16 += 2) {
          if (c16 * 16 < DP) {
            float v[16];
            tmem_ld16(tDV + lane_off + c16 * 16, v);
            tmem_wait_ld();
            stage_write16<NCH>(stage_v, r, c16, v);
          }
        }
        if (NCH != 1) {
          named_bar(1, kComputeThreads);
          drain_q<T, NCH, RW>(stage_v, rw0, kv0, N, D, 1.f, static_cast<const RopeQ<NCH, RW>*>(nullptr), dv_head, lane);
          named_bar(1, kComputeThreads);
        }
#pragma unroll 1
        for (int c16 = g; c16 < 4 * NCH; c16 += 2) {
          if (c16 * 16 < DP) {
            float v[16];
            tmem_ld16(tDK + lane_off + c16 * 16, v);
            tmem_wait_ld();
            stage_write16<NCH>(stage_k, r, c16, v);
          }
        }
        named_bar(1, kComputeThreads);
        if (NCH == 1)
          drain_q<T, NCH, RW>(stage_v, rw0, kv0, N, D, 1.f, static_cast<const RopeQ<NCH, RW>*>(nullptr), dv_head, lane);
        if (RESIDENT && (j & 1))
          drain_q<T, NCH, RW>(stage_k, rw0, kv0, N, D, prm.scale, &tab[RESIDENT ? 1 : 0], dk_head, lane);
        else if (RESIDENT)
          drain_q<T, NCH, RW>(stage_k, rw0, kv0, N, D, prm.scale, &tab[0], dk_head, lane);
        else
          drain_q<T, NCH, RW>(stage_k, rw0, kv0, N, D, prm.scale, &rope_k, dk_head, lane);
      }
      tc_fence_before();
      named_bar(1, kComputeThreads);
      if (leader) mbar_arrive(&sm.acc_free);
      if (hl == 0) FRSA_STAMP(hl * 15 + 12 + jj);
      ++kvi;
    }
    if (RESIDENT) {
      // dQ epilogue: every MMA has completed (last mm_done waited above).
      uint8_t* stage = &sm.p[0][0];
      T* dq_head = reinterpret_cast<T*>(prm.dq) + head_row0 * D;
      for (int i = 0; i < nqt; ++i) {

#pragma unroll 1
        for (int c16 = g; c16 < 4; c16 += 2) {
          if (c16 * 16 < DP) {
            float v[16];
            tmem_ld16(tmem + 384 + 64 * i + lane_off + c16 * 16, v);
            tmem_wait_ld();
            stage_write16<NCH>(stage, r, c16, v);
          }
        }
        named_bar(1, kComputeThreads);
        if (i & 1)
          drain_q<T, NCH, RW>(stage, rw0, i * kTile, N, D, prm.scale, &tab[RESIDENT ? 1 : 0],
                              dq_head, lane);
        else
          drain_q<T, NCH, RW>(stage, rw0, i * kTile, N, D, prm.scale, &tab[0], dq_head, lane);
        tc_fence_before();
        named_bar(1, kComputeThreads);
      }
      if (leader) mbar_arrive(&sm.dq_free);
      if (hl == 0) FRSA_STAMP(hl * 15 + 14);
    }
    }  // unit loop
  }

  FRSA_STAMP(30);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemColsBwd);
  }
}

// dQ = R^T dQ^ (dQ^ already scaled), one thread per 8 columns.
// Delta = rowsum(dO * O) in f32 for every row of [B*H*N, D]: 8 lanes per
// row, one 16-byte granule each per step (fa_rope_full .py:352-357).
template <typename T>
__global__ void delta_rows_kernel(const T* __restrict__ o, const T* __restrict__ d_o,
                                  float* __restrict__ delta, long long rows, int D) {
  const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 3;
  const int gl = threadIdx.x & 7;
  float acc = 0.f;
  if (row < rows) {
    const uint4* orow = reinterpret_cast<const uint4*>(o + row * D);
    const uint4* drow = reinterpret_cast<const uint4*>(d_o + row * D);
    for (int gg = gl; 8 * gg < D; gg += 8) {
      const uint4 a = __ldg(orow + gg), b = __ldg(drow + gg);
      const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
      const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 x = Elt<T>::unpack(aw[e]), y = Elt<T>::unpack(bw[e]);
        acc = fmaf(x.x, y.x, fmaf(x.y, y.y, acc));
      }
    }
  }
  acc += __shfl_xor_sync(0xffffffffu, acc, 1);
  acc += __shfl_xor_sync(0xffffffffu, acc, 2);
  acc += __shfl_xor_sync(0xffffffffu, acc, 4);
  if (gl == 0 && row < rows) delta[row] = acc;
}

template <typename T>
__global__ void dq_finalize_kernel(const float* __restrict__ acc, T* __restrict__ dq,
                                   const float* __restrict__ cosp, const float* __restrict__ sinp,
                                   long long rows, int N, int D, int has_cls) {
  const int gpr = D >> 3;
  const long long gidx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gidx >= rows * gpr) return;
  const long long row = gidx / gpr;
  const int g = static_cast<int>(gidx - row * gpr);
  const int t = static_cast<int>(row % N);
  const float4* src = reinterpret_cast<const float4*>(acc + row * D + g * 8);
  float v[8];
  const float4 a = src[0], b = src[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  const int pos = rope_pos(t, N, has_cls);
  if (pos >= 0) {
    const int D2 = D >> 1;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const float c = __ldg(cosp + static_cast<size_t>(pos) * D2 + g * 4 + p);
      const float s = __ldg(sinp + static_cast<size_t>(pos) * D2 + g * 4 + p);
      const float e = v[2 * p], od = v[2 * p + 1];
      v[2 * p] = e * c + od * s;
      v[2 * p + 1] = od * c - e * s;
    }
  }
  uint4 w;
  w.x = Elt<T>::pack(v[0], v[1]);
  w.y = Elt<T>::pack(v[2], v[3]);
  w.z = Elt<T>::pack(v[4], v[5]);
  w.w = Elt<T>::pack(v[6], v[7]);
  reinterpret_cast<uint4*>(dq + row * D)[g] = w;
}

}  // namespace

bool bwd_needs_workspace(const LaunchShape& s) { return !(s.N <= 2 * kTile && s.D <= 64); }

namespace {

template <typename T, int NCH, bool RESIDENT>
cudaError_t launch_bwd_main(const LaunchShape& s, const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                            const CUtensorMap& tm_v, const CUtensorMap& tm_do,
                            const CUtensorMap& tm_o, const BwdParams& p, cudaStream_t stream) {
  const size_t smem = sizeof(BwdSmem<NCH>) + 1024;
  auto kern = bwd_kernel<T, NCH, RESIDENT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int nsm = 148;
  {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  }
  const long long grid = RESIDENT ? static_cast<long long>(s.BH < nsm ? s.BH : nsm)
                                  : static_cast<long long>(s.BH) * p.nkv;
  kern<<<static_cast<unsigned>(grid), kBwdThreads, smem, stream>>>(tm_q, tm_k, tm_v, tm_do, tm_o,
                                                                     p);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_bwd_t(const LaunchShape& s, const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                         const CUtensorMap& tm_v, const CUtensorMap& tm_do,
                         const CUtensorMap& tm_o, const void* o,
                         const CUtensorMap* tm_grads, const void* d_o, const float* lse,
                         float* delta, const float* cosp, const float* sinp, void* dq, void* dk,
                         void* dv, float* dq_accum, float* delta_buf, cudaStream_t stream) {
  const long long rows = static_cast<long long>(s.BH) * s.N;
  BwdParams p;
  p.cosp = cosp;
  p.sinp = sinp;
  p.lse = lse;
  p.o = o;
  p.delta_out = delta;
  p.dq = dq;
  p.dk = dk;
  p.dv = dv;
  p.dq_accum = dq_accum;
  p.BH = s.BH;
  p.N = s.N;
  p.D = s.D;
  p.nqt = (s.N + kTile - 1) / kTile;
  p.nkv = p.nqt;
  p.has_cls = s.has_cls;
  p.c2 = s.scale * 1.4426950408889634f;
  p.scale = s.scale;
  cudaError_t e;
  if (!bwd_needs_workspace(s)) {
    if (tm_grads == nullptr) return cudaErrorInvalidValue;
    return launch_bwd_small(s, tm_q, tm_k, tm_v, tm_do, tm_o, tm_grads, o, lse, delta, cosp, sinp,
                            dq, dk, dv, stream);
  }
  e = cudaMemsetAsync(dq_accum, 0, static_cast<size_t>(rows) * s.D * sizeof(float), stream);
  if (e != cudaSuccess) return e;
  if (delta_buf != nullptr) {
    // Delta once per row here, instead of once per (key tile, query tile) in
    // the main kernel (which would also re-read O for every key tile).
    const long long threads_d = rows * 8;
    delta_rows_kernel<T><<<static_cast<unsigned>((threads_d + 255) / 256), 256, 0, stream>>>(
        static_cast<const T*>(o), static_cast<const T*>(d_o), delta_buf, rows, s.D);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    p.delta_in = delta_buf;
    p.delta_out = nullptr;   // delta_buf is the caller's delta when one was given
  }
  e = (s.D > 64) ? launch_bwd_main<T, 2, false>(s, tm_q, tm_k, tm_v, tm_do, tm_o, p, stream)
                 : launch_bwd_main<T, 1, false>(s, tm_q, tm_k, tm_v, tm_do, tm_o, p, stream);
  if (e != cudaSuccess) return e;
  const int threads = 256;
  const long long total = rows * (s.D >> 3);
  dq_finalize_kernel<T><<<static_cast<unsigned>((total + threads - 1) / threads), threads, 0,
                          stream>>>(dq_accum, static_cast<T*>(dq), cosp, sinp, rows, s.N, s.D,
                                    s.has_cls);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_bwd(const LaunchShape& s, const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                       const CUtensorMap& tm_v, const CUtensorMap& tm_do, const CUtensorMap& tm_o,
                       const void* o, const CUtensorMap* tm_grads,
                       const void* d_o, const float* lse, float* delta, const float* cosp,
                       const float* sinp, void* dq, void* dk, void* dv, float* dq_accum,
                       float* delta_buf, cudaStream_t stream) {
  if (s.bf16)
    return launch_bwd_t<__nv_bfloat16>(s, tm_q, tm_k, tm_v, tm_do, tm_o, o, tm_grads, d_o, lse,
                                       delta, cosp, sinp, dq, dk, dv, dq_accum, delta_buf, stream);
  return launch_bwd_t<__half>(s, tm_q, tm_k, tm_v, tm_do, tm_o, o, tm_grads, d_o, lse, delta, cosp,
                              sinp, dq, dk, dv, dq_accum, delta_buf, stream);
}

}  // namespace frsa
