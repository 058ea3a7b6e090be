// Backward kernels: dQ, dK, dV of softmax(R(Q) R(K)^T * scale) V for the shapes
// the persistent single-head kernel (frsa_bwd_small.cu) does not cover
// (N > 256 or D > 64).
//
// Restates _attn_bwd_preprocess, _attn_bwd_dk_dv_rope and _attn_bwd_dq_rope
// (fa_rope_full .py:325-357, 374-691, 708-1009) as:
//
//   delta_rows    Delta = rowsum(dO * O) once per row (fa_rope_full .py:352-357).
//   bwd_kernel    persistent key-major tcgen05 kernel. A work unit is one
//                 (batch*head, 128-key tile); CTAs claim units in increasing
//                 order from a ticket counter and walk every 128-query tile:
//                   S^T  = K^ Q^T            (TMEM, f32)
//                   dP^T = V dO^T            (TMEM, f32)
//                   P    = exp2(S^T c2 - lse2_q),  dS = P (dP - Delta_q)  (registers)
//                   dV  += P dO,  dK^ += dS Q^  (TMEM accumulators)
//                   dQ^_j = dS^T K^          (TMEM, this key tile's share)
//                 P and dS are packed into TMEM over the scores (A operands
//                 of the dV and dK products); dS also goes to shared memory
//                 as a [key][query] tile, which the dQ product reads
//                 query-major.
//   dq_finalize   dQ = R^T (sum of the partial slots, in slot order) per row.
//
// dQ is reduced over key tiles in a fixed order, so the result is bitwise
// reproducible (the reference's dQ kernel is deterministic too: one program
// per query tile, fa_rope_full .py:708-1009). Key tile j of a head writes its
// scaled dQ^ share of query tile i into partial slot s = j % S of the
// workspace (S = nslot; when key tiles share a slot, j >= S first waits for
// its predecessor j - S in that slot and adds to it, so each slot holds the
// in-order sum of its key tiles). After the main kernel, dq_finalize sums
// each row's S slots in slot order, un-rotates with R^T (fa_rope_full
// .py:974-993) and writes dQ in the I/O type. No CTA waits for another
// unless slots are shared, and then only for a unit claimed S units earlier.
// Units are claimed in order, so a unit waited for is always held by a
// running CTA; every wait is bounded.
//
// Compared with the reference, S and dP are computed once per (key tile,
// query tile) pair instead of twice, and no separate dQ pass recomputes them.
//
// Warp roles in bwd_kernel: warp 0 TMA producer (and unit claims), warp 1
// TMEM allocator + MMA issuer, warps 4..11 two row warpgroups (thread = key
// row of the tile; for dQ read-back thread = query row).
//
// TMEM columns: [0,128) S^T, [128,256) dP^T, [256, 256+DP) dV,
// [256+DP, 256+2DP) dK^, [256+2DP, 256+3DP) the dQ^ share when that fits in
// 512 columns (D <= 80), else the dQ^ share reuses the dP^T columns.
//
// Pipelining (per CTA). An iteration is one (key tile, query tile) pair; the
// iterations of consecutive units form one sequence. For D <= 64 (two query
// stages) the MMA warp issues S^T/dP^T of iteration t + 1 as soon as the row
// warps have loaded iteration t's S^T/dP^T into registers, before issuing the
// gradient products of t, and the row warps drain iteration t - 1's dQ^
// share (and, at a unit's end, its dV and dK^) while the tensor core runs the
// products of t: the exponentials of one iteration overlap the products of
// the neighbouring ones. With one query stage (D > 64) the next query tile
// can only load once t's products are done, so t's results are drained and
// the next tile prepared right after them.
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
constexpr int kUnitRing = 4;   // claimed units published by the producer
}  // namespace
// Partial dQ slots of the general backward (frsa_bwd): key tiles j and j + 8
// share a slot, in order.
constexpr int kMaxDqSlots = 8;
namespace {

template <int NCH>
struct BwdSmem {
  static constexpr int KVS = (NCH == 1) ? 2 : 1;  // key/value tile stages
  static constexpr int QS = (NCH == 1) ? 2 : 1;   // query/dO tile stages
  uint8_t k[KVS][NCH][kChunkBytes];
  uint8_t v[KVS][NCH][kChunkBytes];
  uint8_t q[QS][NCH][kChunkBytes];
  uint8_t dO[QS][NCH][kChunkBytes];
  uint8_t ds[2][kChunkBytes];  // dS [128 key][128 query], two 64-column chunks
  // Store staging. D <= 64: two areas of two chunks, one for the f32 dQ^
  // shares and one for the dV and dK^ tiles, each with its own store thread,
  // so a unit's dV/dK store and its last dQ^ share are in flight together.
  // With one query stage the dS tile, idle while results drain, and this
  // area form one four-chunk stage for all results.
  static constexpr int NSTAGE = (NCH == 1) ? 4 : 2;
  uint8_t stage[NSTAGE][kChunkBytes];
  alignas(16) float lse2[QS][kTile];   // lse * log2(e) of the query tile (read as float4)
  alignas(16) float delta[QS][kTile];
  uint64_t kv_full[KVS], kv_empty[KVS];
  uint64_t q_full[QS], q_empty[QS];
  uint64_t kq_ready, st_full, st_free, ds_full, mm_done, dq_free, acc_free;
  uint64_t unit_full[kUnitRing], unit_empty[kUnitRing];
  // Result jobs, row warps -> store threads, on channel 0 (dQ^ shares, and
  // everything when there is one stage area) and channel 1 (dV/dK).
  uint64_t stage_full[2], stage_free[2];
  int job_type[2], job_bh[2], job_j[2], job_i[2];
  int unit[kUnitRing];
  uint32_t tmem_base;
  int abort_flag;
};

struct BwdParams {
  const float* cosp;
  const float* sinp;
  const float* lse;
  const void* o;
  float* delta_out;  // optional: receives Delta when non-null (in-kernel Delta only)
  // Optional: Delta of every row, computed by delta_rows_kernel before this
  // kernel; when null the kernel forms Delta itself.
  const float* delta_in = nullptr;
  void* dq;
  void* dk;
  void* dv;
  float* dq_part;    // f32 [nslot][BH, N, D] partial dQ^ sums (no initial value needed)
  int* arrive;       // [BH * nqt] (reserved in the workspace layout; unused)
  int* turns;        // [BH * nqt * nslot] slot turn counters, zero at launch
  int* ticket;       // unit claim counter, zero at launch
  int nslot;         // partial slots S (1 .. nkv)
  int rot_in;        // 1: rotate the Q and K tiles here; 0: they arrive rotated
  int BH, H, N, D, nqt, nkv, has_cls;
  float c2;     // scale * log2(e)
  float scale;
};

template <typename T, int NCH>
__global__ void __launch_bounds__(kBwdThreads, 1)
    bwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
               const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
               const __grid_constant__ CUtensorMap tm_o, const __grid_constant__ CUtensorMap tm_dk,
               const __grid_constant__ CUtensorMap tm_dv,
               const __grid_constant__ CUtensorMap tm_part, const BwdParams prm) {
  using Sm = BwdSmem<NCH>;
  constexpr int KVS = Sm::KVS;
  constexpr int QS = Sm::QS;
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
  const int nunits = prm.BH * prm.nkv;   // unit u = (head u / nkv, key tile u % nkv)
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
    mbar_init(&sm.st_free, 1);
    mbar_init(&sm.dq_free, 1);
    mbar_init(&sm.acc_free, 1);
    for (int c = 0; c < 2; ++c) {
      mbar_init(&sm.stage_full[c], 1);
      mbar_init(&sm.stage_free[c], 1);
    }
    for (int s = 0; s < kUnitRing; ++s) {
      mbar_init(&sm.unit_full[s], 1);
      mbar_init(&sm.unit_empty[s], 1 + kComputeThreads);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, kTmemColsBwd);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const uint32_t tST = tmem, tDPT = tmem + 128, tDV = tmem + 256, tDK = tmem + 256 + DP;
  const uint32_t tDQ = (256 + 3 * DP <= 512) ? tmem + 256 + 2 * DP : tDPT;
  constexpr bool kAhead = (QS == 2);   // S^T/dP^T of t + 1 ahead of t's gradient products
  constexpr bool kSplit = Sm::NSTAGE == 4;   // separate stage areas for dQ^ and dV/dK
  // Number of 16-token steps of tile t that hold tokens (8 for a full tile):
  // products skip the steps of a last tile that are only padding.
  auto valid16 = [&](int t) -> int { return min(8, (N - t * kTile + 15) >> 4); };

  // The n-th claimed unit of this CTA (-1: no more work, or aborting).
  auto next_unit = [&](int n) -> int {
    const int slot = n % kUnitRing;
    mbar_wait(&sm.unit_full[slot], (n / kUnitRing) & 1, abort_flag);
    const int u = *abort_flag ? -1 : *reinterpret_cast<volatile int*>(&sm.unit[slot]);
    mbar_arrive(&sm.unit_empty[slot]);
    return u;
  };

  if (warp < 4) {
  setmaxnreg_dec<kRegsCtl>();
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      int qi = 0;
      for (int n = 0;; ++n) {
        const int slot = n % kUnitRing;
        mbar_wait(&sm.unit_empty[slot], ((n / kUnitRing) & 1) ^ 1, abort_flag);
        int u = atomicAdd(prm.ticket, 1);
        if (u >= nunits || *abort_flag) u = -1;
        sm.unit[slot] = u;
        mbar_arrive(&sm.unit_full[slot]);
        if (u < 0) break;
        const int bh = u / prm.nkv, j = u - bh * prm.nkv, ks = n % KVS;
        mbar_wait(&sm.kv_empty[ks], ((n / KVS) & 1) ^ 1, abort_flag);
        mbar_arrive_expect_tx(&sm.kv_full[ks], 2 * NCH * kChunkBytes);
        for (int c = 0; c < NCH; ++c) {
          tma_load_bh(sm.k[ks][c], &tm_k, &sm.kv_full[ks], c * kChunkCols, j * kTile, bh, prm.H);
          tma_load_bh(sm.v[ks][c], &tm_v, &sm.kv_full[ks], c * kChunkCols, j * kTile, bh, prm.H);
        }
        for (int i = 0; i < nqt; ++i, ++qi) {
          const int qs = qi % QS;
          mbar_wait(&sm.q_empty[qs], ((qi / QS) & 1) ^ 1, abort_flag);
          mbar_arrive_expect_tx(&sm.q_full[qs], 2 * NCH * kChunkBytes);
          for (int c = 0; c < NCH; ++c) {
            tma_load_bh(sm.q[qs][c], &tm_q, &sm.q_full[qs], c * kChunkCols, i * kTile, bh, prm.H);
            tma_load_bh(sm.dO[qs][c], &tm_do, &sm.q_full[qs], c * kChunkCols, i * kTile, bh, prm.H);
            // The tile after it into L2 now: its load is issued only when a
            // stage frees, and then mostly hits L2.
            if (i + 1 < nqt) {
              tma_prefetch_l2_bh(&tm_q, c * kChunkCols, (i + 1) * kTile, bh, prm.H);
              tma_prefetch_l2_bh(&tm_do, c * kChunkCols, (i + 1) * kTile, bh, prm.H);
            }
          }
        }
      }
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------ store threads
    // Lane 0 of warp 2 (channel 0) and, with two stage areas, lane 0 of warp
    // 3 (channel 1) take finished result tiles from their stage area (jobs
    // posted by the row warps) and write them with TMA stores: dV/dK tiles,
    // and dQ^ shares into their partial slot (a plain store for the first key
    // tile of the slot, else an L2 reduce-add after that slot's turn; once a
    // share is in L2 the slot's next turn is released). Nothing here waits on
    // the row warps beyond the job hand-off.
    const int ch = warp - 2;
    if (lane == 0 && (ch == 0 || kSplit)) {
      uint8_t* stage = kAhead ? &sm.stage[0][0] : &sm.ds[0][0];
      uint8_t* kv_area = stage + (kSplit ? 2 * kChunkBytes : 0);
      const int S = prm.nslot;
      for (int m = 0;; ++m) {
        mbar_wait(&sm.stage_full[ch], m & 1, abort_flag);
        const int type = *abort_flag ? 0 : *reinterpret_cast<volatile int*>(&sm.job_type[ch]);
        const int bh = sm.job_bh[ch], j = sm.job_j[ch], i = sm.job_i[ch];
        if (type == 0) break;    // no more jobs
        if (type == 1) {
          // dV chunk c at area chunk c, dK chunk c at area chunk NCH + c.
          for (int c = 0; c < NCH; ++c) {
            if (c * 64 < D) {
              tma_store_bh(&tm_dv, kv_area + c * kChunkBytes, c * kChunkCols, j * kTile, bh, prm.H);
              tma_store_bh(&tm_dk, kv_area + (NCH + c) * kChunkBytes, c * kChunkCols, j * kTile,
                           bh, prm.H);
            }
          }
          tma_store_commit();
          tma_store_wait_read();
          mbar_arrive(&sm.stage_free[ch]);
        } else {
          const int slot = j % S, gen = j / S;
          if (gen > 0)
            flag_wait_geq(prm.turns + (static_cast<size_t>(bh) * nqt + i) * S + slot, gen,
                          abort_flag);
          const int z = slot * prm.BH + bh;
          for (int h = 0; 32 * h < D; ++h) {
            if (gen > 0) tma_reduce_add_3d(&tm_part, stage + h * kChunkBytes, 32 * h, i * kTile, z);
            else tma_store_3d(&tm_part, stage + h * kChunkBytes, 32 * h, i * kTile, z);
          }
          tma_store_commit();
          if (j + S < prm.nkv) {
            // A later key tile adds to this slot: the share must be in L2
            // before its turn is released.
            tma_store_wait_all();
            __threadfence();
            st_release_gpu(prm.turns + (static_cast<size_t>(bh) * nqt + i) * S + slot, gen + 1);
          } else {
            tma_store_wait_read();   // only the stage must be free (the kernel's end waits for the writes)
          }
          mbar_arrive(&sm.stage_free[ch]);
        }
      }
      tma_store_wait_all();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr bool kBf = Elt<T>::kBf16;
      const uint32_t idKV = idesc_f16(kBf, 128, DP, false, true);    // dV, dK^
      const uint32_t idQ = idesc_f16(kBf, 128, DP, true, true);      // dQ^
      // Iteration t = (unit n, query tile i); key tile j of the unit.
      int n = 0, i = 0, t = 0, j = 0;
      int u = next_unit(0);
      auto issue_st = [&](int n_, int i_, int t_) {
        const int ks = n_ % KVS, qs = t_ % QS;
        mbar_wait(&sm.kq_ready, t_ & 1, abort_flag);
        tc_fence_after();
        const uint32_t idS = idesc_f16(kBf, 128, 16 * valid16(i_), false, false);
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
      };
      auto issue_grads = [&](int n_, int i_, int t_, int j_) {
        const int ks = n_ % KVS, qs = t_ % QS;
        mbar_wait(&sm.ds_full, t_ & 1, abort_flag);
        tc_fence_after();
        if (i_ == 0 && n_ > 0) {
          mbar_wait(&sm.acc_free, (n_ - 1) & 1, abort_flag);   // previous unit's dV/dK read out
          tc_fence_after();
        }
        if (t_ > 0) {
          mbar_wait(&sm.dq_free, (t_ - 1) & 1, abort_flag);    // previous dQ^ share read out
          tc_fence_after();
        }
        const int kq = valid16(i_), kkeys = valid16(j_);
        for (int kk = 0; kk < kq; ++kk) {
          // P and dS [key][query] are the A operands, read from TMEM: query
          // columns [16 kk, 16 kk + 16) sit packed in columns
          // 64 (kk / 4) + 8 (kk % 4) of the S^T and dP^T regions.
          const uint32_t pcol = 64 * (kk >> 2) + 8 * (kk & 3);
          const uint32_t acc = (i_ == 0 && kk == 0) ? 0u : 1u;
          // dV += P dO : B = dO [query][d] MN-major.
          mma_ts(tDV, tST + pcol,
                 sw128_desc(smem_u32(sm.dO[qs][0]) + kk * 2048, kChunkBytes, 1024), idKV, acc);
          // dK^ += dS Q^ : B = Q^ [query][d] MN-major.
          mma_ts(tDK, tDPT + pcol,
                 sw128_desc(smem_u32(sm.q[qs][0]) + kk * 2048, kChunkBytes, 1024), idKV, acc);
        }
        // dQ^_j = dS^T K^ : A = dS read query-major (MN-major), B = K^ [key][d]
        // MN-major. Key rows past N hold zero K^ rows and contribute nothing.
        for (int kk = 0; kk < kkeys; ++kk) {
          mma_ss(tDQ, sw128_desc(smem_u32(sm.ds[0]) + kk * 2048, kChunkBytes, 1024),
                 sw128_desc(smem_u32(sm.k[ks][0]) + kk * 2048, kChunkBytes, 1024), idQ,
                 kk > 0 ? 1u : 0u);
        }
        mma_commit(&sm.mm_done);
        mma_commit(&sm.q_empty[qs]);
        if (i_ == nqt - 1) mma_commit(&sm.kv_empty[ks]);
      };
      if (u >= 0) {
        j = u % prm.nkv;
        issue_st(n, i, t);
        while (true) {
          // The iteration after t (same unit, or the next claimed unit).
          int n2 = n, i2 = i + 1, u2 = u;
          if (i2 == nqt) {
            n2 = n + 1;
            i2 = 0;
            u2 = next_unit(n2);
          }
          const bool more = u2 >= 0;
          issue_grads(n, i, t, j);
          if (more) {
            mbar_wait(&sm.st_free, t & 1, abort_flag);
            tc_fence_after();
            issue_st(n2, i2, t + 1);
          }
          if (!more) break;
          n = n2;
          i = i2;
          u = u2;
          j = u % prm.nkv;
          ++t;
        }
      }
    }
  }
  } else {
    setmaxnreg_inc<kRegsCompute>();
    // ------------------------------------------------------------ compute warps
    // Two warpgroups (warps 4..11). For TMEM reads a thread owns row r (its
    // lane quarter wq); warpgroup g takes S/dP columns [64g, 64g + 64) and
    // every other 16-column block of the gradient tiles. Warp-per-row phases
    // (rotation, Delta) give each of the 8 warps 16 rows.
    constexpr int RW = kRowsPerWarp;
    const int cw = warp - 4;                       // compute warp 0..7
    const int g = cw >> 2;                         // warpgroup 0..1
    const int wq = warp & 3;                       // TMEM lane quarter
    const int r = wq * 32 + lane;
    const int rw0 = cw * RW;                       // first row of this warp's row slice
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const bool leader = threadIdx.x == 128;
    const float c2 = prm.c2;
    constexpr int kBlk = 4 * NCH;                  // 16-column blocks of a gradient row

    // Rotate the key tile of the n_-th unit (key tile j_) in its stage.
    auto prep_k = [&](int j_, int n_) {
      if (prm.rot_in) {
        RopeQ<NCH, RW> rope;
        load_rope_q<NCH, RW>(rope, rw0, j_ * kTile, N, prm.has_cls, D, prm.cosp, prm.sinp, lane);
        mbar_wait(&sm.kv_full[n_ % KVS], (n_ / KVS) & 1, abort_flag);
        if (prm.has_cls >= 0) apply_rope_q<T, NCH, RW>(&sm.k[n_ % KVS][0][0], rw0, D, rope, lane);
      } else {
        mbar_wait(&sm.kv_full[n_ % KVS], (n_ / KVS) & 1, abort_flag);
      }
    };
    // Prepare query tile i_ of head bh_ (key tile j_) in stage t_ % QS
    // (iteration t_): lse2 (+inf for padded rows, so their P is exactly 0),
    // rotation of Q, and Delta; then tell the MMA warp.
    // lse2 (+inf for padded rows) and Delta (when precomputed) of query row r
    // of tile i_ of head bh_, for warpgroup 0's threads; loaded an iteration
    // ahead of their use so their global latency is hidden.
    // (The raw lse is kept until use, so nothing waits on these loads early.)
    auto load_rowstats = [&](int bh_, int i_, float& l2, float& dl) {
      const size_t row = static_cast<size_t>(bh_) * N + i_ * kTile + r;
      const bool qv = (i_ * kTile + r) < N;
      l2 = qv ? __ldg(prm.lse + row) : INFINITY;
      dl = (qv && prm.delta_in != nullptr) ? __ldg(prm.delta_in + row) : 0.f;
    };
    auto prep_q = [&](int bh_, int j_, int i_, int t_, float l2, float dl) {
      const int qs_ = t_ % QS;
      const size_t row0 = static_cast<size_t>(bh_) * N;
      const int q0_ = i_ * kTile;
      const bool dpre = prm.delta_in != nullptr;
      if (g == 0) {
        sm.lse2[qs_][r] = l2 * 1.4426950408889634f;   // +inf stays +inf
        if (dpre) sm.delta[qs_][r] = dl;
      }
      // O granules of this warp's query rows (quad layout), read before the
      // tile wait so the load overlaps it.
      const int rq = lane >> 3, gl = lane & 7;
      uint4 og[NCH][RW / 4];
#pragma unroll
      for (int k = 0; k < RW / 4; ++k)
#pragma unroll
        for (int h = 0; h < NCH; ++h) {
          const int tok = q0_ + rw0 + 4 * k + rq, gg = gl + 8 * h;
          og[h][k] = (!dpre && tok < N && 8 * gg < D)
                         ? __ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(prm.o) +
                                                                (row0 + tok) * D) + gg)
                         : make_uint4(0u, 0u, 0u, 0u);
        }
      if (prm.rot_in) {
        RopeQ<NCH, RW> rope;
        load_rope_q<NCH, RW>(rope, rw0, q0_, N, prm.has_cls, D, prm.cosp, prm.sinp, lane);
        mbar_wait(&sm.q_full[qs_], (t_ / QS) & 1, abort_flag);
        if (prm.has_cls >= 0) apply_rope_q<T, NCH, RW>(&sm.q[qs_][0][0], rw0, D, rope, lane);
      } else {
        mbar_wait(&sm.q_full[qs_], (t_ / QS) & 1, abort_flag);
      }
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
          if (prm.delta_out != nullptr && j_ == 0 && q0_ + rr < N)
            prm.delta_out[row0 + q0_ + rr] = dl;
        }
      }
      fence_proxy_async_smem();
      named_bar(1, kComputeThreads);
      if (leader) mbar_arrive(&sm.kq_ready);
    };

    // Results of finished iterations leave through a shared-memory stage: the
    // row warps fill it (thread = tile row, from TMEM) and post a job to the
    // store warps, which write it out with TMA stores:
    //   job 1: dV and dK = R^T dK^ scale of a key tile, bf16 tiles
    //          [128 key][64] (128-byte swizzle): dV chunk c at stage chunk c,
    //          dK chunk c at stage chunk NCH + c;
    //   job 2: a dQ^ share * scale, f32 tiles [128 query][32] (128-byte
    //          swizzle), 32-column block h at stage chunk h;
    //   job 0: no more jobs.
    uint8_t* stage = kAhead ? &sm.stage[0][0] : &sm.ds[0][0];
    const uint32_t stb = smem_u32(stage);
#ifdef FRSA_TRACE
    unsigned trace_flags = 0;   // events of the current iteration
#endif
    const uint32_t stb_kv = stb + (kSplit ? 2 * kChunkBytes : 0);   // dV/dK area
    constexpr int kKvCh = kSplit ? 1 : 0;                             // dV/dK channel
    int jobs[2] = {0, 0};       // jobs posted so far, per channel
    int acquired[2] = {0, 0};   // jobs whose stage release has been taken
    // Wait until the store thread of channel c is done with its area (the
    // last job posted on c).
    auto stage_acquire = [&](int c) {
      if (jobs[c] == acquired[c]) return;
      mbar_wait(&sm.stage_free[c], (jobs[c] - 1) & 1, abort_flag);
      acquired[c] = jobs[c];
    };
    auto post = [&](int c, int type, int bh_, int j_, int i_) {
      fence_proxy_async_smem();
      named_bar(1, kComputeThreads);
      if (leader) {
        sm.job_type[c] = type;
        sm.job_bh[c] = bh_;
        sm.job_j[c] = j_;
        sm.job_i[c] = i_;
        mbar_arrive(&sm.stage_full[c]);
      }
      ++jobs[c];
    };

    // Results of a finished iteration (its products done, mm_done waited):
    // this key tile's dQ^ share of query tile i_, and at the unit's last
    // query tile the unit's dV and dK^ (thread = tile row for TMEM reads).
    int trace_ts = -1;   // trace builds: stamp slots of the current iteration
    auto drain = [&](int bh_, int j_, int i_, bool flush) {
      const bool unit_end = (i_ == nqt - 1);
      // kAhead: the MMA warp's next dQ^ product waits for these columns, so
      // they are read out (two 16-column blocks per thread) and released
      // before anything else. Otherwise nothing waits on them until this
      // drain is over and blocks are read one at a time.
      constexpr int kHeld = kAhead ? kBlk / 2 : 1;
      float qv[kHeld][16];
      if (kAhead && !flush) {
#pragma unroll
        for (int b = 0; b < kHeld; ++b) {
          const int c16 = g + 2 * b;
          if (c16 * 16 < DP) tmem_ld16(tDQ + lane_off + c16 * 16, qv[b]);
        }
        tmem_wait_ld();
        tc_fence_before();
        named_bar(1, kComputeThreads);
        if (leader) mbar_arrive(&sm.dq_free);
      }
      if (trace_ts >= 0) FRSA_STAMP(trace_ts + 6);
      // (without kAhead the previous dQ job was already taken before this
      // iteration's dS was stored)
      if (flush) {
        stage_acquire(0);
        stage_acquire(kKvCh);
        return;
      }
      if (unit_end) {
        stage_acquire(kKvCh);
        const int kv0 = j_ * kTile;
        const int pos = rope_pos(kv0 + r, N, prm.has_cls);
#pragma unroll 1
        for (int c16 = g; c16 < kBlk; c16 += 2) {
          if (c16 * 16 < DP) {
            float v[16], k16[16];
            tmem_ld16(tDV + lane_off + c16 * 16, v);
            tmem_ld16(tDK + lane_off + c16 * 16, k16);
            tmem_wait_ld();
            const int c = c16 >> 2;
#pragma unroll
            for (int h8 = 0; h8 < 2; ++h8) {
              const int col = c16 * 16 + 8 * h8;
              float a[8], bk[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                a[e] = v[8 * h8 + e];
                bk[e] = k16[8 * h8 + e] * prm.scale;
              }
              if (pos >= 0 && col < D) {
                const size_t t0 = static_cast<size_t>(pos) * (D >> 1) + (col >> 1);
                unrotate8(bk, __ldg(reinterpret_cast<const float4*>(prm.cosp + t0)),
                          __ldg(reinterpret_cast<const float4*>(prm.sinp + t0)));
              }
              const uint32_t gr = static_cast<uint32_t>((c16 & 3) * 2 + h8);
              sts_u4(stb_kv + c * kChunkBytes + sw128_off(r, gr), pack8<T>(a));
              sts_u4(stb_kv + (NCH + c) * kChunkBytes + sw128_off(r, gr), pack8<T>(bk));
            }
          }
        }
        tc_fence_before();
        post(kKvCh, 1, bh_, j_, i_);
        if (leader) mbar_arrive(&sm.acc_free);
      }
      stage_acquire(0);
#pragma unroll
      for (int b = 0; b < kBlk / 2; ++b) {
        const int c16 = g + 2 * b;
        if (c16 * 16 < DP) {
          float* qb = qv[kAhead ? b : 0];
          if (!kAhead) {
            tmem_ld16(tDQ + lane_off + c16 * 16, qv[0]);
            tmem_wait_ld();
          }
          const uint32_t tile = stb + (c16 >> 1) * kChunkBytes;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const uint32_t ch = static_cast<uint32_t>((c16 & 1) * 4 + e);
            sts_f4(tile + sw128_off(r, ch),
                   make_float4(qb[4 * e] * prm.scale, qb[4 * e + 1] * prm.scale,
                               qb[4 * e + 2] * prm.scale, qb[4 * e + 3] * prm.scale));
          }
        }
      }
      if (!kAhead) tc_fence_before();
      post(0, 2, bh_, j_, i_);
      if (!kAhead && leader) mbar_arrive(&sm.dq_free);
    };

    FRSA_STAMP(56);
    // The iteration sequence, as the MMA warp walks it. With kAhead, an
    // iteration's results are drained during the next iteration (after its
    // P/dS are published); one extra pass drains the last one.
    int n = 0, i = 0, t = 0;
    int u = next_unit(0);
    if (u >= 0) {
      int bh = u / prm.nkv, j = u - bh * prm.nkv;
      float nl2 = 0.f, ndl = 0.f;   // row statistics of the next query tile
      if (g == 0) load_rowstats(bh, 0, nl2, ndl);
      prep_k(j, n);
      prep_q(bh, j, 0, 0, nl2, ndl);
      int pbh = -1, pj = 0, pi = 0, pt = 0;   // iteration waiting to be drained
      bool have = true;                               // iteration t exists
      int n2 = 0, i2 = 0, u2 = -1, bh2 = 0, j2 = 0;
      bool more = false;
      while (true) {
        const int ts = (t >= 5 && t < 12) ? 8 * (t - 5) : -1;   // trace slots (trace builds)
        trace_ts = ts;
#ifdef FRSA_TRACE
        if (threadIdx.x == FRSA_STAMP_TID && blockIdx.x < 2048 && t < 1024) {
          g_trace_it[blockIdx.x * 1024 + t] = globaltimer();
          g_trace_fl[blockIdx.x * 1024 + t] = trace_flags | (static_cast<unsigned>(i) << 8);
        }
        trace_flags = 0;
#endif
        if (ts >= 0) FRSA_STAMP(ts + 0);
        if (have) {
          n2 = n;
          i2 = i + 1;
          u2 = u;
          if (i2 == nqt) {
            n2 = n + 1;
            i2 = 0;
            u2 = next_unit(n2);
          }
          more = u2 >= 0;
          bh2 = more ? u2 / prm.nkv : 0;
          j2 = more ? u2 - bh2 * prm.nkv : 0;
          if (more && g == 0) load_rowstats(bh2, i2, nl2, ndl);
          if (ts >= 0) FRSA_STAMP(ts + 1);
          // S^T, dP^T of iteration t -> registers; release the TMEM columns.
          const int qs = t % QS;
          const int ncol = 16 * valid16(i);
          mbar_wait(&sm.st_full, t & 1, abort_flag);
          tc_fence_after();
          if (ts >= 0) FRSA_STAMP(ts + 2);
          // P = exp2(S^T c2 - lse2), dS = P (dP^T - Delta), one 32-column half
          // at a time. Padded query columns have lse2 = +inf (P = 0, dS = 0);
          // padded key rows only reach dV/dK rows that are never stored and dQ
          // through zero K^ rows, so no per-element masking is needed.
          const uint32_t lbase = smem_u32(&sm.lse2[qs][g * 64]);
          const uint32_t ebase = smem_u32(&sm.delta[qs][g * 64]);
          const uint32_t dbase = smem_u32(sm.ds[g]);
          uint32_t pk[2][16], dk[2][16];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            float sv[32], dp[32];
            const bool live = 64 * g + 32 * hh < ncol;
            if (live) {
              tmem_ld32(tST + lane_off + g * 64 + 32 * hh, sv);
              tmem_ld32(tDPT + lane_off + g * 64 + 32 * hh, dp);
            }
            tmem_wait_ld();
            if (hh == 1) {
              // S^T/dP^T of iteration t are in registers: release the columns.
              tc_fence_before();
              named_bar(1, kComputeThreads);
              if (leader) mbar_arrive(&sm.st_free);
              if (ts >= 0) FRSA_STAMP(ts + 3);
              // P/dS tiles are free once the previous iteration's products
              // are done (non-kAhead: waited before this iteration began, and
              // the tiles double as the result stage: wait for the store warps).
              if (kAhead && t > 0) {
                mbar_wait(&sm.mm_done, (t - 1) & 1, abort_flag);
                tc_fence_after();
              }
              if (!kAhead) stage_acquire(0);
              if (ts >= 0) FRSA_STAMP(ts + 4);
              if (64 * g < ncol) {
                tmem_st16(tST + lane_off + g * 64, pk[0]);
                tmem_st16(tDPT + lane_off + g * 64, dk[0]);
#pragma unroll
                for (int g4 = 0; g4 < 4; ++g4) {
                  const uint32_t off = sw128_off(r, g4);
                  sts_u4(dbase + off, make_uint4(dk[0][4 * g4], dk[0][4 * g4 + 1],
                                                 dk[0][4 * g4 + 2], dk[0][4 * g4 + 3]));
                }
              }
            }
#pragma unroll
            for (int c4 = 0; c4 < 8; ++c4) {
              const float4 l4 = lds_f4(lbase + (hh * 32 + c4 * 4) * 4);
              const float4 d4 = lds_f4(ebase + (hh * 32 + c4 * 4) * 4);
              const float p0 = ex2(fmaf(sv[4 * c4 + 0], c2, -l4.x));
              const float p1 = ex2(fmaf(sv[4 * c4 + 1], c2, -l4.y));
              const float p2 = ex2(fmaf(sv[4 * c4 + 2], c2, -l4.z));
              const float p3 = ex2(fmaf(sv[4 * c4 + 3], c2, -l4.w));
              pk[hh][2 * c4] = Elt<T>::pack(p0, p1);
              pk[hh][2 * c4 + 1] = Elt<T>::pack(p2, p3);
              dk[hh][2 * c4] = Elt<T>::pack(p0 * (dp[4 * c4 + 0] - d4.x),
                                            p1 * (dp[4 * c4 + 1] - d4.y));
              dk[hh][2 * c4 + 1] = Elt<T>::pack(p2 * (dp[4 * c4 + 2] - d4.z),
                                                p3 * (dp[4 * c4 + 3] - d4.w));
            }
          }
          if (64 * g + 32 < ncol) {
            tmem_st16(tST + lane_off + g * 64 + 16, pk[1]);
            tmem_st16(tDPT + lane_off + g * 64 + 16, dk[1]);
#pragma unroll
            for (int g4 = 0; g4 < 4; ++g4) {
              const uint32_t off = sw128_off(r, 4 + g4);
              sts_u4(dbase + off, make_uint4(dk[1][4 * g4], dk[1][4 * g4 + 1], dk[1][4 * g4 + 2],
                                             dk[1][4 * g4 + 3]));
            }
          }
          tmem_wait_st();
          fence_proxy_async_smem();
          tc_fence_before();
          named_bar(1, kComputeThreads);
          if (leader) mbar_arrive(&sm.ds_full);
          if (ts >= 0) FRSA_STAMP(ts + 5);
        }
        // Drain: kAhead the previous iteration (its products finished before
        // this iteration's P/dS store; on the extra pass wait here), else this
        // one. A last pass with nothing left to drain ("flush") only takes
        // the stage back, completing the query tile the last job finished.
        if (!kAhead && have) {
          mbar_wait(&sm.mm_done, t & 1, abort_flag);
          tc_fence_after();
          pbh = bh; pj = j; pi = i; pt = t;
        } else if (kAhead && !have && pbh >= 0) {
          mbar_wait(&sm.mm_done, pt & 1, abort_flag);
          tc_fence_after();
        }
        const bool flush = !have && pbh < 0;
        if (pbh >= 0 || flush) drain(pbh, pj, pi, flush);
        if (ts >= 0) FRSA_STAMP(ts + 7);
        if (flush) break;
        if (!have) {
          pbh = -1;
          continue;
        }
        // The next query tile: with two stages its load started when the
        // products of t - 1 finished (waited above), so it has landed by now.
        if (more) {
          if (n2 != n) prep_k(j2, n2);
          prep_q(bh2, j2, i2, t + 1, nl2, ndl);
        }
        if (kAhead) {
          pbh = bh; pj = j; pi = i; pt = t;
        }
        if (!more) {
          have = false;
          if (!kAhead) pbh = -1;
          continue;
        }
        n = n2;
        i = i2;
        u = u2;
        bh = bh2;
        j = j2;
        ++t;
      }
    }
    // no more jobs (stage_acquire: with no work nothing was posted)
    if (u < 0) stage_acquire(0);
    post(0, 0, 0, 0, 0);
    if (kSplit) post(1, 0, 0, 0, 0);
    FRSA_STAMP(57);
#ifdef FRSA_TRACE
    if (threadIdx.x == FRSA_STAMP_TID && blockIdx.x < 2048) g_trace[blockIdx.x * 64 + 58] = t + 1;
#endif
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemColsBwd);
  }
}

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

// Row pre-pass of the general backward, once per row of [B*H*N, D]: the
// rotated Q^ = R(Q) and K^ = R(K) (fa_rope_full .py:201-202, 271-272; the same
// f32 arithmetic and single 16-bit rounding as the in-kernel rotation) into
// contiguous buffers, and, when `delta` is given, Delta = rowsum(dO * O)
// (fa_rope_full .py:352-357). Rotating here once, instead of once per (key
// tile, query tile) inside the main kernel, takes the rotation off its
// critical path. q and k may be strided ([B, H, N, D], element strides b, h, n).
// 8 lanes per row, one 16-byte granule each per step.
struct PrepRows {
  const void* q;
  const void* k;
  const void* o;
  const void* d_o;
  long long qs[3], ks[3];   // element strides (b, h, n) of q and k
  const float* cosp;
  const float* sinp;
  void* q_rot;
  void* k_rot;
  float* delta;             // nullptr: no Delta
  long long rows;
  int N, D, H, has_cls;
};

template <typename T>
__global__ void prep_rows_kernel(const PrepRows p) {
  const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 3;
  const int gl = threadIdx.x & 7;
  const bool valid = row < p.rows;
  const long long bh = valid ? row / p.N : 0;
  const int n = valid ? static_cast<int>(row - bh * p.N) : 0;
  const long long b = bh / p.H, h = bh - b * p.H;
  const int pos = rope_pos(n, p.N, p.has_cls);
  const T* qrow = static_cast<const T*>(p.q) + b * p.qs[0] + h * p.qs[1] + n * p.qs[2];
  const T* krow = static_cast<const T*>(p.k) + b * p.ks[0] + h * p.ks[1] + n * p.ks[2];
  uint4* qdst = reinterpret_cast<uint4*>(static_cast<T*>(p.q_rot) + row * p.D);
  uint4* kdst = reinterpret_cast<uint4*>(static_cast<T*>(p.k_rot) + row * p.D);
  float acc = 0.f;
  for (int gg = gl; 8 * gg < p.D; gg += 8) {
    if (valid) {
      float4 c = make_float4(1.f, 1.f, 1.f, 1.f), sn = make_float4(0.f, 0.f, 0.f, 0.f);
      if (pos >= 0) {
        const size_t t0 = static_cast<size_t>(pos) * (p.D >> 1);
        c = __ldg(reinterpret_cast<const float4*>(p.cosp + t0) + gg);
        sn = __ldg(reinterpret_cast<const float4*>(p.sinp + t0) + gg);
      }
      const uint4 xq = __ldg(reinterpret_cast<const uint4*>(qrow) + gg);
      const uint4 xk = __ldg(reinterpret_cast<const uint4*>(krow) + gg);
      qdst[gg] = pos >= 0 ? rotate_granule<T>(xq, c, sn) : xq;
      kdst[gg] = pos >= 0 ? rotate_granule<T>(xk, c, sn) : xk;
      if (p.delta != nullptr) {
        const uint4 a = __ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(p.o) + row * p.D) + gg);
        const uint4 d = __ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(p.d_o) + row * p.D) + gg);
        const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
        const uint32_t bw[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 x = Elt<T>::unpack(aw[e]), y = Elt<T>::unpack(bw[e]);
          acc = fmaf(x.x, y.x, fmaf(x.y, y.y, acc));
        }
      }
    }
  }
  if (p.delta != nullptr) {
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    acc += __shfl_xor_sync(0xffffffffu, acc, 4);
    if (gl == 0 && valid) p.delta[row] = acc;
  }
}

// dQ from the partial slots, after bwd_kernel: every key tile has added its
// scaled dQ^ share into its slot, so each row's dQ^ is the sum of the S
// slots in slot order, un-rotated with R^T (fa_rope_full .py:974-993) and
// stored in the I/O type. One thread per 8-element granule of a row, all S
// slots' loads in flight at once; the grid streams the slots from memory.
// Run as its own launch so that the sums do not sit on the main kernel's
// critical path (they used to be done inside it by the CTA whose key tile
// arrived last, one L2 round trip per slot).
struct DqFinal {
  const float* part;        // [nslot][rows, D] f32
  void* dq;                 // [rows, D] I/O type
  const float* cosp;
  const float* sinp;
  long long rows, slot_stride;
  int nslot, N, D, has_cls;
};

template <typename T>
__global__ void dq_finalize_kernel(const DqFinal p) {
  const int G = p.D >> 3;   // granules of a row
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long row = idx / G;
  if (row >= p.rows) return;
  const int gg = static_cast<int>(idx - row * G);
  const float4* src = reinterpret_cast<const float4*>(p.part + row * p.D) + 2 * gg;
  float4 a[kMaxDqSlots], b[kMaxDqSlots];
#pragma unroll
  for (int s = 0; s < kMaxDqSlots; ++s)
    if (s < p.nslot) {
      a[s] = __ldcs(src + s * (p.slot_stride / 4));
      b[s] = __ldcs(src + s * (p.slot_stride / 4) + 1);
    }
  float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int s = 0; s < kMaxDqSlots; ++s)
    if (s < p.nslot) {   // slot order: v starts at 0, and 0 + x == x
      v[0] += a[s].x; v[1] += a[s].y; v[2] += a[s].z; v[3] += a[s].w;
      v[4] += b[s].x; v[5] += b[s].y; v[6] += b[s].z; v[7] += b[s].w;
    }
  const int n = static_cast<int>(row % p.N);
  const int pos = rope_pos(n, p.N, p.has_cls);
  if (pos >= 0) {
    const size_t t0 = static_cast<size_t>(pos) * (p.D >> 1);
    unrotate8(v, __ldg(reinterpret_cast<const float4*>(p.cosp + t0) + gg),
              __ldg(reinterpret_cast<const float4*>(p.sinp + t0) + gg));
  }
  reinterpret_cast<uint4*>(static_cast<T*>(p.dq) + row * p.D)[gg] = pack8<T>(v);
}

}  // namespace

bool bwd_needs_workspace(const LaunchShape& s) { return !(s.N <= 2 * kTile && s.D <= 64); }

int bwd_slots(const LaunchShape& s) {
  const int nkv = (s.N + kTile - 1) / kTile;
  return nkv < kMaxDqSlots ? nkv : kMaxDqSlots;
}

size_t bwd_counter_ints(const LaunchShape& s, int nslot) {
  const size_t nqt = (static_cast<size_t>(s.N) + kTile - 1) / kTile;
  // arrival counters, slot turn counters, the claim ticket; 16-byte multiple
  return (static_cast<size_t>(s.BH) * nqt * (1 + nslot) + 1 + 3) & ~static_cast<size_t>(3);
}

namespace {

template <typename T, int NCH>
cudaError_t launch_bwd_main(const LaunchShape& s, const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                            const CUtensorMap& tm_v, const CUtensorMap& tm_do,
                            const CUtensorMap& tm_o, const CUtensorMap& tm_dk,
                            const CUtensorMap& tm_dv, const CUtensorMap& tm_part,
                            const BwdParams& p, cudaStream_t stream) {
  // The dynamic window starts 1024-aligned in practice; the slack is cut to
  // what the 227 KiB limit leaves (aligned_smem reports a misfit).
  constexpr size_t kMaxDyn = 232448;
  const size_t smem = (sizeof(BwdSmem<NCH>) + 1024 <= kMaxDyn) ? sizeof(BwdSmem<NCH>) + 1024
                                                                : kMaxDyn;
  auto kern = bwd_kernel<T, NCH>;
  cudaError_t e = set_max_dynamic_smem_once(kern, smem);
  if (e != cudaSuccess) return e;
  const long long nunits = static_cast<long long>(s.BH) * p.nkv;
  const int nsm = device_sm_count();
  const long long grid = nunits < nsm ? nunits : nsm;   // one CTA per SM (512 TMEM columns)
  kern<<<static_cast<unsigned>(grid), kBwdThreads, smem, stream>>>(tm_q, tm_k, tm_v, tm_do, tm_o,
                                                                     tm_dk, tm_dv, tm_part, p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_bwd_ordered(const LaunchShape& s, const CUtensorMap& tm_q,
                               const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                               const CUtensorMap& tm_do, const CUtensorMap& tm_o,
                               const CUtensorMap& tm_dk, const CUtensorMap& tm_dv,
                               const CUtensorMap& tm_part, const void* o,
                               const void* d_o, const float* lse, float* delta,
                               const float* cosp, const float* sinp, void* dq, void* dk, void* dv,
                               float* dq_part, int nslot, int* counters, float* delta_buf,
                               const QkRotation* rot, cudaStream_t stream) {
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
  p.dq_part = dq_part;
  p.nslot = nslot;
  p.BH = s.BH;
  p.H = s.H;
  p.N = s.N;
  p.D = s.D;
  p.nqt = (s.N + kTile - 1) / kTile;
  p.nkv = p.nqt;
  p.arrive = counters;
  p.turns = counters + static_cast<size_t>(s.BH) * p.nqt;
  p.ticket = p.turns + static_cast<size_t>(s.BH) * p.nqt * nslot;
  p.has_cls = s.has_cls;
  p.c2 = s.scale * 1.4426950408889634f;
  p.scale = s.scale;
  if (nslot < 1 || nslot > p.nkv) return cudaErrorInvalidValue;
  // Counters and the claim ticket start at zero; the partial sums need no
  // clearing (the first key tile of each slot stores its share).
  cudaError_t e = cudaMemsetAsync(counters, 0, bwd_counter_ints(s, nslot) * sizeof(int), stream);
  if (e != cudaSuccess) return e;
  p.rot_in = rot == nullptr ? 1 : 0;
  if (rot != nullptr) {
    // Q^, K^ (and Delta) once per row here, instead of per (key tile, query
    // tile) in the main kernel; the caller's maps tm_q / tm_k cover
    // rot->q_rot / rot->k_rot.
    PrepRows pr;
    pr.q = rot->q;
    pr.k = rot->k;
    pr.o = o;
    pr.d_o = d_o;
    for (int d = 0; d < 3; ++d) {
      pr.qs[d] = rot->q_strides[d];
      pr.ks[d] = rot->k_strides[d];
    }
    pr.cosp = cosp;
    pr.sinp = sinp;
    pr.q_rot = rot->q_rot;
    pr.k_rot = rot->k_rot;
    pr.delta = delta_buf;
    pr.rows = rows;
    pr.N = s.N;
    pr.D = s.D;
    pr.H = s.H;
    pr.has_cls = s.has_cls;
    const long long threads_d = rows * 8;
    if (s.bf16)
      prep_rows_kernel<__nv_bfloat16><<<static_cast<unsigned>((threads_d + 255) / 256), 256, 0,
                                        stream>>>(pr);
    else
      prep_rows_kernel<__half><<<static_cast<unsigned>((threads_d + 255) / 256), 256, 0,
                                 stream>>>(pr);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if (delta_buf != nullptr) {
      p.delta_in = delta_buf;
      p.delta_out = nullptr;   // delta_buf is the caller's delta when one was given
    }
  } else if (delta_buf != nullptr) {
    // Delta once per row here, instead of once per (key tile, query tile) in
    // the main kernel (which would also re-read O for every key tile).
    const long long threads_d = rows * 8;
    if (s.bf16)
      delta_rows_kernel<__nv_bfloat16><<<static_cast<unsigned>((threads_d + 255) / 256), 256, 0,
                                         stream>>>(static_cast<const __nv_bfloat16*>(o),
                                                   static_cast<const __nv_bfloat16*>(d_o),
                                                   delta_buf, rows, s.D);
    else
      delta_rows_kernel<__half><<<static_cast<unsigned>((threads_d + 255) / 256), 256, 0,
                                  stream>>>(static_cast<const __half*>(o),
                                            static_cast<const __half*>(d_o), delta_buf, rows, s.D);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    p.delta_in = delta_buf;
    p.delta_out = nullptr;   // delta_buf is the caller's delta when one was given
  }
  if (s.bf16)
    e = (s.D > 64) ? launch_bwd_main<__nv_bfloat16, 2>(s, tm_q, tm_k, tm_v, tm_do, tm_o, tm_dk,
                                                       tm_dv, tm_part, p, stream)
                   : launch_bwd_main<__nv_bfloat16, 1>(s, tm_q, tm_k, tm_v, tm_do, tm_o, tm_dk,
                                                       tm_dv, tm_part, p, stream);
  else
    e = (s.D > 64) ? launch_bwd_main<__half, 2>(s, tm_q, tm_k, tm_v, tm_do, tm_o, tm_dk, tm_dv,
                                                tm_part, p, stream)
                   : launch_bwd_main<__half, 1>(s, tm_q, tm_k, tm_v, tm_do, tm_o, tm_dk, tm_dv,
                                                tm_part, p, stream);
  if (e != cudaSuccess) return e;
  DqFinal f;
  f.part = dq_part;
  f.dq = dq;
  f.cosp = cosp;
  f.sinp = sinp;
  f.rows = rows;
  f.slot_stride = rows * s.D;
  f.nslot = nslot;
  f.N = s.N;
  f.D = s.D;
  f.has_cls = s.has_cls;
  const long long threads_f = rows * (s.D / 8);
  const unsigned blocks_f = static_cast<unsigned>((threads_f + 255) / 256);
  if (s.bf16)
    dq_finalize_kernel<__nv_bfloat16><<<blocks_f, 256, 0, stream>>>(f);
  else
    dq_finalize_kernel<__half><<<blocks_f, 256, 0, stream>>>(f);
  return cudaGetLastError();
}

}  // namespace frsa
