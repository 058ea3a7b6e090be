// Forward kernel: O = softmax(R(Q) R(K)^T * scale) V with 2D RoPE fused.
//
// Restates the computation of _attn_fwd (fa_rope_full .py:91-315) as a
// warp-specialised tcgen05 kernel. One CTA owns a pair of 128-query tiles of
// one (batch*head) (the whole head when N <= 256) and walks the keys in
// 128-key tiles with an online softmax in base 2. The two query tiles share
// every K/V load and K rotation.
//
//   warp 0      TMA producer: the two Q tiles once, then K/V tiles into a
//               ring of KS stages
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..3, 12..13  rotation warps: apply RoPE in shared memory to the Q
//               tiles and to every K tile as soon as TMA has landed it
//   warps 4..11 two compute warpgroups, warpgroup g owns query tile g of the
//               pair: it reads S from TMEM (thread = query row), writes P
//               (16-bit) to its shared P buffers (two when D <= 64, so the
//               next tile's softmax does not wait for this tile's P V), and
//               writes O and the log-sum-exp. O accumulates in TMEM; the
//               softmax base is raised (and O rescaled in TMEM) only when a
//               tile's maximum exceeds it by more than 2^8. The MMA issue
//               order (S_0 next, P_0 V, S_1 next, P_1 V) lets the two groups
//               run out of phase and each group's next softmax overlap its
//               own P V.
//
// TMEM columns: warpgroup g uses [256 g, 256 g + 128) for S and
// [256 g + 128, 256 g + 128 + DP) for O.
#include "frsa_internal.h"
#include "frsa_ptx.cuh"
#include "frsa_rope.cuh"

#undef FRSA_STAMP_TID
#define FRSA_STAMP_TID 128  // first compute thread of this kernel

namespace frsa {

namespace {

constexpr int kFwdCompute = 256;                // two warpgroups
constexpr int kFwdThreads = 128 + kFwdCompute + 64;  // + producer, MMA, four rotation warps
constexpr uint32_t kTmemColsFwd = 512;
constexpr float kFwdSlack = 8.f;   // log2 headroom of the softmax base

template <int NCH>
struct FwdSmem {
  static constexpr int KS = (NCH == 1) ? 2 : 1;  // K/V ring stages
  static constexpr int PB = (NCH == 1) ? 2 : 1;  // P buffers per warpgroup
  uint8_t q[2][NCH][kChunkBytes];      // query tile of warpgroup g
  uint8_t k[KS][NCH][kChunkBytes];     // key ring
  uint8_t v[KS][NCH][kChunkBytes];     // value ring
  uint8_t p[2][PB][2][kChunkBytes];    // P tiles of warpgroup g: [128 q][128 kv], two chunks
  uint64_t q_full[2];
  uint64_t q_ready;
  uint64_t kv_full[KS];
  uint64_t kv_empty[KS];
  uint64_t k_ready[KS];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_full[2][PB];              // P V of a tile using P buffer b has completed
  uint32_t tmem_base;
  int abort_flag;
};

struct FwdParams {
  const float* cosp;
  const float* sinp;
  void* o;
  float* lse;
  int H, N, D, nqt, npair, nkv, has_cls;
  float c2;  // scale * log2(e)
};

template <typename T, int NCH>
__global__ void __launch_bounds__(kFwdThreads, 1)
    fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
               const __grid_constant__ CUtensorMap tm_v, const FwdParams prm) {
  using Sm = FwdSmem<NCH>;
  constexpr int KS = Sm::KS;
  constexpr int PB = Sm::PB;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Sm* smp = aligned_smem<Sm>(smem_raw);
  if (smp == nullptr) return;
  Sm& sm = *smp;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bh = blockIdx.x / prm.npair;
  const int pr = blockIdx.x - bh * prm.npair;
  const int N = prm.N, D = prm.D;
  const int DP = (D + 15) & ~15;   // MMA N for P V
  const int ksteps = DP >> 4;      // MMA K steps over the head dim
  const int nact = min(2, prm.nqt - 2 * pr);  // active query tiles in this pair (1 or 2)
  volatile int* abort_flag = &sm.abort_flag;

  if (threadIdx.x == 0) {
    sm.abort_flag = 0;
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.q_full[s], 1);
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.p_full[s], 1);
      for (int b = 0; b < Sm::PB; ++b) mbar_init(&sm.o_full[s][b], 1);
    }
    mbar_init(&sm.q_ready, 1);
    for (int s = 0; s < KS; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
      mbar_init(&sm.k_ready[s], 1);
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

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      for (int g = 0; g < nact; ++g) {
        mbar_arrive_expect_tx(&sm.q_full[g], NCH * kChunkBytes);
        for (int c = 0; c < NCH; ++c)
          tma_load_bh(sm.q[g][c], &tm_q, &sm.q_full[g], c * kChunkCols, (2 * pr + g) * kTile, bh, prm.H);
      }
      for (int j = 0; j < prm.nkv; ++j) {
        const int s = j % KS;
        mbar_wait(&sm.kv_empty[s], ((j / KS) & 1) ^ 1, abort_flag);
        mbar_arrive_expect_tx(&sm.kv_full[s], 2 * NCH * kChunkBytes);
        for (int c = 0; c < NCH; ++c) {
          tma_load_bh(sm.k[s][c], &tm_k, &sm.kv_full[s], c * kChunkCols, j * kTile, bh, prm.H);
          tma_load_bh(sm.v[s][c], &tm_v, &sm.kv_full[s], c * kChunkCols, j * kTile, bh, prm.H);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr bool kBf = Elt<T>::kBf16;
      const uint32_t idS = idesc_f16(kBf, 128, 128, false, false);
      const uint32_t idO = idesc_f16(kBf, 128, DP, false, true);
      // S_g = Q^_g K^T : A = Q^ [q][d] K-major, B = K^ [kv][d] K-major.
      auto issue_s = [&](int g, int j) {
        const int s = j % KS;
        const uint32_t tS = tmem + 256 * g;
        for (int ks = 0; ks < ksteps; ++ks) {
          const int c = ks >> 2;
          const uint32_t koff = (ks & 3) * 32;
          mma_ss(tS, sw128_desc(smem_u32(sm.q[g][c]) + koff, 16, 1024),
                 sw128_desc(smem_u32(sm.k[s][c]) + koff, 16, 1024), idS, ks > 0);
        }
        mma_commit(&sm.s_full[g]);
      };
      // O_g += P_g V : A = P [q][kv] K-major, B = V [kv][d] MN-major. O
      // accumulates over the key tiles in TMEM.
      auto issue_pv = [&](int g, int j) {
        const int s = j % KS, b = j % PB;
        const uint32_t tO = tmem + 256 * g + 128;
        for (int ks = 0; ks < kTile / 16; ++ks) {
          mma_ss(tO, sw128_desc(smem_u32(sm.p[g][b][ks >> 2]) + (ks & 3) * 32, 16, 1024),
                 sw128_desc(smem_u32(sm.v[s][0]) + ks * 2048, kChunkBytes, 1024), idO,
                 (j | ks) > 0);
        }
        mma_commit(&sm.o_full[g][b]);
      };
      mbar_wait(&sm.q_ready, 0, abort_flag);
      mbar_wait(&sm.k_ready[0], 0, abort_flag);
      tc_fence_after();
      for (int g = 0; g < nact; ++g) issue_s(g, 0);
      for (int j = 0; j < prm.nkv; ++j) {
        const bool more = j + 1 < prm.nkv;
        if (KS == 1) {
          // One K/V stage: tile j+1 can only land after every P V of tile j.
          for (int g = 0; g < nact; ++g) {
            mbar_wait(&sm.p_full[g], j & 1, abort_flag);
            tc_fence_after();
            issue_pv(g, j);
          }
          mma_commit(&sm.kv_empty[0]);
          if (more) {
            mbar_wait(&sm.k_ready[0], (j + 1) & 1, abort_flag);
            tc_fence_after();
            for (int g = 0; g < nact; ++g) issue_s(g, j + 1);
          }
        } else {
          // S_g of tile j+1 goes ahead of P_g V of tile j (P is in shared
          // memory, so S may overwrite the scores as soon as the softmax has
          // published P): the group's next softmax overlaps this P V.
          for (int g = 0; g < nact; ++g) {
            mbar_wait(&sm.p_full[g], j & 1, abort_flag);
            tc_fence_after();
            if (more) {
              if (g == 0) {
                mbar_wait(&sm.k_ready[(j + 1) % KS], ((j + 1) / KS) & 1, abort_flag);
                tc_fence_after();
              }
              issue_s(g, j + 1);
            }
            issue_pv(g, j);
          }
          mma_commit(&sm.kv_empty[j % KS]);
        }
      }
    }
  } else if (warp < 4 || warp >= 12) {
    // ------------------------------------------------------------ rotation warps
    // Warps 2, 3, 12, 13; each rotates a quarter of every tile, 16 rows at a
    // time with the table values loaded before the tile's TMA wait.
    const int rwp = warp < 4 ? warp - 2 : warp - 10;
    auto rotate_tile = [&](uint8_t* tile, int tok0, uint64_t* full, uint32_t parity) {
#pragma unroll 1
      for (int blk = 0; blk < 2; ++blk) {
        const int r0 = rwp * 32 + blk * 16;
        RopeQ<NCH, 16> rope;
        load_rope_q<NCH, 16>(rope, r0, tok0, N, prm.has_cls, D, prm.cosp, prm.sinp, lane);
        if (blk == 0) mbar_wait(full, parity, abort_flag);
        if (prm.has_cls >= 0) apply_rope_q<T, NCH, 16>(tile, r0, D, rope, lane);
      }
    };
    for (int g = 0; g < nact; ++g)
      rotate_tile(&sm.q[g][0][0], (2 * pr + g) * kTile, &sm.q_full[g], 0);
    fence_proxy_async_smem();
    named_bar(1, 128);
    if (threadIdx.x == 64) mbar_arrive(&sm.q_ready);
    for (int j = 0; j < prm.nkv; ++j) {
      const int s = j % KS;
      rotate_tile(&sm.k[s][0][0], j * kTile, &sm.kv_full[s], (j / KS) & 1);
      fence_proxy_async_smem();
      named_bar(1, 128);
      if (threadIdx.x == 64) mbar_arrive(&sm.k_ready[s]);
    }
  } else {
    // ------------------------------------------------------------ compute warpgroups
    const int cw = warp - 4;
    const int g = cw >> 2;                 // warpgroup = query tile of the pair
    const int wq = warp & 3;               // TMEM lane quarter
    const int r = wq * 32 + lane;          // query row in the tile == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const bool leader = threadIdx.x == 128 + 128 * g;
    const int q0 = (2 * pr + g) * kTile;
    const int qrow = q0 + r;
    const float c2 = prm.c2;
    const uint32_t tS = tmem + 256 * g + lane_off;
    const uint32_t tO = tmem + 256 * g + 128 + lane_off;

    if (g < nact) {
      float m2 = -INFINITY, l = 0.f;
      const bool row_valid = qrow < N;
      // A warp whose 32 query rows are all padding skips the softmax math: its
      // P rows only ever reach O rows that are not stored.
      const bool warp_active = (q0 + wq * 32) < N;

      FRSA_STAMP(3);

      for (int j = 0; j < prm.nkv; ++j) {
        const int kv0 = j * kTile;
        const int nvalid = min(kTile, N - kv0);
        const int b = j % PB;
        mbar_wait(&sm.s_full[g], j & 1, abort_flag);
        // P buffer b was last read by the P V of tile j - PB.
        if (j >= PB) mbar_wait(&sm.o_full[g][b], ((j - PB) / PB) & 1, abort_flag);
        tc_fence_after();
        if (j < 12) FRSA_STAMP(8 + 2 * j);
        if (warp_active) {
          // pass 1: row max over the valid columns
          float mx = -INFINITY;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float sv[2][32];
            tmem_ld32(tS + h * 64, sv[0]);
            tmem_ld32(tS + h * 64 + 32, sv[1]);
            tmem_wait_ld();
#pragma unroll
            for (int u = 0; u < 2; ++u)
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (h * 64 + u * 32 + i < nvalid) mx = fmaxf(mx, sv[u][i]);
          }
          // The exponent base m2 is raised only when a tile's maximum exceeds
          // it by more than kFwdSlack (log2 units; P stays <= 2^kFwdSlack):
          // then l and the O accumulated in TMEM so far are rescaled, after
          // the previous P V has completed.
          const bool up = mx * c2 > m2 + kFwdSlack;
          if (__any_sync(0xffffffffu, up)) {
            const float m_new = up ? mx * c2 : m2;
            const float alpha = ex2(m2 - m_new);   // 0 on the first tile
            l *= alpha;
            if (j > 0) {
              const int pj = j - 1;
              mbar_wait(&sm.o_full[g][pj % PB], (pj / PB) & 1, abort_flag);
              tc_fence_after();
#pragma unroll
              for (int c16 = 0; c16 < 4 * NCH; ++c16) {
                if (c16 * 16 < DP) {
                  float ov[16];
                  tmem_ld16(tO + c16 * 16, ov);
                  tmem_wait_ld();
                  uint32_t w[16];
#pragma unroll
                  for (int i = 0; i < 16; ++i) w[i] = __float_as_uint(ov[i] * alpha);
                  tmem_st16(tO + c16 * 16, w);
                }
              }
              tmem_wait_st();
            }
            m2 = m_new;
          }
          // pass 2: P = exp2(S c2 - m2), row sum, 16-bit P into buffer b
          float sum = 0.f;
          const uint32_t pb0 = smem_u32(sm.p[g][b][0]);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float sv[2][32];
            tmem_ld32(tS + h * 64, sv[0]);
            tmem_ld32(tS + h * 64 + 32, sv[1]);
            tmem_wait_ld();
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int cbase = h * 64 + u * 32;
              if (cbase + 32 <= nvalid) {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                  sv[u][i] = ex2(fmaf(sv[u][i], c2, -m2));
                  sum += sv[u][i];
                }
              } else if (cbase < nvalid) {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                  sv[u][i] = (cbase + i < nvalid) ? ex2(fmaf(sv[u][i], c2, -m2)) : 0.f;
                  sum += sv[u][i];
                }
              } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) sv[u][i] = 0.f;
              }
#pragma unroll
              for (int g4 = 0; g4 < 4; ++g4) {
                uint4 w;
                w.x = Elt<T>::pack(sv[u][g4 * 8 + 0], sv[u][g4 * 8 + 1]);
                w.y = Elt<T>::pack(sv[u][g4 * 8 + 2], sv[u][g4 * 8 + 3]);
                w.z = Elt<T>::pack(sv[u][g4 * 8 + 4], sv[u][g4 * 8 + 5]);
                w.w = Elt<T>::pack(sv[u][g4 * 8 + 6], sv[u][g4 * 8 + 7]);
                sts_u4(pb0 + h * kChunkBytes + sw128_off(r, u * 4 + g4), w);
              }
            }
          }
          l += sum;
        }
        fence_proxy_async_smem();
        tc_fence_before();
        named_bar(2 + g, 128);
        if (leader) mbar_arrive(&sm.p_full[g]);
        if (j < 12) FRSA_STAMP(9 + 2 * j);
      }
      FRSA_STAMP(7);

      // epilogue: lse = (m + log2 l) ln 2 and O / l, read from TMEM once the
      // last P V has completed and written through this group's first P
      // buffer (free) as an f32 staging area, one 64-column block at a time,
      // by warp-per-row coalesced stores.
      if (row_valid)
        prm.lse[static_cast<size_t>(bh) * N + qrow] = (m2 + lg2(l)) * 0.69314718055994531f;
      {
        const int lj = prm.nkv - 1;
        mbar_wait(&sm.o_full[g][lj % PB], (lj / PB) & 1, abort_flag);
        tc_fence_after();
      }
      const float inv_l = warp_active ? 1.f / l : 0.f;
      uint8_t* stage = &sm.p[g][0][0][0];
      T* o_head = reinterpret_cast<T*>(prm.o) + static_cast<size_t>(bh) * N * D;
#pragma unroll
      for (int blk = 0; blk < NCH; ++blk) {
        if (blk * 64 < D) {
#pragma unroll
          for (int c16 = 0; c16 < 4; ++c16) {
            float v[16];
            if (warp_active) {
              tmem_ld16(tO + blk * 64 + c16 * 16, v);
              tmem_wait_ld();
            }
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] = warp_active ? v[e] * inv_l : 0.f;
            stage_write16<1>(stage, r, c16, v);
          }
          named_bar(2 + g, 128);
          drain_block_q<T, 32>(stage, wq * 32, q0, N, D, blk, o_head, lane);
          named_bar(2 + g, 128);
        }
      }
      FRSA_STAMP(30);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemColsFwd);
  }
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
  const size_t smem = sizeof(FwdSmem<NCH>) + 1024;
  auto kern = fwd_kernel<T, NCH>;
  cudaError_t e = set_max_dynamic_smem_once(kern, smem);
  if (e != cudaSuccess) return e;
  const long long units = static_cast<long long>(s.BH) * p.npair;
  kern<<<static_cast<unsigned>(units), kFwdThreads, smem, stream>>>(tm_q, tm_k, tm_v, p);
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
