// Persistent forward kernel for short sequences: N <= 256 and D <= 64 (the
// ViT-S/B shapes, N = 197). Same computation as fwd_kernel
// (fa_rope_full .py:91-315), organised so that consecutive heads overlap:
//
//   - the CTA is persistent (one per SM) and walks heads bh = blockIdx.x,
//     blockIdx.x + gridDim.x, ...; Q and K/V tiles are double-buffered per
//     head, so the next head loads and rotates while this one computes;
//   - the scores of a query tile against all keys (N <= 256) are one
//     tensor-core product into tensor memory, so the softmax runs once per
//     head with the exact row maximum: no running rescale, and O is read from
//     tensor memory once, at the end;
//   - P never touches shared memory: the softmax writes it (16-bit, two per
//     32-bit column) over S in tensor memory and the P V product takes its A
//     operand from there;
//   - the RoPE tables (identical for every head) are two shared "table tiles"
//     of packed f16 (cos, sin) pairs filled once per CTA;
//   - Q and K tiles are released as soon as the score products are done and V
//     after the last P V, so loads run up to two heads ahead; O rows are
//     stored straight from registers.
//
// Roles: warp 0 TMA producer, warp 1 TMEM allocator + MMA issuer, warps 2..3
// and 12..15 rotate Q and K tiles in place, warps 4..11 two softmax
// warpgroups (warpgroup g = query tile g; thread = query row = TMEM lane).
//
// TMEM columns: warpgroup g uses [256 g, 256 g + 256) for S over all keys; P
// is packed into its first 128 columns and O = P V lands in
// [256 g + 128, 256 g + 192), over scores already consumed.
#include "frsa_internal.h"
#include "frsa_ptx.cuh"
#include "frsa_rope.cuh"

#undef FRSA_STAMP_TID
#define FRSA_STAMP_TID 128

namespace frsa {

namespace {

constexpr int kFsThreads = 512;
constexpr int kFsRotThreads = 192;   // warps 2-3 and 12-15
// Registers per thread after the per-warpgroup split (launch: 128 each, 512
// threads): warpgroups 0 and 3 (producer, MMA, rotation) 88, the two softmax
// warpgroups 168: 88 + 88 + 2 x 168 = 4 x 128.
constexpr uint32_t kFsRegsAux = 88, kFsRegsSoft = 168;

struct FsSmem {
  uint8_t q[2][2][kChunkBytes];    // [head stage][query tile]
  uint8_t k[2][2][kChunkBytes];    // [head stage][key tile]; the two tiles of a stage are
  uint8_t v[2][2][kChunkBytes];    // contiguous, so one descriptor spans all 256 keys
  uint8_t tab[2][kChunkBytes];     // f16 (cos, sin) table tiles of token tiles 0, 1
  uint64_t q_full[2], q_ready[2], q_empty[2];
  uint64_t k_full[2], k_ready[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2], p_hi[2], p_full[2], o_full[2], o_free[2];
  uint32_t tmem_base;
  int abort_flag;
};

struct FsParams {
  const float* cosp;
  const float* sinp;
  void* o;
  float* lse;
  int BH, H, N, D, nqt, nkv, has_cls;
  float c2;
};

template <typename T>
__global__ void __launch_bounds__(kFsThreads, 1)
    fwd_small_kernel(const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const FsParams prm) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  FsSmem* smp = aligned_smem<FsSmem>(smem_raw);
  if (smp == nullptr) return;
  FsSmem& sm = *smp;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int N = prm.N, D = prm.D;
  const int DP = (D + 15) & ~15;
  const int ksteps = DP >> 4;
  const int nk16 = (N + 15) & ~15;   // key columns the products compute
  // P of keys [128, nk16) fits past the scores (nk16 + (nk16 - 128) / 2 <= 256).
  const bool split = nk16 > kTile && nk16 <= 208;
  const int nqt = prm.nqt, nkv = prm.nkv;
  volatile int* abort_flag = &sm.abort_flag;

  if (threadIdx.x == 0) {
    sm.abort_flag = 0;
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.q_full[s], 1);
      mbar_init(&sm.q_ready[s], 1);
      mbar_init(&sm.q_empty[s], 1);
      mbar_init(&sm.k_full[s], 1);
      mbar_init(&sm.k_ready[s], 1);
      mbar_init(&sm.k_empty[s], 1);
      mbar_init(&sm.v_full[s], 1);
      mbar_init(&sm.v_empty[s], 1);
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.p_hi[s], 4);     // one arrival per softmax warp
      mbar_init(&sm.p_full[s], 4);
      mbar_init(&sm.o_full[s], 1);
      mbar_init(&sm.o_free[s], 4);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp < 4 || warp >= 12) {
  setmaxnreg_dec<kFsRegsAux>();
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      int hl = 0;
      for (int bh = blockIdx.x; bh < prm.BH; bh += gridDim.x, ++hl) {
        const int st = hl & 1;
        const uint32_t fp = ((hl >> 1) & 1) ^ 1;
        mbar_wait(&sm.q_empty[st], fp, abort_flag);
        mbar_arrive_expect_tx(&sm.q_full[st], nqt * kChunkBytes);
        for (int g = 0; g < nqt; ++g)
          tma_load_bh(sm.q[st][g], &tm_q, &sm.q_full[st], 0, g * kTile, bh, prm.H);
        // Q and K are released when the score products of their head are
        // done, V after its last P V: loads run up to two heads ahead.
        mbar_wait(&sm.k_empty[st], fp, abort_flag);
        mbar_arrive_expect_tx(&sm.k_full[st], nkv * kChunkBytes);
        for (int j = 0; j < nkv; ++j)
          tma_load_bh(sm.k[st][j], &tm_k, &sm.k_full[st], 0, j * kTile, bh, prm.H);
        mbar_wait(&sm.v_empty[st], fp, abort_flag);
        mbar_arrive_expect_tx(&sm.v_full[st], nkv * kChunkBytes);
        for (int j = 0; j < nkv; ++j)
          tma_load_bh(sm.v[st][j], &tm_v, &sm.v_full[st], 0, j * kTile, bh, prm.H);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr bool kBf = Elt<T>::kBf16;
      const uint32_t idS = idesc_f16(kBf, 128, nk16, false, false);
      const uint32_t idO = idesc_f16(kBf, 128, DP, false, true);
      const int pvsteps = nk16 >> 4;
      // S_g = Q_g K^T over all keys at once (N = nk16 <= 256): columns
      // [256 g, 256 g + nk16). It overwrites O_g of the previous head, so it
      // waits until the softmax group has read that.
      auto issue_s = [&](int g, int hl) {
        const int st = hl & 1;
        if (hl > 0) {
          mbar_wait(&sm.o_free[g], (hl - 1) & 1, abort_flag);
          tc_fence_after();
        }
#pragma unroll 1
        for (int ks = 0; ks < ksteps; ++ks) {
          const uint32_t koff = ks * 32;
          mma_ss(tmem + 256 * g, sw128_desc(smem_u32(sm.q[st][g]) + koff, 16, 1024),
                 sw128_desc(smem_u32(sm.k[st][0]) + koff, 16, 1024), idS, ks > 0);
        }
        mma_commit(&sm.s_full[g]);
        if (g == nqt - 1) {
          mma_commit(&sm.q_empty[st]);
          mma_commit(&sm.k_empty[st]);
        }
      };
      // O_g = P_g V : A = P (16-bit, packed over the first nk16 / 2 columns
      // of S_g), B = V [key][d] MN-major; O_g lands in columns
      // [256 g + 128, +DP), which held scores the softmax has consumed. The
      // last product of a head releases its K/V stage.
      auto issue_pv = [&](int g, int hl) {
        const int st = hl & 1;
        if (g == 0) mbar_wait(&sm.v_full[st], (hl >> 1) & 1, abort_flag);
        int ks0 = 0;
        if (split) {
          // Keys [128, nk16) first: their P sits past the scores.
          mbar_wait(&sm.p_hi[g], hl & 1, abort_flag);
          tc_fence_after();
#pragma unroll 1
          for (int ks = 8; ks < pvsteps; ++ks)
            mma_ts(tmem + 256 * g + 128, tmem + 256 * g + nk16 + (ks - 8) * 8,
                   sw128_desc(smem_u32(sm.v[st][0]) + ks * 2048, kChunkBytes, 1024), idO,
                   ks > 8);
          ks0 = 1;
        }
        mbar_wait(&sm.p_full[g], hl & 1, abort_flag);
        tc_fence_after();
        const int kend = split ? 8 : pvsteps;
#pragma unroll 1
        for (int ks = 0; ks < kend; ++ks)
          mma_ts(tmem + 256 * g + 128, tmem + 256 * g + ks * 8,
                 sw128_desc(smem_u32(sm.v[st][0]) + ks * 2048, kChunkBytes, 1024), idO,
                 ks + ks0 > 0);
        mma_commit(&sm.o_full[g]);
        if (g == nqt - 1) mma_commit(&sm.v_empty[st]);
      };
      // The two query tiles run half a head apart, so that one group's
      // softmax overlaps the other group's products:
      //   S(h,0)  PV(h-1,1)  S(h,1)  PV(h,0)  S(h+1,0)  PV(h,1) ...
      int hl = 0;
      for (int bh = blockIdx.x; bh < prm.BH; bh += gridDim.x, ++hl) {
        const uint32_t hp = (hl >> 1) & 1;
        mbar_wait(&sm.q_ready[hl & 1], hp, abort_flag);
        mbar_wait(&sm.k_ready[hl & 1], hp, abort_flag);
        tc_fence_after();
        issue_s(0, hl);
        if (nqt > 1) {
          if (hl > 0) issue_pv(1, hl - 1);
          issue_s(1, hl);
        }
        issue_pv(0, hl);
      }
      if (nqt > 1 && hl > 0) issue_pv(1, hl - 1);
    }
  } else {
    // ------------------------------------------------------------ rotation warps
    // 192 threads; thread t rotates token rows t, t + 192, ... of a stage.
    const int t = warp < 4 ? threadIdx.x - 64 : threadIdx.x - 320;
    for (int rr = t; rr < 2 * kTile; rr += kFsRotThreads)
      store_tabrow(smem_u32(sm.tab[rr >> 7]), rr & (kTile - 1), rope_pos(rr, N, prm.has_cls), D,
                   prm.cosp, prm.sinp);
    named_bar(1, kFsRotThreads);
    int hl = 0;
    for (int bh = blockIdx.x; bh < prm.BH; bh += gridDim.x, ++hl) {
      const int st = hl & 1;
      const uint32_t hp = (hl >> 1) & 1;
      // Rows past N were zero-filled by the loads and stay zero.
      mbar_wait(&sm.q_full[st], hp, abort_flag);
      for (int rr = t; prm.has_cls >= 0 && rr < N; rr += kFsRotThreads)
        rotate_row_t<T, 4>(smem_u32(sm.q[st][rr >> 7]), smem_u32(sm.tab[rr >> 7]), rr & (kTile - 1),
                           D);
      fence_proxy_async_smem();
      named_bar(1, kFsRotThreads);
      if (t == 0) mbar_arrive(&sm.q_ready[st]);
      mbar_wait(&sm.k_full[st], hp, abort_flag);
      for (int rr = t; prm.has_cls >= 0 && rr < N; rr += kFsRotThreads)
        rotate_row_t<T, 4>(smem_u32(sm.k[st][rr >> 7]), smem_u32(sm.tab[rr >> 7]), rr & (kTile - 1),
                           D);
      fence_proxy_async_smem();
      named_bar(1, kFsRotThreads);
      if (t == 0) mbar_arrive(&sm.k_ready[st]);
    }
  }
  } else {
    setmaxnreg_inc<kFsRegsSoft>();
    // ------------------------------------------------------------ softmax warpgroups
    // One pass per head: the whole score row is in TMEM, so the maximum is
    // exact and nothing is rescaled.
    const int cw = warp - 4;
    const int g = cw >> 2;
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const int q0 = g * kTile;
    const int qrow = q0 + r;
    const float c2 = prm.c2;
    const uint32_t tS = tmem + 256 * g + lane_off;
    const uint32_t tO = tmem + 256 * g + 128 + lane_off;
    const int npair = (nk16 + 63) >> 6;   // 64-column steps over the computed keys
    // A warp whose 32 query rows are all padding skips the softmax math: its P
    // rows only ever reach O rows that are not stored.
    const bool warp_active = (q0 + wq * 32) < N;
#ifdef FRSA_TRACE
    int tr_i = 0;
    const bool tr_lead = (threadIdx.x & 127) == 0;
#define FS_TR(ev)                                                                   \
  do {                                                                              \
    if (tr_lead && blockIdx.x < 2048 && tr_i < 512) {                               \
      g_trace_it[blockIdx.x * 1024 + g * 512 + tr_i] = globaltimer();               \
      g_trace_fl[blockIdx.x * 1024 + g * 512 + tr_i] = (ev);                        \
      ++tr_i;                                                                       \
    }                                                                               \
  } while (0)
#else
#define FS_TR(ev) \
  do {            \
  } while (0)
#endif
    if (g < nqt) {
      int hl = 0;
      for (int bh = blockIdx.x; bh < prm.BH; bh += gridDim.x, ++hl) {
        FS_TR(0);
        mbar_wait(&sm.s_full[g], hl & 1, abort_flag);
        tc_fence_after();
        FS_TR(1);
        float m2 = 0.f, l = 1.f;
        if (warp_active) {
          float mxp[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll 1
          for (int h = 0; h < npair; ++h) {
            float sv[2][32];
            tmem_ld32(tS + h * 64, sv[0]);
            tmem_ld32(tS + h * 64 + 32, sv[1]);
            tmem_wait_ld();
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int cbase = h * 64 + u * 32;
              if (cbase + 32 <= N) {
#pragma unroll
                for (int i = 0; i < 32; ++i) mxp[i & 3] = fmaxf(mxp[i & 3], sv[u][i]);
              } else {
#pragma unroll
                for (int i = 0; i < 32; ++i)
                  if (cbase + i < N) mxp[i & 3] = fmaxf(mxp[i & 3], sv[u][i]);
              }
            }
          }
          m2 = fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])) * c2;
          FS_TR(2);
          float sp[4] = {0.f, 0.f, 0.f, 0.f};
          // Split: the 64-key steps past key 128 go first and their P goes to
          // columns [nk16, ...), past the scores, so P V can start on them
          // while keys [0, 128) are processed (then published by p_full).
#pragma unroll 1
          for (int hh = 0; hh < npair; ++hh) {
            const int h = split ? (hh < npair - 2 ? hh + 2 : hh - (npair - 2)) : hh;
            float sv[2][32];
            tmem_ld32(tS + h * 64, sv[0]);
            tmem_ld32(tS + h * 64 + 32, sv[1]);
            tmem_wait_ld();
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int cbase = h * 64 + u * 32;
              if (split && cbase >= nk16) continue;
              uint32_t pk[16];
              if (cbase + 32 <= N) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  const float a = ex2(fmaf(sv[u][2 * i], c2, -m2));
                  const float b = ex2(fmaf(sv[u][2 * i + 1], c2, -m2));
                  sp[i & 3] += a + b;
                  pk[i] = Elt<T>::pack(a, b);
                }
              } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  const float a = (cbase + 2 * i < N) ? ex2(fmaf(sv[u][2 * i], c2, -m2)) : 0.f;
                  const float b =
                      (cbase + 2 * i + 1 < N) ? ex2(fmaf(sv[u][2 * i + 1], c2, -m2)) : 0.f;
                  sp[i & 3] += a + b;
                  pk[i] = Elt<T>::pack(a, b);
                }
              }
              // P columns [cbase, cbase + 32) -> packed TMEM columns from
              // cbase / 2 (already read: the write front trails the read front),
              // or from nk16 + (cbase - 128) / 2 for the split's high keys.
              tmem_st16(tS + (split && cbase >= kTile ? nk16 + (cbase - kTile) / 2 : cbase / 2),
                        pk);
            }
            if (split && hh == npair - 3) {
              tmem_wait_st();
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&sm.p_hi[g]);
            }
          }
          tmem_wait_st();
          l = (sp[0] + sp[1]) + (sp[2] + sp[3]);
        } else if (split) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.p_hi[g]);
        }
        tc_fence_before();
        // Each warp publishes its own rows (no cross-warp barrier here).
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.p_full[g]);
        FS_TR(3);

        if (qrow < N)
          prm.lse[static_cast<size_t>(bh) * N + qrow] = (m2 + lg2(l)) * 0.69314718055994531f;
        mbar_wait(&sm.o_full[g], hl & 1, abort_flag);
        tc_fence_after();
        FS_TR(4);
        // Epilogue: O / l as 16-bit rows, stored straight from registers
        // (each thread writes its whole 2 D-byte row).
        if (warp_active) {
          const float inv_l = 1.f / l;
          T* orow = static_cast<T*>(prm.o) + (static_cast<size_t>(bh) * N + qrow) * D;
#pragma unroll
          for (int c32 = 0; c32 < 2; ++c32) {
            if (c32 * 32 < DP) {
              float ov[32];
              tmem_ld32(tO + c32 * 32, ov);
              tmem_wait_ld();
              if (qrow < N) {
#pragma unroll
                for (int gg = 0; gg < 4; ++gg) {
                  if (8 * (4 * c32 + gg) < D) {
                    float u[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) u[e] = ov[8 * gg + e] * inv_l;
                    *reinterpret_cast<uint4*>(orow + 8 * (4 * c32 + gg)) = pack8<T>(u);
                  }
                }
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.o_free[g]);
        FS_TR(5);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <typename T>
cudaError_t launch_fwd_small_t(const LaunchShape& s, const CUtensorMap& tm_q,
                               const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                               const float* cosp, const float* sinp, void* o, float* lse,
                               cudaStream_t stream) {
  FsParams p;
  p.o = o;
  p.cosp = cosp;
  p.sinp = sinp;
  p.lse = lse;
  p.BH = s.BH;
  p.H = s.H;
  p.N = s.N;
  p.D = s.D;
  p.nqt = (s.N + kTile - 1) / kTile;
  p.nkv = p.nqt;
  p.has_cls = s.has_cls;
  p.c2 = s.scale * 1.4426950408889634f;
  // The dynamic window starts 1024-aligned in practice; 256 bytes of slack keep
  // the ~224 KiB layout under the 227 KiB limit (aligned_smem reports a misfit).
  const size_t smem = sizeof(FsSmem) + 256;
  auto kern = fwd_small_kernel<T>;
  cudaError_t e = set_max_dynamic_smem_once(kern, smem);
  if (e != cudaSuccess) return e;
  const int nsm = device_sm_count();
  const int grid = s.BH < nsm ? s.BH : nsm;
  kern<<<grid, kFsThreads, smem, stream>>>(tm_q, tm_k, tm_v, p);
  return cudaGetLastError();
}

}  // namespace

bool fwd_small_applies(const LaunchShape& s) { return s.N <= 2 * kTile && s.D <= 64; }

cudaError_t launch_fwd_small(const LaunchShape& s, const CUtensorMap& tm_q,
                             const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                             const float* cosp, const float* sinp, void* o, float* lse,
                             cudaStream_t stream) {
  return s.bf16 ? launch_fwd_small_t<__nv_bfloat16>(s, tm_q, tm_k, tm_v, cosp, sinp, o, lse,
                                                    stream)
                : launch_fwd_small_t<__half>(s, tm_q, tm_k, tm_v, cosp, sinp, o, lse, stream);
}

}  // namespace frsa
