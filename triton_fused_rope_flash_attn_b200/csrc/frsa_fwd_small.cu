// Persistent forward kernel for short sequences: N <= 256 and D <= 64 (the
// ViT-S/B shapes, N = 197). Same computation as fwd_kernel
// (fa_rope_full .py:91-315), organised so that consecutive heads overlap:
//
//   - the CTA is persistent (one per SM) and walks heads bh = blockIdx.x,
//     blockIdx.x + gridDim.x, ...; Q and K/V tiles are double-buffered per
//     head, so the next head loads and rotates while this one computes;
//   - P never touches shared memory: the softmax writes it (16-bit, two per
//     32-bit column) over S in tensor memory and the P V product takes its A
//     operand from there;
//   - the RoPE tables (identical for every head) are two shared "table tiles"
//     of packed f16 (cos, sin) pairs filled once per CTA;
//   - O is staged as 16-bit rows in the head's finished Q tile and written by
//     a TMA store (rows past N are clipped by the tensor map).
//
// Roles: warp 0 TMA producer, warp 1 TMEM allocator + MMA issuer, warps 2..3
// rotate Q and K tiles in place, warps 4..11 two softmax warpgroups (warpgroup
// g = query tile g; thread = query row = TMEM lane).
//
// TMEM columns: warpgroup g uses [256 g, 256 g + 128) for S (P packed into its
// first 64 columns) and [256 g + 128, 256 g + 192) for the per-tile P V.
#include "frsa_internal.h"
#include "frsa_ptx.cuh"
#include "frsa_rope.cuh"

#undef FRSA_STAMP_TID
#define FRSA_STAMP_TID 128

namespace frsa {

namespace {

constexpr int kFsThreads = 384;

struct FsSmem {
  uint8_t q[2][2][kChunkBytes];    // [head stage][query tile]
  uint8_t k[2][2][kChunkBytes];    // [head stage][key tile]
  uint8_t v[2][2][kChunkBytes];
  uint8_t tab[2][kChunkBytes];     // f16 (cos, sin) table tiles of token tiles 0, 1
  uint64_t q_full[2], q_ready[2], q_empty[2];
  uint64_t kv_full[2][2], k_ready[2][2], kv_empty[2][2];
  uint64_t s_full[2], p_full[2], o_full[2];
  uint32_t tmem_base;
  int abort_flag;
};

struct FsParams {
  const float* cosp;
  const float* sinp;
  float* lse;
  int BH, N, D, nqt, nkv, has_cls;
  float c2;
};

template <typename T>
__global__ void __launch_bounds__(kFsThreads, 1)
    fwd_small_kernel(const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v,
                     const __grid_constant__ CUtensorMap tm_o, const FsParams prm) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  FsSmem* smp = aligned_smem<FsSmem>(smem_raw);
  if (smp == nullptr) return;
  FsSmem& sm = *smp;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int N = prm.N, D = prm.D;
  const int DP = (D + 15) & ~15;
  const int ksteps = DP >> 4;
  const int nqt = prm.nqt, nkv = prm.nkv;
  volatile int* abort_flag = &sm.abort_flag;

  if (threadIdx.x == 0) {
    sm.abort_flag = 0;
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.q_full[s], 1);
      mbar_init(&sm.q_ready[s], 1);
      mbar_init(&sm.q_empty[s], nqt);   // one arrival per softmax warpgroup
      for (int j = 0; j < 2; ++j) {
        mbar_init(&sm.kv_full[s][j], 1);
        mbar_init(&sm.k_ready[s][j], 1);
        mbar_init(&sm.kv_empty[s][j], 1);
      }
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.p_full[s], 4);   // one arrival per softmax warp
      mbar_init(&sm.o_full[s], 1);
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

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_o);
      int hl = 0;
      for (int bh = blockIdx.x; bh < prm.BH; bh += gridDim.x, ++hl) {
        const int st = hl & 1;
        const uint32_t fp = ((hl >> 1) & 1) ^ 1;
        mbar_wait(&sm.q_empty[st], fp, abort_flag);
        mbar_arrive_expect_tx(&sm.q_full[st], nqt * kChunkBytes);
        for (int g = 0; g < nqt; ++g)
          tma_load_3d(sm.q[st][g], &tm_q, &sm.q_full[st], 0, g * kTile, bh);
        for (int j = 0; j < nkv; ++j) {
          mbar_wait(&sm.kv_empty[st][j], fp, abort_flag);
          mbar_arrive_expect_tx(&sm.kv_full[st][j], 2 * kChunkBytes);
          tma_load_3d(sm.k[st][j], &tm_k, &sm.kv_full[st][j], 0, j * kTile, bh);
          tma_load_3d(sm.v[st][j], &tm_v, &sm.kv_full[st][j], 0, j * kTile, bh);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr bool kBf = Elt<T>::kBf16;
      const uint32_t idS = idesc_f16(kBf, 128, 128, false, false);
      const uint32_t idO = idesc_f16(kBf, 128, DP, false, true);
      int hl = 0;
      for (int bh = blockIdx.x; bh < prm.BH; bh += gridDim.x, ++hl) {
        const int st = hl & 1;
        const uint32_t hp = (hl >> 1) & 1;
        auto issue_s = [&](int g, int j) {
          for (int ks = 0; ks < ksteps; ++ks) {
            const uint32_t koff = ks * 32;
            mma_ss(tmem + 256 * g, sw128_desc(smem_u32(sm.q[st][g]) + koff, 16, 1024),
                   sw128_desc(smem_u32(sm.k[st][j]) + koff, 16, 1024), idS, ks > 0);
          }
          mma_commit(&sm.s_full[g]);
        };
        // O_g = P_g V : A = P in TMEM (over S), B = V [kv][d] MN-major.
        auto issue_pv = [&](int g, int j) {
          for (int ks = 0; ks < kTile / 16; ++ks)
            mma_ts(tmem + 256 * g + 128, tmem + 256 * g + ks * 8,
                   sw128_desc(smem_u32(sm.v[st][j]) + ks * 2048, kChunkBytes, 1024), idO, ks > 0);
          mma_commit(&sm.o_full[g]);
        };
        mbar_wait(&sm.q_ready[st], hp, abort_flag);
        mbar_wait(&sm.k_ready[st][0], hp, abort_flag);
        tc_fence_after();
        for (int g = 0; g < nqt; ++g) {
          // S_g of this head overwrites P_g of the previous one; the softmax
          // group has read O_g of that head before arriving p_full, and the
          // previous P V (same pipe, in order) reads P_g before this S writes.
          issue_s(g, 0);
        }
        for (int j = 0; j < nkv; ++j) {
          const int c = hl * nkv + j;
          for (int g = 0; g < nqt; ++g) {
            mbar_wait(&sm.p_full[g], c & 1, abort_flag);
            tc_fence_after();
            issue_pv(g, j);
            if (j + 1 < nkv) {
              if (g == 0) {
                mbar_wait(&sm.k_ready[st][j + 1], hp, abort_flag);
                tc_fence_after();
              }
              // S_g of the next tile overwrites P_g: the P V just issued reads
              // it first (same pipe, in order).
              issue_s(g, j + 1);
            }
          }
          mma_commit(&sm.kv_empty[st][j]);
        }
      }
    }
  } else if (warp < 4) {
    // ------------------------------------------------------------ rotation warps
    // 64 threads, thread t handles tile rows t and t + 64.
    const int t = threadIdx.x - 64;
    for (int rr = t; rr < kTile; rr += 64) {
      store_tabrow(smem_u32(sm.tab[0]), rr, rope_pos(rr, N, prm.has_cls), D, prm.cosp, prm.sinp);
      store_tabrow(smem_u32(sm.tab[1]), rr, rope_pos(kTile + rr, N, prm.has_cls), D, prm.cosp,
                   prm.sinp);
    }
    named_bar(1, 64);
    int hl = 0;
    for (int bh = blockIdx.x; bh < prm.BH; bh += gridDim.x, ++hl) {
      const int st = hl & 1;
      const uint32_t hp = (hl >> 1) & 1;
      mbar_wait(&sm.q_full[st], hp, abort_flag);
      for (int g = 0; g < nqt; ++g)
        for (int rr = t; rr < kTile; rr += 64)
          rotate_row_t<T, 4>(smem_u32(sm.q[st][g]), smem_u32(sm.tab[g]), rr, D);
      fence_proxy_async_smem();
      named_bar(1, 64);
      if (t == 0) mbar_arrive(&sm.q_ready[st]);
      for (int j = 0; j < nkv; ++j) {
        mbar_wait(&sm.kv_full[st][j], hp, abort_flag);
        for (int rr = t; rr < kTile; rr += 64)
          rotate_row_t<T, 4>(smem_u32(sm.k[st][j]), smem_u32(sm.tab[j]), rr, D);
        fence_proxy_async_smem();
        named_bar(1, 64);
        if (t == 0) mbar_arrive(&sm.k_ready[st][j]);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warpgroups
    const int cw = warp - 4;
    const int g = cw >> 2;
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const bool leader = threadIdx.x == 128 + 128 * g;
    const int q0 = g * kTile;
    const int qrow = q0 + r;
    const float c2 = prm.c2;
    const uint32_t tS = tmem + 256 * g + lane_off;
    const uint32_t tO = tmem + 256 * g + 128 + lane_off;
    // A warp whose 32 query rows are all padding skips the softmax math: its P
    // rows only ever reach O rows that are not stored.
    const bool warp_active = (q0 + wq * 32) < N;
    if (g < nqt) {
      int hl = 0;
      for (int bh = blockIdx.x; bh < prm.BH; bh += gridDim.x, ++hl) {
        const int st = hl & 1;
        float o_acc[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) o_acc[i] = 0.f;
        float m2 = -INFINITY, l = 0.f;
        for (int j = 0; j < nkv; ++j) {
          const int c = hl * nkv + j;
          const int nvalid = min(kTile, N - j * kTile);
          mbar_wait(&sm.s_full[g], c & 1, abort_flag);
          tc_fence_after();
          float alpha = 1.f;
          if (warp_active) {
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
            const float m_new = fmaxf(m2, mx * c2);
            alpha = ex2(m2 - m_new);
            float sum = 0.f;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              float sv[2][32];
              tmem_ld32(tS + h * 64, sv[0]);
              tmem_ld32(tS + h * 64 + 32, sv[1]);
              tmem_wait_ld();
#pragma unroll
              for (int u = 0; u < 2; ++u) {
                const int cbase = h * 64 + u * 32;
                uint32_t pk[16];
                if (cbase + 32 <= nvalid) {
#pragma unroll
                  for (int i = 0; i < 16; ++i) {
                    const float a = ex2(fmaf(sv[u][2 * i], c2, -m_new));
                    const float b = ex2(fmaf(sv[u][2 * i + 1], c2, -m_new));
                    sum += a + b;
                    pk[i] = Elt<T>::pack(a, b);
                  }
                } else if (cbase < nvalid) {
#pragma unroll
                  for (int i = 0; i < 16; ++i) {
                    const float a =
                        (cbase + 2 * i < nvalid) ? ex2(fmaf(sv[u][2 * i], c2, -m_new)) : 0.f;
                    const float b = (cbase + 2 * i + 1 < nvalid)
                                        ? ex2(fmaf(sv[u][2 * i + 1], c2, -m_new))
                                        : 0.f;
                    sum += a + b;
                    pk[i] = Elt<T>::pack(a, b);
                  }
                } else {
#pragma unroll
                  for (int i = 0; i < 16; ++i) pk[i] = 0u;
                }
                // P columns [cbase, cbase + 32) -> packed TMEM columns from
                // cbase / 2 (already read: the write front trails the read front).
                tmem_st16(tS + cbase / 2, pk);
              }
            }
            tmem_wait_st();
            l = l * alpha + sum;
            m2 = m_new;
          }
          tc_fence_before();
          // Each warp publishes its own rows (no cross-warp barrier here).
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.p_full[g]);

          mbar_wait(&sm.o_full[g], c & 1, abort_flag);
          tc_fence_after();
          if (warp_active) {
#pragma unroll
            for (int c32 = 0; c32 < 2; ++c32) {
              if (c32 * 32 < DP) {
                float ov[32];
                tmem_ld32(tO + c32 * 32, ov);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i)
                  o_acc[c32 * 32 + i] = fmaf(o_acc[c32 * 32 + i], alpha, ov[i]);
              }
            }
          }
          tc_fence_before();
        }
        // epilogue: lse, then O / l as 16-bit rows into this head's (finished)
        // Q tile and a TMA store of the tile.
        if (qrow < N)
          prm.lse[static_cast<size_t>(bh) * N + qrow] = (m2 + lg2(l)) * 0.69314718055994531f;
        const float inv_l = warp_active ? 1.f / l : 0.f;
        const uint32_t stage = smem_u32(sm.q[st][g]);
#pragma unroll
        for (int gg = 0; gg < 8; ++gg) {
          float u[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) u[e] = o_acc[8 * gg + e] * inv_l;
          sts_u4(stage + sw128_off(r, gg), pack8<T>(u));
        }
        fence_proxy_async_smem();
        named_bar(2 + g, 128);
        if (leader) {
          tma_store_3d(&tm_o, sm.q[st][g], 0, q0, bh);
          tma_store_commit();
          tma_store_wait_read();
          mbar_arrive(&sm.q_empty[st]);
        }
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

int sm_count() {
  static int cache[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

template <typename T>
cudaError_t launch_fwd_small_t(const LaunchShape& s, const CUtensorMap& tm_q,
                               const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                               const CUtensorMap& tm_o, const float* cosp, const float* sinp,
                               float* lse, cudaStream_t stream) {
  FsParams p;
  p.cosp = cosp;
  p.sinp = sinp;
  p.lse = lse;
  p.BH = s.BH;
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
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const int grid = s.BH < sm_count() ? s.BH : sm_count();
  kern<<<grid, kFsThreads, smem, stream>>>(tm_q, tm_k, tm_v, tm_o, p);
  return cudaGetLastError();
}

}  // namespace

bool fwd_small_applies(const LaunchShape& s) { return s.N <= 2 * kTile && s.D <= 64; }

cudaError_t launch_fwd_small(const LaunchShape& s, const CUtensorMap& tm_q,
                             const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                             const CUtensorMap& tm_o, const float* cosp, const float* sinp,
                             float* lse, cudaStream_t stream) {
  return s.bf16 ? launch_fwd_small_t<__nv_bfloat16>(s, tm_q, tm_k, tm_v, tm_o, cosp, sinp, lse,
                                                    stream)
                : launch_fwd_small_t<__half>(s, tm_q, tm_k, tm_v, tm_o, cosp, sinp, lse, stream);
}

}  // namespace frsa
