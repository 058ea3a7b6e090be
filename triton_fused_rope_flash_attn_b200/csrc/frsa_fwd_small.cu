// Persistent forward kernel for short sequences: N <= 256 and D <= 64 (the
// ViT-S/B shapes, N = 197). Same computation as fwd_kernel
// (fa_rope_full .py:91-315); specialised so that per head nothing waits on
// global-memory latency except the tile loads themselves:
//
//   - the CTA is persistent (one per SM) and walks heads bh = blockIdx.x,
//     blockIdx.x + gridDim.x, ...; the next head's tiles are loaded and
//     rotated while the current head's softmax and epilogue run;
//   - the RoPE tables (identical for every head) are copied into shared memory
//     once per CTA, so rotation reads them with shared loads;
//   - every K/V tile of a head has its own buffer (at most two), and the whole
//     head is one unit: two query tiles, one per compute warpgroup.
//
// Roles: warp 0 TMA producer, warp 1 TMEM allocator + MMA issuer, warps 2..3
// rotate Q and K tiles in place, warps 4..11 two softmax warpgroups (warpgroup
// g = query tile g; thread = query row = TMEM lane).
//
// TMEM columns: warpgroup g uses [256 g, 256 g + 128) for S and
// [256 g + 128, 256 g + 192) for the per-tile P V.
#include "frsa_internal.h"
#include "frsa_ptx.cuh"
#include "frsa_rope.cuh"

#undef FRSA_STAMP_TID
#define FRSA_STAMP_TID 128

namespace frsa {

namespace {

constexpr int kFsThreads = 384;
constexpr int kFsMaxPos = 256;

struct FsSmem {
  uint8_t q[2][kChunkBytes];      // query tiles of the head
  uint8_t k[2][kChunkBytes];      // key tiles of the head
  uint8_t v[2][kChunkBytes];      // value tiles of the head
  uint8_t p[2][2][kChunkBytes];   // P tile of warpgroup g, two 64-column chunks
  float cos_t[kFsMaxPos * 32];    // RoPE tables, [pos][32] (D/2 <= 32 used)
  float sin_t[kFsMaxPos * 32];
  uint64_t q_full, q_ready, q_empty;
  uint64_t kv_full[2], k_ready[2], kv_empty[2];
  uint64_t s_full[2], p_full[2], o_full[2];
  uint32_t tmem_base;
  int abort_flag;
};

struct FsParams {
  const float* cosp;
  const float* sinp;
  void* o;
  float* lse;
  int BH, N, D, nqt, nkv, has_cls;
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
  const int N = prm.N, D = prm.D, D2 = D >> 1;
  const int DP = (D + 15) & ~15;
  const int ksteps = DP >> 4;
  const int nqt = prm.nqt, nkv = prm.nkv;
  volatile int* abort_flag = &sm.abort_flag;

  // RoPE tables into shared memory (rows actually used: N - has_cls).
  {
    const int rows = N - prm.has_cls;
    for (int idx = threadIdx.x; idx < rows * 32; idx += kFsThreads) {
      const int pos = idx >> 5, p = idx & 31;
      sm.cos_t[idx] = p < D2 ? __ldg(prm.cosp + static_cast<size_t>(pos) * D2 + p) : 0.f;
      sm.sin_t[idx] = p < D2 ? __ldg(prm.sinp + static_cast<size_t>(pos) * D2 + p) : 0.f;
    }
  }
  if (threadIdx.x == 0) {
    sm.abort_flag = 0;
    mbar_init(&sm.q_full, 1);
    mbar_init(&sm.q_ready, 1);
    mbar_init(&sm.q_empty, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.k_ready[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.p_full[s], 1);
      mbar_init(&sm.o_full[s], 1);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  FRSA_STAMP_T(31, 128);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  FRSA_STAMP_T(30, 128);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      int hl = 0;
      for (int bh = blockIdx.x; bh < prm.BH; bh += gridDim.x, ++hl) {
        const uint32_t free_par = (hl & 1) ^ 1;
        mbar_wait(&sm.q_empty, free_par, abort_flag);
        mbar_arrive_expect_tx(&sm.q_full, nqt * kChunkBytes);
        for (int g = 0; g < nqt; ++g) tma_load_3d(sm.q[g], &tm_q, &sm.q_full, 0, g * kTile, bh);
        for (int j = 0; j < nkv; ++j) {
          mbar_wait(&sm.kv_empty[j], free_par, abort_flag);
          mbar_arrive_expect_tx(&sm.kv_full[j], 2 * kChunkBytes);
          tma_load_3d(sm.k[j], &tm_k, &sm.kv_full[j], 0, j * kTile, bh);
          tma_load_3d(sm.v[j], &tm_v, &sm.kv_full[j], 0, j * kTile, bh);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr bool kBf = Elt<T>::kBf16;
      const uint32_t idS = idesc_f16(kBf, 128, 128, false, false);
      const uint32_t idO = idesc_f16(kBf, 128, DP, false, true);
      auto issue_s = [&](int g, int j) {
        for (int ks = 0; ks < ksteps; ++ks) {
          const uint32_t koff = ks * 32;
          mma_ss(tmem + 256 * g, sw128_desc(smem_u32(sm.q[g]) + koff, 16, 1024),
                 sw128_desc(smem_u32(sm.k[j]) + koff, 16, 1024), idS, ks > 0);
        }
        mma_commit(&sm.s_full[g]);
      };
      auto issue_pv = [&](int g, int j) {
        for (int ks = 0; ks < kTile / 16; ++ks) {
          mma_ss(tmem + 256 * g + 128,
                 sw128_desc(smem_u32(sm.p[g][ks >> 2]) + (ks & 3) * 32, 16, 1024),
                 sw128_desc(smem_u32(sm.v[j]) + ks * 2048, kChunkBytes, 1024), idO, ks > 0);
        }
        mma_commit(&sm.o_full[g]);
      };
      int hl = 0;
      for (int bh = blockIdx.x; bh < prm.BH; bh += gridDim.x, ++hl) {
        const uint32_t hp = hl & 1;
        mbar_wait(&sm.q_ready, hp, abort_flag);
        mbar_wait(&sm.k_ready[0], hp, abort_flag);
        tc_fence_after();
        for (int g = 0; g < nqt; ++g) issue_s(g, 0);
        // The Q tiles are free for the next head once the last S MMA reading
        // them completes, long before this head's P V products.
        if (nkv == 1) mma_commit(&sm.q_empty);
        for (int j = 0; j < nkv; ++j) {
          const int c = hl * nkv + j;
          for (int g = 0; g < nqt; ++g) {
            mbar_wait(&sm.p_full[g], c & 1, abort_flag);
            tc_fence_after();
            issue_pv(g, j);
            if (j + 1 < nkv) {
              if (g == 0) {
                mbar_wait(&sm.k_ready[j + 1], hp, abort_flag);
                tc_fence_after();
              }
              issue_s(g, j + 1);
              if (j + 2 == nkv && g == nqt - 1) mma_commit(&sm.q_empty);
            }
          }
          mma_commit(&sm.kv_empty[j]);
        }
      }
    }
  } else if (warp < 4) {
    // ------------------------------------------------------------ rotation warps
    const int rwp = warp - 2;
    const uint32_t cos_sm = smem_u32(sm.cos_t), sin_sm = smem_u32(sm.sin_t);
    int hl = 0;
    for (int bh = blockIdx.x; bh < prm.BH; bh += gridDim.x, ++hl) {
      const uint32_t hp = hl & 1;
      mbar_wait(&sm.q_full, hp, abort_flag);
      if (hl < 2) FRSA_STAMP_T(hl * 12 + 0, 64);
      for (int g = 0; g < nqt; ++g)
        rotate_q_tabsm<T>(smem_u32(sm.q[g]), rwp * 64, 64, g * kTile, N, prm.has_cls, D,
                          cos_sm, sin_sm, lane);
      fence_proxy_async_smem();
      named_bar(1, 64);
      if (threadIdx.x == 64) mbar_arrive(&sm.q_ready);
      if (hl < 2) FRSA_STAMP_T(hl * 12 + 1, 64);
      for (int j = 0; j < nkv; ++j) {
        mbar_wait(&sm.kv_full[j], hp, abort_flag);
        if (hl < 2) FRSA_STAMP_T(hl * 12 + 2 + j, 64);
        rotate_q_tabsm<T>(smem_u32(sm.k[j]), rwp * 64, 64, j * kTile, N, prm.has_cls, D,
                          cos_sm, sin_sm, lane);
        fence_proxy_async_smem();
        named_bar(1, 64);
        if (threadIdx.x == 64) mbar_arrive(&sm.k_ready[j]);
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
    const bool warp_active = (q0 + wq * 32) < N;
    const uint32_t pb0 = smem_u32(sm.p[g][0]);
    if (g < nqt) {
      int hl = 0;
      for (int bh = blockIdx.x; bh < prm.BH; bh += gridDim.x, ++hl) {
        float o_acc[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) o_acc[i] = 0.f;
        float m2 = -INFINITY, l = 0.f;
        for (int j = 0; j < nkv; ++j) {
          const int c = hl * nkv + j;
          const int nvalid = min(kTile, N - j * kTile);
          mbar_wait(&sm.s_full[g], c & 1, abort_flag);
          tc_fence_after();
          if (hl < 2) FRSA_STAMP_T(hl * 12 + 4 + j * 3, 128);
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
                if (cbase + 32 <= nvalid) {
#pragma unroll
                  for (int i = 0; i < 32; ++i) {
                    sv[u][i] = ex2(fmaf(sv[u][i], c2, -m_new));
                    sum += sv[u][i];
                  }
                } else if (cbase < nvalid) {
#pragma unroll
                  for (int i = 0; i < 32; ++i) {
                    sv[u][i] = (cbase + i < nvalid) ? ex2(fmaf(sv[u][i], c2, -m_new)) : 0.f;
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
            l = l * alpha + sum;
            m2 = m_new;
          }
          fence_proxy_async_smem();
          tc_fence_before();
          named_bar(2 + g, 128);
          if (leader) mbar_arrive(&sm.p_full[g]);
          if (hl < 2) FRSA_STAMP_T(hl * 12 + 5 + j * 3, 128);

          mbar_wait(&sm.o_full[g], c & 1, abort_flag);
          tc_fence_after();
          if (hl < 2) FRSA_STAMP_T(hl * 12 + 6 + j * 3, 128);
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
        // epilogue through this group's P tile (the head's last P V is done)
        if (qrow < N)
          prm.lse[static_cast<size_t>(bh) * N + qrow] = (m2 + lg2(l)) * 0.69314718055994531f;
        const float inv_l = warp_active ? 1.f / l : 0.f;
        uint8_t* stage = &sm.p[g][0][0];
#pragma unroll
        for (int c16 = 0; c16 < 4; ++c16) {
          float v[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = o_acc[c16 * 16 + e] * inv_l;
          stage_write16<1>(stage, r, c16, v);
        }
        named_bar(2 + g, 128);
        drain_block_q<T, 32>(stage, wq * 32, q0, N, D, 0,
                                reinterpret_cast<T*>(prm.o) + static_cast<size_t>(bh) * N * D,
                                lane);
        named_bar(2 + g, 128);
        if (hl < 2) FRSA_STAMP_T(hl * 12 + 10, 128);
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
                               const float* cosp, const float* sinp, void* o, float* lse,
                               cudaStream_t stream) {
  FsParams p;
  p.cosp = cosp;
  p.sinp = sinp;
  p.o = o;
  p.lse = lse;
  p.BH = s.BH;
  p.N = s.N;
  p.D = s.D;
  p.nqt = (s.N + kTile - 1) / kTile;
  p.nkv = p.nqt;
  p.has_cls = s.has_cls;
  p.c2 = s.scale * 1.4426950408889634f;
  const size_t smem = sizeof(FsSmem) + 1024;
  auto kern = fwd_small_kernel<T>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const int grid = s.BH < sm_count() ? s.BH : sm_count();
  kern<<<grid, kFsThreads, smem, stream>>>(tm_q, tm_k, tm_v, p);
  return cudaGetLastError();
}

}  // namespace

bool fwd_small_applies(const LaunchShape& s) { return s.N <= 2 * kTile && s.D <= 64; }

cudaError_t launch_fwd_small(const LaunchShape& s, const CUtensorMap& tm_q,
                             const CUtensorMap& tm_k, const CUtensorMap& tm_v, const float* cosp,
                             const float* sinp, void* o, float* lse, cudaStream_t stream) {
  return s.bf16 ? launch_fwd_small_t<__nv_bfloat16>(s, tm_q, tm_k, tm_v, cosp, sinp, o, lse, stream)
                : launch_fwd_small_t<__half>(s, tm_q, tm_k, tm_v, cosp, sinp, o, lse, stream);
}

}  // namespace frsa
