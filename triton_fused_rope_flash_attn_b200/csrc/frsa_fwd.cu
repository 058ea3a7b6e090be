// Forward kernel: O = softmax(R(Q) R(K)^T * scale) V with 2D RoPE fused.
//
// Restates the computation of _attn_fwd (fa_rope_full .py:91-315) as a
// warp-specialised tcgen05 kernel. One CTA owns one (batch*head, 128-query tile)
// unit and walks the keys in 128-key tiles with an online softmax in base 2.
//
//   warp 0      TMA producer: Q tile once, then K/V tiles into a 2-stage ring
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..5  "row" warpgroup: rotates Q and each K tile in shared memory,
//               reads S from TMEM (thread = query row), writes P (16-bit) to
//               shared memory, accumulates O in registers from the per-tile
//               P V product, and writes O and the log-sum-exp.
//
// TMEM columns: [0,128) S tile (f32), [128, 128+DP) per-tile P V (f32).
#include "frsa_internal.h"
#include "frsa_ptx.cuh"
#include "frsa_rope.cuh"

namespace frsa {

namespace {

constexpr int kFwdThreads = 192;
constexpr uint32_t kTmemColsFwd = 256;

template <int NCH>
struct FwdSmem {
  uint8_t q[NCH][kChunkBytes];
  uint8_t k[2][NCH][kChunkBytes];
  uint8_t v[2][NCH][kChunkBytes];
  uint8_t p[2][kChunkBytes];  // P tile [128 q][128 kv], two 64-column K chunks
  uint64_t q_full;
  uint64_t kv_full[2];
  uint64_t kv_empty[2];
  uint64_t k_ready[2];
  uint64_t s_full;
  uint64_t p_full;
  uint64_t o_full;
  uint32_t tmem_base;
  int abort_flag;
};

struct FwdParams {
  const float* cosp;
  const float* sinp;
  void* o;
  float* lse;
  int N, D, nqt, nkv, has_cls;
  float c2;  // scale * log2(e)
};

template <typename T, int NCH>
__global__ void __launch_bounds__(kFwdThreads, (NCH == 1 ? 2 : 1))
    fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
               const __grid_constant__ CUtensorMap tm_v, const FwdParams prm) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  FwdSmem<NCH>* smp = aligned_smem<FwdSmem<NCH>>(smem_raw);
  if (smp == nullptr) return;
  FwdSmem<NCH>& sm = *smp;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int unit = blockIdx.x;
  const int bh = unit / prm.nqt;
  const int qt = unit - bh * prm.nqt;
  const int q0 = qt * kTile;
  const int N = prm.N, D = prm.D;
  const int DP = (D + 15) & ~15;   // MMA N for P V
  const int ksteps = DP >> 4;      // MMA K steps over the head dim
  volatile int* abort_flag = &sm.abort_flag;

  if (threadIdx.x == 0) {
    sm.abort_flag = 0;
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
      mbar_init(&sm.k_ready[s], 1);
    }
    mbar_init(&sm.s_full, 1);
    mbar_init(&sm.p_full, 1);
    mbar_init(&sm.o_full, 1);
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
  const uint32_t tS = tmem;
  const uint32_t tO = tmem + kTile;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(&sm.q_full, NCH * kChunkBytes);
      for (int c = 0; c < NCH; ++c) tma_load_3d(sm.q[c], &tm_q, &sm.q_full, c * kChunkCols, q0, bh);
      for (int j = 0; j < prm.nkv; ++j) {
        const int s = j & 1;
        mbar_wait(&sm.kv_empty[s], ((j >> 1) & 1) ^ 1, abort_flag);
        mbar_arrive_expect_tx(&sm.kv_full[s], 2 * NCH * kChunkBytes);
        for (int c = 0; c < NCH; ++c) {
          tma_load_3d(sm.k[s][c], &tm_k, &sm.kv_full[s], c * kChunkCols, j * kTile, bh);
          tma_load_3d(sm.v[s][c], &tm_v, &sm.kv_full[s], c * kChunkCols, j * kTile, bh);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr bool kBf = Elt<T>::kBf16;
      const uint32_t idS = idesc_f16(kBf, 128, 128, false, false);
      const uint32_t idO = idesc_f16(kBf, 128, DP, false, true);
      for (int j = 0; j < prm.nkv; ++j) {
        const int s = j & 1;
        mbar_wait(&sm.k_ready[s], (j >> 1) & 1, abort_flag);
        tc_fence_after();
        // S = Q^ K^T : A = Q^ [q][d] K-major, B = K^ [kv][d] K-major.
        for (int ks = 0; ks < ksteps; ++ks) {
          const int c = ks >> 2;
          const uint32_t koff = (ks & 3) * 32;
          const uint64_t a = sw128_desc(smem_u32(sm.q[c]) + koff, 16, 1024);
          const uint64_t b = sw128_desc(smem_u32(sm.k[s][c]) + koff, 16, 1024);
          mma_ss(tS, a, b, idS, ks > 0);
        }
        mma_commit(&sm.s_full);
        mbar_wait(&sm.p_full, j & 1, abort_flag);
        tc_fence_after();
        // O_j = P V : A = P [q][kv] K-major, B = V [kv][d] MN-major.
        for (int ks = 0; ks < kTile / 16; ++ks) {
          const uint64_t a = sw128_desc(smem_u32(sm.p[ks >> 2]) + (ks & 3) * 32, 16, 1024);
          const uint64_t b = sw128_desc(smem_u32(sm.v[s][0]) + ks * 2048, kChunkBytes, 1024);
          mma_ss(tO, a, b, idO, ks > 0);
        }
        mma_commit(&sm.o_full);
        mma_commit(&sm.kv_empty[s]);
      }
    }
  } else {
    // ------------------------------------------------------------ row warpgroup
    const int wq = warp & 3;               // TMEM lane quarter this warp may access
    const int r = wq * 32 + lane;          // tile row == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const int tid = threadIdx.x - 64;      // 0..127 inside the warpgroup
    const int qrow = q0 + r;
    const float c2 = prm.c2;

    float o_acc[64 * NCH];
#pragma unroll
    for (int i = 0; i < 64 * NCH; ++i) o_acc[i] = 0.f;
    float m2 = -INFINITY, l = 0.f;

    // Q rotation, then K_0 rotation.
    FRSA_STAMP(0);
    {
      RopeRows<NCH> rope;
      load_rope_rows<NCH>(rope, wq * 32, q0, N, prm.has_cls, D, prm.cosp, prm.sinp, lane);
      mbar_wait(&sm.q_full, 0, abort_flag);
      FRSA_STAMP(1);
      apply_rope_rows<T, NCH>(&sm.q[0][0], wq * 32, D, rope, lane);
      load_rope_rows<NCH>(rope, wq * 32, 0, N, prm.has_cls, D, prm.cosp, prm.sinp, lane);
      mbar_wait(&sm.kv_full[0], 0, abort_flag);
      FRSA_STAMP(2);
      apply_rope_rows<T, NCH>(&sm.k[0][0][0], wq * 32, D, rope, lane);
    }
    fence_proxy_async_smem();
    named_bar(1, 128);
    if (tid == 0) mbar_arrive(&sm.k_ready[0]);
    FRSA_STAMP(3);

    for (int j = 0; j < prm.nkv; ++j) {
      const int kv0 = j * kTile;
      const int nvalid = min(kTile, N - kv0);
      mbar_wait(&sm.s_full, j & 1, abort_flag);
      tc_fence_after();
      FRSA_STAMP(4 + 5 * j);

      // pass 1: row max of the valid columns
      float mx = -INFINITY;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        float sv[32];
        tmem_ld32(tS + lane_off + cc * 32, sv);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (cc * 32 + i < nvalid) mx = fmaxf(mx, sv[i]);
      }
      const float m_new = fmaxf(m2, mx * c2);
      const float alpha = ex2(m2 - m_new);
      // pass 2: P = exp2(S c2 - m), row sum, 16-bit P into shared memory
      float sum = 0.f;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        float sv[32];
        tmem_ld32(tS + lane_off + cc * 32, sv);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float pv = (cc * 32 + i < nvalid) ? ex2(fmaf(sv[i], c2, -m_new)) : 0.f;
          sv[i] = pv;
          sum += pv;
        }
        uint8_t* pchunk = sm.p[cc >> 1];
#pragma unroll
        for (int g4 = 0; g4 < 4; ++g4) {
          uint4 w;
          w.x = Elt<T>::pack(sv[g4 * 8 + 0], sv[g4 * 8 + 1]);
          w.y = Elt<T>::pack(sv[g4 * 8 + 2], sv[g4 * 8 + 3]);
          w.z = Elt<T>::pack(sv[g4 * 8 + 4], sv[g4 * 8 + 5]);
          w.w = Elt<T>::pack(sv[g4 * 8 + 6], sv[g4 * 8 + 7]);
          *reinterpret_cast<uint4*>(pchunk + sw128_off(r, (cc & 1) * 4 + g4)) = w;
        }
      }
      l = l * alpha + sum;
      m2 = m_new;
      fence_proxy_async_smem();
      tc_fence_before();
      named_bar(1, 128);
      if (tid == 0) mbar_arrive(&sm.p_full);
      FRSA_STAMP(5 + 5 * j);

      // rotate the next K tile while this tile's P V runs
      if (j + 1 < prm.nkv) {
        const int s1 = (j + 1) & 1;
        RopeRows<NCH> rope;
        load_rope_rows<NCH>(rope, wq * 32, kv0 + kTile, N, prm.has_cls, D, prm.cosp, prm.sinp,
                            lane);
        mbar_wait(&sm.kv_full[s1], ((j + 1) >> 1) & 1, abort_flag);
        apply_rope_rows<T, NCH>(&sm.k[s1][0][0], wq * 32, D, rope, lane);
        fence_proxy_async_smem();
        named_bar(1, 128);
        if (tid == 0) mbar_arrive(&sm.k_ready[s1]);
      }
      FRSA_STAMP(6 + 5 * j);

      // O = O * alpha + P V
      mbar_wait(&sm.o_full, j & 1, abort_flag);
      tc_fence_after();
      FRSA_STAMP(7 + 5 * j);
#pragma unroll
      for (int c16 = 0; c16 < 4 * NCH; ++c16) {
        if (c16 * 16 < DP) {
          float ov[16];
          tmem_ld16(tO + lane_off + c16 * 16, ov);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o_acc[c16 * 16 + i] = fmaf(o_acc[c16 * 16 + i], alpha, ov[i]);
        }
      }
      tc_fence_before();
    }

    // epilogue: O / l and lse = (m + log2 l) ln 2. Rows go through an f32
    // staging tile (the K stages, idle once the last P V has completed) and
    // are written by warp-per-row coalesced stores.
    const float inv_l = 1.f / l;
    if (qrow < N)
      prm.lse[static_cast<size_t>(bh) * N + qrow] = (m2 + lg2(l)) * 0.69314718055994531f;
    uint8_t* stage = &sm.k[0][0][0];
#pragma unroll
    for (int c16 = 0; c16 < 4 * NCH; ++c16) {
      if (c16 * 16 < DP) {
        float v[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] = o_acc[c16 * 16 + e] * inv_l;
        stage_write16<NCH>(stage, r, c16, v);
      }
    }
    named_bar(1, 128);
    drain_rows_warp<T, NCH, 32>(stage, wq * 32, q0, N, D, 1.f, nullptr,
                            reinterpret_cast<T*>(prm.o) + static_cast<size_t>(bh) * N * D, lane);
    FRSA_STAMP(30);
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
  p.N = s.N;
  p.D = s.D;
  p.nqt = (s.N + kTile - 1) / kTile;
  p.nkv = p.nqt;
  p.has_cls = s.has_cls;
  p.c2 = s.scale * 1.4426950408889634f;
  // The dynamic window starts 1024-aligned in practice; the slack covers a
  // smaller alignment and keeps two NCH=1 CTAs within one SM's 228 KiB.
  const size_t smem = sizeof(FwdSmem<NCH>) + 256;
  auto kern = fwd_kernel<T, NCH>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const long long units = static_cast<long long>(s.BH) * p.nqt;
  kern<<<static_cast<unsigned>(units), kFwdThreads, smem, stream>>>(tm_q, tm_k, tm_v, p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_fwd(const LaunchShape& s, const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                       const CUtensorMap& tm_v, const float* cosp, const float* sinp, void* o,
                       float* lse, cudaStream_t stream) {
  const bool two = s.D > 64;
  if (s.bf16) {
    return two ? launch_fwd_t<__nv_bfloat16, 2>(s, tm_q, tm_k, tm_v, cosp, sinp, o, lse, stream)
               : launch_fwd_t<__nv_bfloat16, 1>(s, tm_q, tm_k, tm_v, cosp, sinp, o, lse, stream);
  }
  return two ? launch_fwd_t<__half, 2>(s, tm_q, tm_k, tm_v, cosp, sinp, o, lse, stream)
             : launch_fwd_t<__half, 1>(s, tm_q, tm_k, tm_v, cosp, sinp, o, lse, stream);
}

}  // namespace frsa
