// float32 compute on TF32 tensor cores (tcgen05.mma kind::tf32), the
// reference's mode for float32 inputs without autocast (fa_rope_full
// .py:65-73: the kernels run with DTYPE = float32 and Triton's dots use TF32).
//
// Tiles hold 32-bit elements: a 128-row tile of D columns is D/32 chunks of
// 128 rows x 128 bytes (32 floats), each in the 128-byte swizzled layout TMA
// writes (box {32, 128, 1}). A K step of kind::tf32 is 8 elements = 32 bytes,
// the same byte step as a 16-bit K16 step, so the K-major descriptors advance
// exactly as in the 16-bit kernels; MN-major operands (V, dO, Q^ in the P V,
// dV and dK products) advance 8 rows = 1024 bytes per step with 16 KiB between
// 32-column chunks. MN-major 32-bit operands need a different shared layout
// than K-major ones: the 128-byte swizzle with 32-byte atoms (32-byte
// granules XOR (row & 3); descriptor layout type 1, 4-row groups 512 bytes
// apart), which TMA writes with CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B. P and dS
// stay float32 in TMEM, where the TS form reads them as TF32.
//
// This kernel favours simplicity over speed (one CTA per query tile, no
// persistence): float32 compute is the reference's slow, accurate mode. The
// float32 backward runs on the 16-bit kernels (see the host wrapper).
#include "frsa_internal.h"
#include "frsa_ptx.cuh"
#include "frsa_rope.cuh"

#undef FRSA_STAMP_TID
#define FRSA_STAMP_TID 128

namespace frsa {

namespace {

// kind::tf32 instruction descriptor: D f32 (bit 4), A/B format TF32 = 2
// (bits 7-9, 10-12), A/B major (bits 15, 16), N >> 3 (bits 17-22), M >> 4
// (bits 24-28).
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Descriptor of an MN-major 32-bit operand in the 32-byte-atom 128-byte
// swizzle: LBO = bytes between 32-column chunks, SBO = 512 (4-row groups).
__device__ __forceinline__ uint64_t mn32_desc(uint32_t smem_addr, uint32_t chunk_stride) {
  const uint64_t d = sw128_desc(smem_addr, chunk_stride, 512);
  return (d & ~(7ull << 61)) | (1ull << 61);
}

// 32 consecutive 32-bit columns of this thread's TMEM lane (32x32b.x32 store).
__device__ __forceinline__ void tmem_st32f(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(
          taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]),
      "f"(v[8]), "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]),
      "f"(v[15]), "f"(v[16]), "f"(v[17]), "f"(v[18]), "f"(v[19]), "f"(v[20]), "f"(v[21]),
      "f"(v[22]), "f"(v[23]), "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]), "f"(v[28]),
      "f"(v[29]), "f"(v[30]), "f"(v[31])
      : "memory");
}

// Byte offset of granule g (floats 4g..4g+3) of row r in a multi-chunk
// 32-bit tile.
__device__ __forceinline__ uint32_t f32_off(int r, int g) {
  return static_cast<uint32_t>(g >> 3) * kChunkBytes + sw128_off(r, g & 7);
}

// Rotate row r of a 32-bit tile in place for token position pos (pos < 0: the
// CLS token or padding, left as is): pairs (2p, 2p+1) -> (e c - o s, o c + e s)
// with (c, s) = (COSP, SINP)[pos, p] (fa_rope_full .py:201-202, 271-272).
__device__ __forceinline__ void rotate_row_f32(uint32_t tile, int r, int pos, int D,
                                               const float* __restrict__ cosp,
                                               const float* __restrict__ sinp) {
  if (pos < 0) return;
  const int D2 = D >> 1;
  const float2* cr = reinterpret_cast<const float2*>(cosp + static_cast<size_t>(pos) * D2);
  const float2* sr = reinterpret_cast<const float2*>(sinp + static_cast<size_t>(pos) * D2);
#pragma unroll 4
  for (int g = 0; g < (D >> 2); ++g) {
    const float2 c = __ldg(cr + g), s = __ldg(sr + g);
    const uint32_t a = tile + f32_off(r, g);
    const float4 x = lds_f4(a);
    const float4 y = make_float4(x.x * c.x - x.y * s.x, x.y * c.x + x.x * s.x,
                                 x.z * c.y - x.w * s.y, x.w * c.y + x.z * s.y);
    sts_u4(a, make_uint4(__float_as_uint(y.x), __float_as_uint(y.y), __float_as_uint(y.z),
                         __float_as_uint(y.w)));
  }
}

// ============================================================== forward

constexpr int kT32Threads = 256;

template <int NC>
struct T32FwdSmem {
  static constexpr int KS = (NC <= 2) ? 2 : 1;   // K/V ring stages
  uint8_t q[NC][kChunkBytes];
  uint8_t k[KS][NC][kChunkBytes];
  uint8_t v[KS][NC][kChunkBytes];
  uint64_t q_full, q_ready;
  uint64_t kv_full[KS], kv_empty[KS], k_ready[KS];
  uint64_t s_full, p_full, o_full;
  uint32_t tmem_base;
  int abort_flag;
};

struct T32FwdParams {
  const float* cosp;
  const float* sinp;
  float* o;
  float* lse;
  int N, D, nqt, nkv, has_cls;
  float c2;
};

// One CTA per (head, 128-query tile). Warp 0: TMA producer; warp 1: TMEM
// allocator and MMA issuer; warps 2-3: RoPE of the Q tile and of each K tile
// in shared memory; warps 4-7: online softmax (thread = query row = TMEM
// lane), P written back over S as float32, O accumulated in registers from
// the per-tile P V, O / l and the LSE written at the end.
// TMEM: S (and P) in columns [0, 128), the per-tile P V in [128, 128 + DP).
template <int NC>
__global__ void __launch_bounds__(kT32Threads, 1)
    fwd_tf32_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const T32FwdParams prm) {
  using Sm = T32FwdSmem<NC>;
  constexpr int KS = Sm::KS;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Sm* smp = aligned_smem<Sm>(smem_raw);
  if (smp == nullptr) return;
  Sm& sm = *smp;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bh = blockIdx.x / prm.nqt;
  const int qt = blockIdx.x - bh * prm.nqt;
  const int N = prm.N, D = prm.D;
  const int DP = (D + 15) & ~15;
  const int nkv = prm.nkv;
  volatile int* abort_flag = &sm.abort_flag;

  if (threadIdx.x == 0) {
    sm.abort_flag = 0;
    mbar_init(&sm.q_full, 1);
    mbar_init(&sm.q_ready, 1);
    for (int s = 0; s < KS; ++s) {
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
    tmem_alloc(&sm.tmem_base, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const uint32_t tS = tmem, tO = tmem + 128;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(&sm.q_full, NC * kChunkBytes);
      for (int c = 0; c < NC; ++c)
        tma_load_3d(sm.q[c], &tm_q, &sm.q_full, 32 * c, qt * kTile, bh);
      for (int j = 0; j < nkv; ++j) {
        const int s = j % KS;
        mbar_wait(&sm.kv_empty[s], ((j / KS) & 1) ^ 1, abort_flag);
        mbar_arrive_expect_tx(&sm.kv_full[s], 2 * NC * kChunkBytes);
        for (int c = 0; c < NC; ++c) {
          tma_load_3d(sm.k[s][c], &tm_k, &sm.kv_full[s], 32 * c, j * kTile, bh);
          tma_load_3d(sm.v[s][c], &tm_v, &sm.kv_full[s], 32 * c, j * kTile, bh);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idS = idesc_tf32(128, 128, false, false);
      const uint32_t idO = idesc_tf32(128, DP, false, true);
      const int ksteps = DP >> 3;   // K8 steps over the head dim
      mbar_wait(&sm.q_ready, 0, abort_flag);
      for (int j = 0; j <= nkv; ++j) {
        if (j > 0) {
          // O_j-1 = P V_j-1 : A = P in TMEM (float32 read as TF32), B = V
          // [kv][d] MN-major (32-byte-atom swizzle; 8 kv rows per K step).
          const int s = (j - 1) % KS;
          mbar_wait(&sm.p_full, (j - 1) & 1, abort_flag);
          tc_fence_after();
#pragma unroll 1
          for (int kk = 0; kk < kTile / 8; ++kk)
            mma_tf32_ts(tO, tS + 8 * kk, mn32_desc(smem_u32(sm.v[s][0]) + kk * 1024, kChunkBytes),
                        idO, kk > 0);
          mma_commit(&sm.o_full);
          mma_commit(&sm.kv_empty[s]);
        }
        if (j < nkv) {
          // S_j = Q^ K^_j^T (both K-major); overwrites P_j-1 after the P V
          // above has read it (same pipe, in order).
          const int s = j % KS;
          mbar_wait(&sm.k_ready[s], (j / KS) & 1, abort_flag);
          tc_fence_after();
#pragma unroll 1
          for (int kk = 0; kk < ksteps; ++kk) {
            const uint32_t off = (kk >> 2) * kChunkBytes + (kk & 3) * 32;
            mma_tf32_ss(tS, sw128_desc(smem_u32(sm.q[0]) + off, 16, 1024),
                        sw128_desc(smem_u32(sm.k[s][0]) + off, 16, 1024), idS, kk > 0);
          }
          mma_commit(&sm.s_full);
        }
      }
    }
  } else if (warp < 4) {
    // Rotation warps: 64 threads, thread t rotates rows t and t + 64.
    const int t = threadIdx.x - 64;
    mbar_wait(&sm.q_full, 0, abort_flag);
    for (int rr = t; rr < kTile; rr += 64)
      rotate_row_f32(smem_u32(sm.q[0]), rr, rope_pos(qt * kTile + rr, N, prm.has_cls), D,
                     prm.cosp, prm.sinp);
    fence_proxy_async_smem();
    named_bar(1, 64);
    if (t == 0) mbar_arrive(&sm.q_ready);
    for (int j = 0; j < nkv; ++j) {
      const int s = j % KS;
      mbar_wait(&sm.kv_full[s], (j / KS) & 1, abort_flag);
      for (int rr = t; rr < kTile; rr += 64)
        rotate_row_f32(smem_u32(sm.k[s][0]), rr, rope_pos(j * kTile + rr, N, prm.has_cls), D,
                       prm.cosp, prm.sinp);
      fence_proxy_async_smem();
      named_bar(1, 64);
      if (t == 0) mbar_arrive(&sm.k_ready[s]);
    }
  } else {
    // Softmax warpgroup: thread = query row = TMEM lane.
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const bool leader = threadIdx.x == 128;
    const int qrow = qt * kTile + r;
    const float c2 = prm.c2;
    float o_acc[32 * NC];
#pragma unroll
    for (int i = 0; i < 32 * NC; ++i) o_acc[i] = 0.f;
    float m2 = -INFINITY, l = 0.f;
    for (int j = 0; j < nkv; ++j) {
      const int nvalid = min(kTile, N - j * kTile);
      mbar_wait(&sm.s_full, j & 1, abort_flag);
      tc_fence_after();
      float mx = -INFINITY;
#pragma unroll 1
      for (int cb = 0; cb < 4; ++cb) {
        float sv[32];
        tmem_ld32(tS + lane_off + 32 * cb, sv);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (32 * cb + i < nvalid) mx = fmaxf(mx, sv[i]);
      }
      const float m_new = fmaxf(m2, mx * c2);
      const float alpha = ex2(m2 - m_new);
      float sum = 0.f;
#pragma unroll 1
      for (int cb = 0; cb < 4; ++cb) {
        float sv[32];
        tmem_ld32(tS + lane_off + 32 * cb, sv);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float p = (32 * cb + i < nvalid) ? ex2(fmaf(sv[i], c2, -m_new)) : 0.f;
          sum += p;
          sv[i] = p;
        }
        tmem_st32f(tS + lane_off + 32 * cb, sv);
      }
      tmem_wait_st();
      l = l * alpha + sum;
      m2 = m_new;
      tc_fence_before();
      named_bar(2, 128);
      if (leader) mbar_arrive(&sm.p_full);
      mbar_wait(&sm.o_full, j & 1, abort_flag);
      tc_fence_after();
#pragma unroll
      for (int cb = 0; cb < NC; ++cb) {
        if (32 * cb < DP) {
          float ov[32];
          tmem_ld32(tO + lane_off + 32 * cb, ov);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o_acc[32 * cb + i] = fmaf(o_acc[32 * cb + i], alpha, ov[i]);
        }
      }
      tc_fence_before();
      named_bar(2, 128);   // O read before the next P V overwrites it
    }
    if (qrow < N) {
      const size_t row = static_cast<size_t>(bh) * N + qrow;
      prm.lse[row] = (m2 + lg2(l)) * 0.69314718055994531f;
      const float inv_l = 1.f / l;
      float4* dst = reinterpret_cast<float4*>(prm.o + row * D);
#pragma unroll
      for (int g = 0; g < 8 * NC; ++g)
        if (4 * g < D)
          dst[g] = make_float4(o_acc[4 * g] * inv_l, o_acc[4 * g + 1] * inv_l,
                               o_acc[4 * g + 2] * inv_l, o_acc[4 * g + 3] * inv_l);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

template <int NC>
cudaError_t launch_fwd_tf32_t(const LaunchShape& s, const CUtensorMap& tm_q,
                              const CUtensorMap& tm_k, const CUtensorMap& tm_v, const float* cosp,
                              const float* sinp, float* o, float* lse, cudaStream_t stream) {
  T32FwdParams p;
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
  const size_t smem = sizeof(T32FwdSmem<NC>) + 1024;
  auto kern = fwd_tf32_kernel<NC>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const long long units = static_cast<long long>(s.BH) * p.nqt;
  kern<<<static_cast<unsigned>(units), kT32Threads, smem, stream>>>(tm_q, tm_k, tm_v, p);
  return cudaGetLastError();
}


}  // namespace

cudaError_t launch_fwd_tf32(const LaunchShape& s, const CUtensorMap& tm_q,
                            const CUtensorMap& tm_k, const CUtensorMap& tm_v, const float* cosp,
                            const float* sinp, float* o, float* lse, cudaStream_t stream) {
  switch ((s.D + 31) / 32) {
    case 1: return launch_fwd_tf32_t<1>(s, tm_q, tm_k, tm_v, cosp, sinp, o, lse, stream);
    case 2: return launch_fwd_tf32_t<2>(s, tm_q, tm_k, tm_v, cosp, sinp, o, lse, stream);
    case 3: return launch_fwd_tf32_t<3>(s, tm_q, tm_k, tm_v, cosp, sinp, o, lse, stream);
    default: return launch_fwd_tf32_t<4>(s, tm_q, tm_k, tm_v, cosp, sinp, o, lse, stream);
  }
}

}  // namespace frsa
