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
// These kernels favour simplicity over speed (one CTA per tile unit, no
// persistence): float32 compute is the reference's slow, accurate mode.
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
  int H, N, D, nqt, nkv, has_cls;
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
        tma_load_bh(sm.q[c], &tm_q, &sm.q_full, 32 * c, qt * kTile, bh, prm.H);
      for (int j = 0; j < nkv; ++j) {
        const int s = j % KS;
        mbar_wait(&sm.kv_empty[s], ((j / KS) & 1) ^ 1, abort_flag);
        mbar_arrive_expect_tx(&sm.kv_full[s], 2 * NC * kChunkBytes);
        for (int c = 0; c < NC; ++c) {
          tma_load_bh(sm.k[s][c], &tm_k, &sm.kv_full[s], 32 * c, j * kTile, bh, prm.H);
          tma_load_bh(sm.v[s][c], &tm_v, &sm.kv_full[s], 32 * c, j * kTile, bh, prm.H);
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
  p.H = s.H;
  p.N = s.N;
  p.D = s.D;
  p.nqt = (s.N + kTile - 1) / kTile;
  p.nkv = p.nqt;
  p.has_cls = s.has_cls;
  p.c2 = s.scale * 1.4426950408889634f;
  const size_t smem = sizeof(T32FwdSmem<NC>) + 1024;
  auto kern = fwd_tf32_kernel<NC>;
  cudaError_t e = set_max_dynamic_smem_once(kern, smem);
  if (e != cudaSuccess) return e;
  const long long units = static_cast<long long>(s.BH) * p.nqt;
  kern<<<static_cast<unsigned>(units), kT32Threads, smem, stream>>>(tm_q, tm_k, tm_v, p);
  return cudaGetLastError();
}



// ============================================================== backward
//
// Split like the reference's backward (fa_rope_full .py:325-1009): a Delta
// pass, a dK/dV kernel over key tiles (thread = key row) and a dQ kernel over
// query tiles (thread = query row). Operands read both K-major and MN-major
// are loaded twice, once per shared layout.

// Byte offset of granule g (floats 4g..4g+3) of row r in a multi-chunk 32-bit
// tile stored in the 32-byte-atom swizzle (MN-major operand layout).
__device__ __forceinline__ uint32_t f32_off_a32(int r, int g) {
  return static_cast<uint32_t>(g >> 3) * kChunkBytes + static_cast<uint32_t>(r) * 128u +
         ((static_cast<uint32_t>((g & 7) >> 1) ^ (static_cast<uint32_t>(r) & 3u)) << 5) +
         (static_cast<uint32_t>(g & 1) << 4);
}

// rotate_row_f32 for a tile in the 32-byte-atom layout.
__device__ __forceinline__ void rotate_row_f32_a32(uint32_t tile, int r, int pos, int D,
                                                   const float* __restrict__ cosp,
                                                   const float* __restrict__ sinp) {
  if (pos < 0) return;
  const int D2 = D >> 1;
  const float2* cr = reinterpret_cast<const float2*>(cosp + static_cast<size_t>(pos) * D2);
  const float2* sr = reinterpret_cast<const float2*>(sinp + static_cast<size_t>(pos) * D2);
#pragma unroll 4
  for (int g = 0; g < (D >> 2); ++g) {
    const float2 c = __ldg(cr + g), s = __ldg(sr + g);
    const uint32_t a = tile + f32_off_a32(r, g);
    const float4 x = lds_f4(a);
    const float4 y = make_float4(x.x * c.x - x.y * s.x, x.y * c.x + x.x * s.x,
                                 x.z * c.y - x.w * s.y, x.w * c.y + x.z * s.y);
    sts_u4(a, make_uint4(__float_as_uint(y.x), __float_as_uint(y.y), __float_as_uint(y.z),
                         __float_as_uint(y.w)));
  }
}

// A row of a TMEM accumulator ([tcol, tcol + 32 NC) of this thread's lane),
// times `scale`, un-rotated with R^T for token position pos (pos < 0: as is),
// stored as D floats to dst when `store` (fa_rope_full .py:640-662, 974-993).
// tcgen05.ld is warp-collective: every lane of the warp must call this; lanes
// whose row is not a token pass store = false.
template <int NC>
__device__ __forceinline__ void drain_row_f32(uint32_t tcol, float scale, int pos, int D,
                                              const float* __restrict__ cosp,
                                              const float* __restrict__ sinp, float* dst,
                                              bool store) {
  const int D2 = D >> 1;
#pragma unroll 1
  for (int cb = 0; cb < NC; ++cb) {
    float v[32];
    tmem_ld32(tcol + 32 * cb, v);
    tmem_wait_ld();
    if (!store) continue;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      const int gg = 8 * cb + g;
      if (4 * gg < D) {
        float4 y = make_float4(v[4 * g] * scale, v[4 * g + 1] * scale, v[4 * g + 2] * scale,
                               v[4 * g + 3] * scale);
        if (pos >= 0) {
          const float2 c = __ldg(reinterpret_cast<const float2*>(cosp + static_cast<size_t>(pos) * D2) + gg);
          const float2 s = __ldg(reinterpret_cast<const float2*>(sinp + static_cast<size_t>(pos) * D2) + gg);
          y = make_float4(y.x * c.x + y.y * s.x, y.y * c.x - y.x * s.x, y.z * c.y + y.w * s.y,
                          y.w * c.y - y.z * s.y);
        }
        reinterpret_cast<float4*>(dst)[gg] = y;
      }
    }
  }
}

// Delta = rowsum(dO O) (fa_rope_full .py:325-357), one thread per row.
__global__ void delta_f32_kernel(const float* __restrict__ o, const float* __restrict__ d_o,
                                 float* __restrict__ delta, long long rows, int D) {
  const long long row = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const float4* a = reinterpret_cast<const float4*>(o + row * D);
  const float4* b = reinterpret_cast<const float4*>(d_o + row * D);
  float acc = 0.f;
  for (int g = 0; g < (D >> 2); ++g) {
    const float4 x = __ldg(a + g), y = __ldg(b + g);
    acc = fmaf(x.x, y.x, fmaf(x.y, y.y, fmaf(x.z, y.z, fmaf(x.w, y.w, acc))));
  }
  delta[row] = acc;
}

struct T32BwdParams {
  const float* cosp;
  const float* sinp;
  const float* lse;
  const float* delta;
  float* dq;
  float* dk;
  float* dv;
  int H, N, D, nqt, nkv, has_cls;
  float c2, scale;
};

template <int NC>
struct T32KvSmem {
  uint8_t k[NC][kChunkBytes];    // K^_j, K-major layout
  uint8_t v[NC][kChunkBytes];    // V_j, K-major layout
  uint8_t qa[NC][kChunkBytes];   // Q^_i, K-major layout (S^T)
  uint8_t qb[NC][kChunkBytes];   // Q^_i, MN-major layout (dK)
  uint8_t da[NC][kChunkBytes];   // dO_i, K-major layout (dP^T)
  uint8_t db[NC][kChunkBytes];   // dO_i, MN-major layout (dV)
  float lse2[kTile];
  float delta[kTile];
  uint64_t kv_full, k_ready, q_full, q_ready, q_empty, st_full, p_full, acc_full;
  uint32_t tmem_base;
  int abort_flag;
};

// dK, dV of key tile j of head bh, over all query tiles. TMEM: S^T [0,128)
// (then P^T), dP^T [128,256) (then dS^T), dV [256, 256+DP), dK^ [384, 384+DP).
template <int NC>
__global__ void __launch_bounds__(kT32Threads, 1)
    bwd_kv_tf32_kernel(const __grid_constant__ CUtensorMap tm_k16,
                       const __grid_constant__ CUtensorMap tm_v16,
                       const __grid_constant__ CUtensorMap tm_q16,
                       const __grid_constant__ CUtensorMap tm_q32,
                       const __grid_constant__ CUtensorMap tm_do16,
                       const __grid_constant__ CUtensorMap tm_do32, const T32BwdParams prm) {
  using Sm = T32KvSmem<NC>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Sm* smp = aligned_smem<Sm>(smem_raw);
  if (smp == nullptr) return;
  Sm& sm = *smp;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bh = blockIdx.x / prm.nkv;
  const int jt = blockIdx.x - bh * prm.nkv;
  const int N = prm.N, D = prm.D;
  const int DP = (D + 15) & ~15;
  const int nqt = prm.nqt;
  volatile int* abort_flag = &sm.abort_flag;

  if (threadIdx.x == 0) {
    sm.abort_flag = 0;
    mbar_init(&sm.kv_full, 1);
    mbar_init(&sm.k_ready, 1);
    mbar_init(&sm.q_full, 1);
    mbar_init(&sm.q_ready, 1);
    mbar_init(&sm.q_empty, 1);
    mbar_init(&sm.st_full, 1);
    mbar_init(&sm.p_full, 1);
    mbar_init(&sm.acc_full, 1);
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
  const uint32_t tS = tmem, tDP = tmem + 128, tDV = tmem + 256, tDK = tmem + 384;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(&sm.kv_full, 2 * NC * kChunkBytes);
      for (int c = 0; c < NC; ++c) {
        tma_load_bh(sm.k[c], &tm_k16, &sm.kv_full, 32 * c, jt * kTile, bh, prm.H);
        tma_load_bh(sm.v[c], &tm_v16, &sm.kv_full, 32 * c, jt * kTile, bh, prm.H);
      }
      for (int i = 0; i < nqt; ++i) {
        mbar_wait(&sm.q_empty, (i & 1) ^ 1, abort_flag);
        mbar_arrive_expect_tx(&sm.q_full, 4 * NC * kChunkBytes);
        for (int c = 0; c < NC; ++c) {
          tma_load_bh(sm.qa[c], &tm_q16, &sm.q_full, 32 * c, i * kTile, bh, prm.H);
          tma_load_bh(sm.qb[c], &tm_q32, &sm.q_full, 32 * c, i * kTile, bh, prm.H);
          tma_load_bh(sm.da[c], &tm_do16, &sm.q_full, 32 * c, i * kTile, bh, prm.H);
          tma_load_bh(sm.db[c], &tm_do32, &sm.q_full, 32 * c, i * kTile, bh, prm.H);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idS = idesc_tf32(128, 128, false, false);
      const uint32_t idG = idesc_tf32(128, DP, false, true);
      const int ksteps = DP >> 3;
      mbar_wait(&sm.k_ready, 0, abort_flag);
      for (int i = 0; i < nqt; ++i) {
        mbar_wait(&sm.q_ready, i & 1, abort_flag);
        tc_fence_after();
        // S^T = K^ Q^^T, dP^T = V dO^T (all K-major).
#pragma unroll 1
        for (int kk = 0; kk < ksteps; ++kk) {
          const uint32_t off = (kk >> 2) * kChunkBytes + (kk & 3) * 32;
          mma_tf32_ss(tS, sw128_desc(smem_u32(sm.k[0]) + off, 16, 1024),
                      sw128_desc(smem_u32(sm.qa[0]) + off, 16, 1024), idS, kk > 0);
          mma_tf32_ss(tDP, sw128_desc(smem_u32(sm.v[0]) + off, 16, 1024),
                      sw128_desc(smem_u32(sm.da[0]) + off, 16, 1024), idS, kk > 0);
        }
        mma_commit(&sm.st_full);
        mbar_wait(&sm.p_full, i & 1, abort_flag);
        tc_fence_after();
        // dV += P dO, dK^ += dS Q^ : A = P^T / dS^T in TMEM (lane = key), B =
        // dO / Q^ [query][d] MN-major (8 query rows per K step).
#pragma unroll 1
        for (int kk = 0; kk < kTile / 8; ++kk) {
          const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
          mma_tf32_ts(tDV, tS + 8 * kk, mn32_desc(smem_u32(sm.db[0]) + kk * 1024, kChunkBytes),
                      idG, acc);
          mma_tf32_ts(tDK, tDP + 8 * kk, mn32_desc(smem_u32(sm.qb[0]) + kk * 1024, kChunkBytes),
                      idG, acc);
        }
        mma_commit(&sm.q_empty);
      }
      mma_commit(&sm.acc_full);
    }
  } else if (warp < 4) {
    const int t = threadIdx.x - 64;
    mbar_wait(&sm.kv_full, 0, abort_flag);
    for (int rr = t; rr < kTile; rr += 64)
      rotate_row_f32(smem_u32(sm.k[0]), rr, rope_pos(jt * kTile + rr, N, prm.has_cls), D,
                     prm.cosp, prm.sinp);
    fence_proxy_async_smem();
    named_bar(1, 64);
    if (t == 0) mbar_arrive(&sm.k_ready);
    for (int i = 0; i < nqt; ++i) {
      mbar_wait(&sm.q_full, i & 1, abort_flag);
      for (int rr = t; rr < kTile; rr += 64) {
        const int tok = i * kTile + rr;
        const int pos = rope_pos(tok, N, prm.has_cls);
        rotate_row_f32(smem_u32(sm.qa[0]), rr, pos, D, prm.cosp, prm.sinp);
        rotate_row_f32_a32(smem_u32(sm.qb[0]), rr, pos, D, prm.cosp, prm.sinp);
        // Padded query rows get lse2 = +inf: their P (and dS) is exactly 0.
        const size_t row = static_cast<size_t>(bh) * N + tok;
        sm.lse2[rr] = (tok < N) ? prm.lse[row] * 1.4426950408889634f : INFINITY;
        sm.delta[rr] = (tok < N) ? prm.delta[row] : 0.f;
      }
      fence_proxy_async_smem();
      named_bar(1, 64);
      if (t == 0) mbar_arrive(&sm.q_ready);
    }
  } else {
    // Elementwise warps: thread = key row = TMEM lane.
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const bool leader = threadIdx.x == 128;
    const float c2 = prm.c2;
    for (int i = 0; i < nqt; ++i) {
      mbar_wait(&sm.st_full, i & 1, abort_flag);
      tc_fence_after();
#pragma unroll 1
      for (int cb = 0; cb < 4; ++cb) {
        float sv[32], dp[32];
        tmem_ld32(tS + lane_off + 32 * cb, sv);
        tmem_ld32(tDP + lane_off + 32 * cb, dp);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float p = ex2(fmaf(sv[e], c2, -sm.lse2[32 * cb + e]));
          sv[e] = p;
          dp[e] = p * (dp[e] - sm.delta[32 * cb + e]);
        }
        tmem_st32f(tS + lane_off + 32 * cb, sv);
        tmem_st32f(tDP + lane_off + 32 * cb, dp);
      }
      tmem_wait_st();
      tc_fence_before();
      named_bar(2, 128);
      if (leader) mbar_arrive(&sm.p_full);
    }
    mbar_wait(&sm.acc_full, 0, abort_flag);
    tc_fence_after();
    const int tok = jt * kTile + r;
    const bool valid = tok < N;
    const size_t row = static_cast<size_t>(bh) * N + (valid ? tok : 0);
    drain_row_f32<NC>(tDV + lane_off, 1.f, -1, D, prm.cosp, prm.sinp, prm.dv + row * D, valid);
    drain_row_f32<NC>(tDK + lane_off, prm.scale, rope_pos(tok, N, prm.has_cls), D, prm.cosp,
                      prm.sinp, prm.dk + row * D, valid);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int NC>
struct T32QSmem {
  uint8_t q[NC][kChunkBytes];    // Q^_i, K-major
  uint8_t d[NC][kChunkBytes];    // dO_i, K-major
  uint8_t ka[NC][kChunkBytes];   // K^_j, K-major (S)
  uint8_t kb[NC][kChunkBytes];   // K^_j, MN-major (dQ)
  uint8_t v[NC][kChunkBytes];    // V_j, K-major (dP)
  uint64_t q_full, q_ready, kv_full, k_ready, kv_empty, st_full, p_full, acc_full;
  uint32_t tmem_base;
  int abort_flag;
};

// dQ of query tile i of head bh, over all key tiles. TMEM: S [0,128) (then
// dS), dP [128,256), dQ^ [256, 256+DP).
template <int NC>
__global__ void __launch_bounds__(kT32Threads, 1)
    bwd_q_tf32_kernel(const __grid_constant__ CUtensorMap tm_q16,
                      const __grid_constant__ CUtensorMap tm_do16,
                      const __grid_constant__ CUtensorMap tm_k16,
                      const __grid_constant__ CUtensorMap tm_k32,
                      const __grid_constant__ CUtensorMap tm_v16, const T32BwdParams prm) {
  using Sm = T32QSmem<NC>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Sm* smp = aligned_smem<Sm>(smem_raw);
  if (smp == nullptr) return;
  Sm& sm = *smp;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bh = blockIdx.x / prm.nqt;
  const int it = blockIdx.x - bh * prm.nqt;
  const int N = prm.N, D = prm.D;
  const int DP = (D + 15) & ~15;
  const int nkv = prm.nkv;
  volatile int* abort_flag = &sm.abort_flag;

  if (threadIdx.x == 0) {
    sm.abort_flag = 0;
    mbar_init(&sm.q_full, 1);
    mbar_init(&sm.q_ready, 1);
    mbar_init(&sm.kv_full, 1);
    mbar_init(&sm.k_ready, 1);
    mbar_init(&sm.kv_empty, 1);
    mbar_init(&sm.st_full, 1);
    mbar_init(&sm.p_full, 1);
    mbar_init(&sm.acc_full, 1);
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
  const uint32_t tS = tmem, tDP = tmem + 128, tDQ = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(&sm.q_full, 2 * NC * kChunkBytes);
      for (int c = 0; c < NC; ++c) {
        tma_load_bh(sm.q[c], &tm_q16, &sm.q_full, 32 * c, it * kTile, bh, prm.H);
        tma_load_bh(sm.d[c], &tm_do16, &sm.q_full, 32 * c, it * kTile, bh, prm.H);
      }
      for (int j = 0; j < nkv; ++j) {
        mbar_wait(&sm.kv_empty, (j & 1) ^ 1, abort_flag);
        mbar_arrive_expect_tx(&sm.kv_full, 3 * NC * kChunkBytes);
        for (int c = 0; c < NC; ++c) {
          tma_load_bh(sm.ka[c], &tm_k16, &sm.kv_full, 32 * c, j * kTile, bh, prm.H);
          tma_load_bh(sm.kb[c], &tm_k32, &sm.kv_full, 32 * c, j * kTile, bh, prm.H);
          tma_load_bh(sm.v[c], &tm_v16, &sm.kv_full, 32 * c, j * kTile, bh, prm.H);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idS = idesc_tf32(128, 128, false, false);
      const uint32_t idG = idesc_tf32(128, DP, false, true);
      const int ksteps = DP >> 3;
      mbar_wait(&sm.q_ready, 0, abort_flag);
      for (int j = 0; j < nkv; ++j) {
        mbar_wait(&sm.k_ready, j & 1, abort_flag);
        tc_fence_after();
        // S = Q^ K^^T, dP = dO V^T (K-major).
#pragma unroll 1
        for (int kk = 0; kk < ksteps; ++kk) {
          const uint32_t off = (kk >> 2) * kChunkBytes + (kk & 3) * 32;
          mma_tf32_ss(tS, sw128_desc(smem_u32(sm.q[0]) + off, 16, 1024),
                      sw128_desc(smem_u32(sm.ka[0]) + off, 16, 1024), idS, kk > 0);
          mma_tf32_ss(tDP, sw128_desc(smem_u32(sm.d[0]) + off, 16, 1024),
                      sw128_desc(smem_u32(sm.v[0]) + off, 16, 1024), idS, kk > 0);
        }
        mma_commit(&sm.st_full);
        mbar_wait(&sm.p_full, j & 1, abort_flag);
        tc_fence_after();
        // dQ^ += dS K^ : A = dS in TMEM (lane = query), B = K^ [key][d] MN-major.
#pragma unroll 1
        for (int kk = 0; kk < kTile / 8; ++kk)
          mma_tf32_ts(tDQ, tS + 8 * kk, mn32_desc(smem_u32(sm.kb[0]) + kk * 1024, kChunkBytes),
                      idG, (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&sm.kv_empty);
      }
      mma_commit(&sm.acc_full);
    }
  } else if (warp < 4) {
    const int t = threadIdx.x - 64;
    mbar_wait(&sm.q_full, 0, abort_flag);
    for (int rr = t; rr < kTile; rr += 64)
      rotate_row_f32(smem_u32(sm.q[0]), rr, rope_pos(it * kTile + rr, N, prm.has_cls), D,
                     prm.cosp, prm.sinp);
    fence_proxy_async_smem();
    named_bar(1, 64);
    if (t == 0) mbar_arrive(&sm.q_ready);
    for (int j = 0; j < nkv; ++j) {
      mbar_wait(&sm.kv_full, j & 1, abort_flag);
      for (int rr = t; rr < kTile; rr += 64) {
        const int pos = rope_pos(j * kTile + rr, N, prm.has_cls);
        rotate_row_f32(smem_u32(sm.ka[0]), rr, pos, D, prm.cosp, prm.sinp);
        rotate_row_f32_a32(smem_u32(sm.kb[0]), rr, pos, D, prm.cosp, prm.sinp);
      }
      fence_proxy_async_smem();
      named_bar(1, 64);
      if (t == 0) mbar_arrive(&sm.k_ready);
    }
  } else {
    // Elementwise warps: thread = query row = TMEM lane.
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const bool leader = threadIdx.x == 128;
    const float c2 = prm.c2;
    const int tok = it * kTile + r;
    const size_t row = static_cast<size_t>(bh) * N + tok;
    // Padded query rows: lse2 = +inf gives P = dS = 0.
    const float lse2 = (tok < N) ? prm.lse[row] * 1.4426950408889634f : INFINITY;
    const float dl = (tok < N) ? prm.delta[row] : 0.f;
    for (int j = 0; j < nkv; ++j) {
      const int nvalid = min(kTile, N - j * kTile);
      mbar_wait(&sm.st_full, j & 1, abort_flag);
      tc_fence_after();
#pragma unroll 1
      for (int cb = 0; cb < 4; ++cb) {
        float sv[32], dp[32];
        tmem_ld32(tS + lane_off + 32 * cb, sv);
        tmem_ld32(tDP + lane_off + 32 * cb, dp);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          // Key columns past the sequence (zero keys) get P = 0.
          const float p = (32 * cb + e < nvalid) ? ex2(fmaf(sv[e], c2, -lse2)) : 0.f;
          sv[e] = p * (dp[e] - dl);
        }
        tmem_st32f(tS + lane_off + 32 * cb, sv);
      }
      tmem_wait_st();
      tc_fence_before();
      named_bar(2, 128);
      if (leader) mbar_arrive(&sm.p_full);
    }
    mbar_wait(&sm.acc_full, 0, abort_flag);
    tc_fence_after();
    drain_row_f32<NC>(tDQ + lane_off, prm.scale, rope_pos(tok, N, prm.has_cls), D, prm.cosp,
                      prm.sinp, prm.dq + (tok < N ? row : 0) * D, tok < N);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int NC>
cudaError_t launch_bwd_tf32_t(const LaunchShape& s, const CUtensorMap* maps, const float* o,
                              const float* d_o, const float* lse, float* delta,
                              const float* cosp, const float* sinp, float* dq, float* dk,
                              float* dv, cudaStream_t stream) {
  // maps: q16, q32, k16, k32, v16, do16, do32
  const long long rows = static_cast<long long>(s.BH) * s.N;
  delta_f32_kernel<<<static_cast<unsigned>((rows + 255) / 256), 256, 0, stream>>>(o, d_o, delta,
                                                                                  rows, s.D);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  T32BwdParams p;
  p.cosp = cosp;
  p.sinp = sinp;
  p.lse = lse;
  p.delta = delta;
  p.dq = dq;
  p.dk = dk;
  p.dv = dv;
  p.H = s.H;
  p.N = s.N;
  p.D = s.D;
  p.nqt = (s.N + kTile - 1) / kTile;
  p.nkv = p.nqt;
  p.has_cls = s.has_cls;
  p.c2 = s.scale * 1.4426950408889634f;
  p.scale = s.scale;
  {
    const size_t smem = sizeof(T32KvSmem<NC>) + 1024;
    auto kern = bwd_kv_tf32_kernel<NC>;
    e = set_max_dynamic_smem_once(kern, smem);
    if (e != cudaSuccess) return e;
    kern<<<static_cast<unsigned>(static_cast<long long>(s.BH) * p.nkv), kT32Threads, smem,
           stream>>>(maps[2], maps[4], maps[0], maps[1], maps[5], maps[6], p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  {
    const size_t smem = sizeof(T32QSmem<NC>) + 1024;
    auto kern = bwd_q_tf32_kernel<NC>;
    e = set_max_dynamic_smem_once(kern, smem);
    if (e != cudaSuccess) return e;
    kern<<<static_cast<unsigned>(static_cast<long long>(s.BH) * p.nqt), kT32Threads, smem,
           stream>>>(maps[0], maps[5], maps[2], maps[3], maps[4], p);
  }
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

bool tf32_bwd_supported(const LaunchShape& s) { return s.D <= 64; }

cudaError_t launch_bwd_tf32(const LaunchShape& s, const CUtensorMap* maps, const float* o,
                            const float* d_o, const float* lse, float* delta, const float* cosp,
                            const float* sinp, float* dq, float* dk, float* dv,
                            cudaStream_t stream) {
  return (s.D <= 32) ? launch_bwd_tf32_t<1>(s, maps, o, d_o, lse, delta, cosp, sinp, dq, dk, dv,
                                            stream)
                     : launch_bwd_tf32_t<2>(s, maps, o, d_o, lse, delta, cosp, sinp, dq, dk, dv,
                                            stream);
}

}  // namespace frsa
