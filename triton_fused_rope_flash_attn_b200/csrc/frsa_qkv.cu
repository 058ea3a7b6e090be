// The step before the attention: the QKV projection with 2D RoPE applied in
// its epilogue.
//
//   qkv[m, f] = sum_c x[m, c] W[f, c] + bias[f]      (m = b N + n, f < 3 C)
//   q = R(qkv[:, 0:C]), k = R(qkv[:, C:2C]), v = qkv[:, 2C:3C], split into
//   heads and written as [B, H, N, D] (the attention's layout)
//
// R is the reference's pair rotation for token n (table row n - has_cls, the
// CLS token untouched; fa_rope_full .py:177-179, 201-202). With q and k
// rotated here, the attention runs with identity tables, so the rotation
// leaves the attention kernels' critical path.
//
// One CTA per 128 x 128 output tile: warp 0 streams x and W tiles (128 rows x
// 64 columns, 128-byte swizzle) through a 3-stage TMA ring, warp 1 issues
// tcgen05.mma (M = 128 tokens, N = 128 features, K16 steps, f32 accumulator in
// TMEM), warps 4-7 run the epilogue (thread = token row = TMEM lane). A tile
// of 128 features is two heads of one of q, k, v when C and D divide 128.
#include "frsa_internal.h"
#include "frsa_ptx.cuh"

namespace frsa {

namespace {

constexpr int kQkvThreads = 256;
constexpr int kQkvStages = 3;

struct QkvSmem {
  uint8_t a[kQkvStages][kChunkBytes];   // x tile: 128 tokens x 64 channels
  uint8_t b[kQkvStages][kChunkBytes];   // W tile: 128 features x 64 channels
  uint64_t full[kQkvStages], empty[kQkvStages], acc_full;
  uint32_t tmem_base;
  int abort_flag;
};

struct QkvParams {
  const float* bias;   // [3 C] float32
  const float* cosp;
  const float* sinp;
  void* q;
  void* k;
  void* v;
  long long M;         // B * N tokens
  int N, C, H, D, has_cls, kblocks;
};

template <typename T>
__global__ void __launch_bounds__(kQkvThreads, 1)
    qkv_rope_kernel(const __grid_constant__ CUtensorMap tm_x,
                    const __grid_constant__ CUtensorMap tm_w, const QkvParams prm) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  QkvSmem* smp = aligned_smem<QkvSmem>(smem_raw);
  if (smp == nullptr) return;
  QkvSmem& sm = *smp;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int mt = blockIdx.x, ft = blockIdx.y;   // token tile, feature tile
  const int nk = prm.kblocks;
  volatile int* abort_flag = &sm.abort_flag;

  if (threadIdx.x == 0) {
    sm.abort_flag = 0;
    for (int s = 0; s < kQkvStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    mbar_init(&sm.acc_full, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_x);
      tma_prefetch_desc(&tm_w);
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % kQkvStages;
        mbar_wait(&sm.empty[s], ((kb / kQkvStages) & 1) ^ 1, abort_flag);
        mbar_arrive_expect_tx(&sm.full[s], 2 * kChunkBytes);
        tma_load_2d(sm.a[s], &tm_x, &sm.full[s], kb * 64, mt * kTile);
        tma_load_2d(sm.b[s], &tm_w, &sm.full[s], kb * 64, ft * kTile);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id = idesc_f16(Elt<T>::kBf16, 128, 128, false, false);
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % kQkvStages;
        mbar_wait(&sm.full[s], (kb / kQkvStages) & 1, abort_flag);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_ss(tmem, sw128_desc(smem_u32(sm.a[s]) + kk * 32, 16, 1024),
                 sw128_desc(smem_u32(sm.b[s]) + kk * 32, 16, 1024), id, (kb | kk) != 0);
        mma_commit(&sm.empty[s]);   // stage s free once these products have read it
      }
      mma_commit(&sm.acc_full);
    }
  } else if (warp >= 4) {
    // Epilogue: thread = token row r of the tile = TMEM lane.
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const long long m = static_cast<long long>(mt) * kTile + r;
    mbar_wait(&sm.acc_full, 0, abort_flag);
    tc_fence_after();
    // tcgen05.ld is warp-collective: every lane loads; only rows that are
    // tokens (m < M) are stored.
    const bool valid = m < prm.M;
    const int C = prm.C, D = prm.D, N = prm.N;
    const long long mm = valid ? m : 0;
    const int b = static_cast<int>(mm / N), n = static_cast<int>(mm - static_cast<long long>(b) * N);
    const int f0 = ft * kTile;
    const int which = f0 / C;                  // 0 q, 1 k, 2 v
    const bool rot = which < 2;
    const int pos = (prm.has_cls && n == 0) ? -1 : n - prm.has_cls;
    T* dstbase = static_cast<T*>(which == 0 ? prm.q : which == 1 ? prm.k : prm.v);
    const int D2 = D >> 1;
#pragma unroll 1
    for (int c32 = 0; c32 < 4; ++c32) {
      float v[32];
      tmem_ld32(tmem + lane_off + 32 * c32, v);
      tmem_wait_ld();
      if (!valid) continue;
      const int fc = f0 + 32 * c32;            // first feature of these 32
      const int h = (fc % C) / D, d0 = fc % D; // head and first head-dim index
#pragma unroll
      for (int e = 0; e < 32; ++e) v[e] += __ldg(prm.bias + fc + e);
      if (rot && pos >= 0) {
        const float* cr = prm.cosp + static_cast<size_t>(pos) * D2 + (d0 >> 1);
        const float* sr = prm.sinp + static_cast<size_t>(pos) * D2 + (d0 >> 1);
#pragma unroll
        for (int p = 0; p < 16; ++p) {
          const float c = __ldg(cr + p), s = __ldg(sr + p);
          const float e0 = v[2 * p], o0 = v[2 * p + 1];
          v[2 * p] = e0 * c - o0 * s;
          v[2 * p + 1] = o0 * c + e0 * s;
        }
      }
      T* dst = dstbase + ((static_cast<size_t>(b) * prm.H + h) * N + n) * D + d0;
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) w[e] = Elt<T>::pack(v[8 * g + 2 * e], v[8 * g + 2 * e + 1]);
        reinterpret_cast<uint4*>(dst)[g] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

}  // namespace

cudaError_t launch_qkv_rope(bool bf16, const CUtensorMap& tm_x, const CUtensorMap& tm_w,
                            const float* bias, const float* cosp, const float* sinp, void* q,
                            void* k, void* v, long long M, int N, int C, int H, int D,
                            int has_cls, cudaStream_t stream) {
  QkvParams p;
  p.bias = bias;
  p.cosp = cosp;
  p.sinp = sinp;
  p.q = q;
  p.k = k;
  p.v = v;
  p.M = M;
  p.N = N;
  p.C = C;
  p.H = H;
  p.D = D;
  p.has_cls = has_cls;
  p.kblocks = C / 64;
  const size_t smem = sizeof(QkvSmem) + 1024;
  const dim3 grid(static_cast<unsigned>((M + kTile - 1) / kTile), static_cast<unsigned>(3 * C / kTile));
  if (bf16) {
    auto kern = qkv_rope_kernel<__nv_bfloat16>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    kern<<<grid, kQkvThreads, smem, stream>>>(tm_x, tm_w, p);
  } else {
    auto kern = qkv_rope_kernel<__half>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    kern<<<grid, kQkvThreads, smem, stream>>>(tm_x, tm_w, p);
  }
  return cudaGetLastError();
}

}  // namespace frsa
