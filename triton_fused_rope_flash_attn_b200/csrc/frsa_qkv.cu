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
// Persistent: one CTA per SM walks 128 x 128 output tiles (token tile major,
// so consecutive CTAs reuse a token tile of x from L2). Warp 0 streams x and W
// tiles (128 rows x 64 columns, 128-byte swizzle) through a 4-stage TMA ring;
// warp 1 issues tcgen05.mma (M = 128 tokens, N = 128 features, K16 steps)
// into one of two TMEM accumulators; warps 4-7 run the epilogue of the other
// accumulator (thread = token row = TMEM lane), so a tile's epilogue overlaps
// the next tile's products. Warps 4-7 and 8-11 are two epilogue groups, each
// taking two of the four 32-column groups of every 128 columns. A tile of 128 features lies within one of q, k, v
// when C divides by 128, and 32-column groups lie within one head when D
// divides by 32.
#include "frsa_internal.h"
#include "frsa_ptx.cuh"
#include "frsa_rope.cuh"

namespace frsa {

namespace {

constexpr int kQkvThreads = 384;
constexpr int kQkvStages = 4;

template <int BN>
struct QkvSmem {
  uint8_t a[kQkvStages][kChunkBytes];             // x tile: 128 tokens x 64 channels
  uint8_t b[kQkvStages][BN / kTile][kChunkBytes];  // W tile: BN features x 64 channels
  uint64_t full[kQkvStages], empty[kQkvStages];
  uint64_t acc_full[2], acc_empty[2];
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
  int N, C, H, D, has_cls, kblocks, nft, ntiles;
};

template <typename T, int BN>
__global__ void __launch_bounds__(kQkvThreads, 1)
    qkv_rope_kernel(const __grid_constant__ CUtensorMap tm_x,
                    const __grid_constant__ CUtensorMap tm_w, const QkvParams prm) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  QkvSmem<BN>* smp = aligned_smem<QkvSmem<BN>>(smem_raw);
  if (smp == nullptr) return;
  QkvSmem<BN>& sm = *smp;
  constexpr int NB = BN / kTile;   // 128-row W boxes per tile
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nk = prm.kblocks;
  volatile int* abort_flag = &sm.abort_flag;

  if (threadIdx.x == 0) {
    sm.abort_flag = 0;
    for (int s = 0; s < kQkvStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.acc_full[s], 1);
      mbar_init(&sm.acc_empty[s], 1);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 2 * BN);
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
      int kc = 0;   // running k-block count (ring position)
      for (int t = blockIdx.x; t < prm.ntiles; t += gridDim.x) {
        const int mt = t / prm.nft, ft = t - mt * prm.nft;
        for (int kb = 0; kb < nk; ++kb, ++kc) {
          const int s = kc % kQkvStages;
          mbar_wait(&sm.empty[s], ((kc / kQkvStages) & 1) ^ 1, abort_flag);
          mbar_arrive_expect_tx(&sm.full[s], (1 + NB) * kChunkBytes);
          tma_load_2d(sm.a[s], &tm_x, &sm.full[s], kb * 64, mt * kTile);
          for (int h = 0; h < NB; ++h)
            tma_load_2d(sm.b[s][h], &tm_w, &sm.full[s], kb * 64, ft * BN + h * kTile);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id = idesc_f16(Elt<T>::kBf16, 128, BN, false, false);
      int kc = 0, tl = 0;
      for (int t = blockIdx.x; t < prm.ntiles; t += gridDim.x, ++tl) {
        const int ab = tl & 1;   // accumulator buffer
        mbar_wait(&sm.acc_empty[ab], ((tl >> 1) & 1) ^ 1, abort_flag);
        tc_fence_after();
        for (int kb = 0; kb < nk; ++kb, ++kc) {
          const int s = kc % kQkvStages;
          mbar_wait(&sm.full[s], (kc / kQkvStages) & 1, abort_flag);
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_ss(tmem + BN * ab, sw128_desc(smem_u32(sm.a[s]) + kk * 32, 16, 1024),
                   sw128_desc(smem_u32(sm.b[s][0]) + kk * 32, 16, 1024), id, (kb | kk) != 0);
          mma_commit(&sm.empty[s]);   // stage s free once these products have read it
        }
        mma_commit(&sm.acc_full[ab]);
      }
    }
  } else if (warp >= 4) {
    // Epilogue: thread = token row r of the tile = TMEM lane. tcgen05.ld is
    // warp-collective: every lane loads; only rows that are tokens are stored.
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const bool leader = threadIdx.x == 128;
    const int eg = (warp - 4) >> 2;   // epilogue group: 32-column groups 2 eg, 2 eg + 1
    const int C = prm.C, D = prm.D, N = prm.N;
    const int D2 = D >> 1;
    int tl = 0;
    for (int t = blockIdx.x; t < prm.ntiles; t += gridDim.x, ++tl) {
      const int ab = tl & 1;
      const int mt = t / prm.nft, ft = t - mt * prm.nft;
      const long long m = static_cast<long long>(mt) * kTile + r;
      const bool valid = m < prm.M;
      const long long mm = valid ? m : 0;
      const int b = static_cast<int>(mm / N), n = static_cast<int>(mm - static_cast<long long>(b) * N);
      const int f0 = ft * BN;
      const int which = f0 / C;                  // 0 q, 1 k, 2 v
      const bool rot = which < 2;
      const int pos = (prm.has_cls && n == 0) ? -1 : n - prm.has_cls;
      T* dstbase = static_cast<T*>(which == 0 ? prm.q : which == 1 ? prm.k : prm.v);
      mbar_wait(&sm.acc_full[ab], (tl >> 1) & 1, abort_flag);
      tc_fence_after();
#pragma unroll 1
      for (int hb = 0; hb < NB; ++hb) {
        float v[2][32];
#pragma unroll
        for (int c = 0; c < 2; ++c)
          tmem_ld32(tmem + BN * ab + lane_off + 128 * hb + 32 * (2 * eg + c), v[c]);
        tmem_wait_ld();
        if (hb == NB - 1) {
          // Accumulator read: the next tile's products may overwrite it.
          tc_fence_before();
          named_bar(1, 256);
          if (leader) mbar_arrive(&sm.acc_empty[ab]);
        }
        if (!valid) continue;
#pragma unroll
        for (int c32 = 0; c32 < 2; ++c32) {
          const int fc = f0 + 128 * hb + 32 * (2 * eg + c32);  // first feature of these 32
          const int h = (fc % C) / D, d0 = fc % D;  // head and first head-dim index
          const float4* bias4 = reinterpret_cast<const float4*>(prm.bias + fc);
#pragma unroll
          for (int e4 = 0; e4 < 8; ++e4) {
            const float4 bb = __ldg(bias4 + e4);
            v[c32][4 * e4] += bb.x;
            v[c32][4 * e4 + 1] += bb.y;
            v[c32][4 * e4 + 2] += bb.z;
            v[c32][4 * e4 + 3] += bb.w;
          }
          if (rot && pos >= 0) {
            const float4* cr =
                reinterpret_cast<const float4*>(prm.cosp + static_cast<size_t>(pos) * D2 + (d0 >> 1));
            const float4* sr =
                reinterpret_cast<const float4*>(prm.sinp + static_cast<size_t>(pos) * D2 + (d0 >> 1));
#pragma unroll
            for (int p4 = 0; p4 < 4; ++p4) {
              const float4 c4 = __ldg(cr + p4), s4 = __ldg(sr + p4);
              const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const int p = 4 * p4 + q;
                const float e0 = v[c32][2 * p], o0 = v[c32][2 * p + 1];
                v[c32][2 * p] = e0 * cc[q] - o0 * ss[q];
                v[c32][2 * p + 1] = o0 * cc[q] + e0 * ss[q];
              }
            }
          }
          T* dst = dstbase + ((static_cast<size_t>(b) * prm.H + h) * N + n) * D + d0;
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
              w[e] = Elt<T>::pack(v[c32][8 * g + 2 * e], v[c32][8 * g + 2 * e + 1]);
            reinterpret_cast<uint4*>(dst)[g] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * BN);
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
  // 128 x 256 tiles when a tile of 256 features stays within one of q, k, v.
  const int BN = (C % 256 == 0) ? 256 : 128;
  p.nft = 3 * C / BN;
  const long long ntiles = ((M + kTile - 1) / kTile) * p.nft;
  p.ntiles = static_cast<int>(ntiles);
  const int nsm = device_sm_count();
  const dim3 grid(static_cast<unsigned>(ntiles < nsm ? ntiles : nsm));
  auto launch = [&](auto kern, size_t smem) -> cudaError_t {
    cudaError_t e = set_max_dynamic_smem_once(kern, smem);
    if (e != cudaSuccess) return e;
    kern<<<grid, kQkvThreads, smem, stream>>>(tm_x, tm_w, p);
    return cudaGetLastError();
  };
  if (BN == 256)
    return bf16 ? launch(qkv_rope_kernel<__nv_bfloat16, 256>, sizeof(QkvSmem<256>) + 1024)
                : launch(qkv_rope_kernel<__half, 256>, sizeof(QkvSmem<256>) + 1024);
  return bf16 ? launch(qkv_rope_kernel<__nv_bfloat16, 128>, sizeof(QkvSmem<128>) + 1024)
              : launch(qkv_rope_kernel<__half, 128>, sizeof(QkvSmem<128>) + 1024);
}

namespace {

// Backward of the projection's epilogue: the gradients of q, k, v
// ([B, H, N, D] each, with respect to the rotated q and k) become the
// gradient of the projection output, dqkv [B*N, 3C] (the layout the two
// GEMMs dx = dqkv W and dW = dqkv^T x read), with R^T applied to the q and k
// parts in f32 and one rounding. One thread per 8-element granule of a dqkv
// row: the stores are coalesced, the loads read 16 bytes of one head row.
struct QkvBwdParams {
  const void* dq;
  const void* dk;
  const void* dv;
  const float* cosp;
  const float* sinp;
  void* dqkv;
  long long M;   // B * N
  int N, C, H, D, has_cls;
};

template <typename T>
__global__ void qkv_rope_bwd_kernel(const QkvBwdParams p) {
  const int G = 3 * p.C / 8;   // granules of a dqkv row
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long m = idx / G;
  if (m >= p.M) return;
  const int f = 8 * static_cast<int>(idx - m * G);
  const int part = f / p.C, fc = f - part * p.C;
  const int h = fc / p.D, d0 = fc - h * p.D;
  const long long b = m / p.N;
  const int n = static_cast<int>(m - b * p.N);
  const void* g = part == 0 ? p.dq : (part == 1 ? p.dk : p.dv);
  const uint4 x = __ldg(reinterpret_cast<const uint4*>(
      static_cast<const T*>(g) + ((b * p.H + h) * p.N + n) * p.D + d0));
  float v[8];
  const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 t = Elt<T>::unpack(w[e]);
    v[2 * e] = t.x;
    v[2 * e + 1] = t.y;
  }
  const int pos = part < 2 ? rope_pos(n, p.N, p.has_cls) : -1;
  if (pos >= 0) {
    const size_t t0 = static_cast<size_t>(pos) * (p.D >> 1) + (d0 >> 1);
    unrotate8(v, __ldg(reinterpret_cast<const float4*>(p.cosp + t0)),
              __ldg(reinterpret_cast<const float4*>(p.sinp + t0)));
  }
  reinterpret_cast<uint4*>(static_cast<T*>(p.dqkv) + m * 3 * p.C + f)[0] = pack8<T>(v);
}

}  // namespace

cudaError_t launch_qkv_rope_bwd(bool bf16, const void* dq, const void* dk, const void* dv,
                                const float* cosp, const float* sinp, void* dqkv, long long M,
                                int N, int C, int H, int D, int has_cls, cudaStream_t stream) {
  QkvBwdParams p;
  p.dq = dq;
  p.dk = dk;
  p.dv = dv;
  p.cosp = cosp;
  p.sinp = sinp;
  p.dqkv = dqkv;
  p.M = M;
  p.N = N;
  p.C = C;
  p.H = H;
  p.D = D;
  p.has_cls = has_cls;
  const long long threads = M * (3LL * C / 8);
  if (threads == 0) return cudaSuccess;
  const unsigned blocks = static_cast<unsigned>((threads + 255) / 256);
  if (bf16)
    qkv_rope_bwd_kernel<__nv_bfloat16><<<blocks, 256, 0, stream>>>(p);
  else
    qkv_rope_bwd_kernel<__half><<<blocks, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace frsa
