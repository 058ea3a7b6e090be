// Internal launcher interface shared by the C-ABI layer and the kernel files.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace frsa {

// Tile geometry shared by every kernel: 128-row tiles, 64-column (128-byte)
// swizzle chunks of 16-bit elements.
constexpr int kTile = 128;
constexpr int kChunkCols = 64;
constexpr int kChunkBytes = kTile * kChunkCols * 2;  // 16 KiB

struct LaunchShape {
  int BH;        // B * H
  int N;         // sequence length
  int D;         // head dim (multiple of 8, <= 128)
  int has_cls;
  float scale;
  bool bf16;     // true: bf16, false: f16 (16-bit kernels)
  bool f32;      // float32 I/O and TF32 compute (the frsa_tf32.cu kernels)
};

// Forward. tm_q/k/v: 3-D maps {D, N, BH} with box {64, 128, 1}, 128B swizzle.
// tm_o: the same map over O (used by the persistent kernel's TMA store).
cudaError_t launch_fwd(const LaunchShape& s, const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                       const CUtensorMap& tm_v, const CUtensorMap& tm_o, const float* cosp,
                       const float* sinp, void* o, float* lse, cudaStream_t stream);

// float32 compute on TF32 tensor cores. Maps: {D, N, BH} float32, box {32, 128, 1}.
cudaError_t launch_fwd_tf32(const LaunchShape& s, const CUtensorMap& tm_q,
                            const CUtensorMap& tm_k, const CUtensorMap& tm_v, const float* cosp,
                            const float* sinp, float* o, float* lse, cudaStream_t stream);

// float32 backward on TF32 tensor cores (D <= 64): a Delta pass into `delta`
// (fp32 [BH, N]), a dK/dV kernel and a dQ kernel. maps: q, k, v, dO in the
// K-major layout and q, k, dO in the MN-major (32-byte-atom) layout, in the
// order q16, q32, k16, k32, v16, do16, do32.
bool tf32_bwd_supported(const LaunchShape& s);
cudaError_t launch_bwd_tf32(const LaunchShape& s, const CUtensorMap* maps, const float* o,
                            const float* d_o, const float* lse, float* delta, const float* cosp,
                            const float* sinp, float* dq, float* dk, float* dv,
                            cudaStream_t stream);

// QKV projection with RoPE in the epilogue (frsa_qkv.cu). tm_x: 2-D {C, M},
// tm_w: 2-D {C, 3C}, both box {64, 128}, 128-byte swizzle.
cudaError_t launch_qkv_rope(bool bf16, const CUtensorMap& tm_x, const CUtensorMap& tm_w,
                            const float* bias, const float* cosp, const float* sinp, void* q,
                            void* k, void* v, long long M, int N, int C, int H, int D,
                            int has_cls, cudaStream_t stream);

// Persistent forward for N <= 256, D <= 64 (RoPE tables resident in shared memory).
bool fwd_small_applies(const LaunchShape& s);
cudaError_t launch_fwd_small(const LaunchShape& s, const CUtensorMap& tm_q,
                             const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                             const float* cosp, const float* sinp, void* o, float* lse,
                             cudaStream_t stream);

// Persistent backward for N <= 256, D <= 64 (dQ reduced on chip).
cudaError_t launch_bwd_small(const LaunchShape& s, const CUtensorMap& tm_q,
                             const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                             const CUtensorMap& tm_do, const CUtensorMap& tm_o,
                             const CUtensorMap* tm_grads, const void* o, const float* lse,
                             float* delta, const float* cosp, const float* sinp, void* dq,
                             void* dk, void* dv, cudaStream_t stream);

// Backward (delta preprocess + main kernel + optional dQ finalize).
// dq_accum: fp32 [BH, N, D] workspace or nullptr when bwd_needs_workspace() is false.
// tm_grads: maps over dQ, dK, dV (in that order), required when
// bwd_needs_workspace() is false (the persistent kernel stores through them).
bool bwd_needs_workspace(const LaunchShape& s);
cudaError_t launch_bwd(const LaunchShape& s, const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                       const CUtensorMap& tm_v, const CUtensorMap& tm_do, const CUtensorMap& tm_o,
                       const void* o, const CUtensorMap* tm_grads, const void* d_o, const float* lse,
                       float* delta, const float* cosp, const float* sinp, void* dq, void* dk,
                       void* dv, float* dq_accum, float* delta_buf, cudaStream_t stream);
// delta_buf (atomic mode, optional): B*H*N floats that receive Delta in a
// pre-pass, which the main kernel then reads instead of forming it per tile.

}  // namespace frsa
