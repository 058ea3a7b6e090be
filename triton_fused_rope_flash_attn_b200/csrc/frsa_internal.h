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
  int H;         // heads (maps address [B, H, N, D] tensors as {D, N, H, B})
  int N;         // sequence length
  int D;         // head dim (multiple of 8, <= 128)
  int has_cls;   // 0 or 1; -1: no RoPE (q and k arrive rotated, nothing is rotated)
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
// Its backward epilogue: dq, dk, dv [B, H, N, D] -> dqkv [B*N, 3C], R^T on q, k.
cudaError_t launch_qkv_rope_bwd(bool bf16, const void* dq, const void* dk, const void* dv,
                                const float* cosp, const float* sinp, void* dqkv, long long M,
                                int N, int C, int H, int D, int has_cls, cudaStream_t stream);

// f32 <-> 16-bit conversion with the rotation (frsa_convert.cu): in: q, k, v
// f32 -> R(q), R(k), v 16-bit; out: 16-bit dq^, dk^, dv -> R^T dq^, R^T dk^, dv f32.
cudaError_t launch_convert(bool in, bool bf16, const void* const* src, void* const* dst,
                           const float* cosp, const float* sinp, long long rows, int N, int D,
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

// True when the shape needs the general backward (and its workspace): N > 256
// or D > 64. Otherwise the persistent single-head kernel runs (launch_bwd_small).
bool bwd_needs_workspace(const LaunchShape& s);
// Partial dQ slots frsa_bwd uses for this shape (min(key tiles, 8)).
int bwd_slots(const LaunchShape& s);
// int32 words of counters (arrivals, slot turns, claim ticket) the general
// backward needs with `nslot` partial slots.
size_t bwd_counter_ints(const LaunchShape& s, int nslot);

// Rotation pre-pass of the general backward: q and k (element strides b, h,
// n) are rotated once into contiguous buffers q_rot / k_rot, which the
// kernel's maps tm_q / tm_k then cover.
struct QkRotation {
  const void* q;
  const void* k;
  long long q_strides[3];
  long long k_strides[3];
  void* q_rot;
  void* k_rot;
};

// General backward: optional row pre-pass (rotation of q and k when `rot` is
// given; Delta into delta_buf when that is non-null, then read by the main
// kernel; when null the kernel forms Delta itself and writes `delta` if
// given), then the persistent key-tile kernel with the ordered dQ reduction
// (which rotates the Q and K tiles itself when `rot` is null).
// dq_part: f32 [nslot, BH, N, D] partial sums (1 <= nslot <= key tiles);
// counters: bwd_counter_ints(s, nslot) int32 words (cleared here on `stream`).
// tm_dk / tm_dv: the usual maps over dK / dV; tm_part: f32 map {D, N, nslot*BH}
// over dq_part with box {32, 128, 1} and the 128-byte swizzle.
cudaError_t launch_bwd_ordered(const LaunchShape& s, const CUtensorMap& tm_q,
                               const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                               const CUtensorMap& tm_do, const CUtensorMap& tm_o,
                               const CUtensorMap& tm_dk, const CUtensorMap& tm_dv,
                               const CUtensorMap& tm_part, const void* o,
                               const void* d_o, const float* lse, float* delta,
                               const float* cosp, const float* sinp, void* dq, void* dk, void* dv,
                               float* dq_part, int nslot, int* counters, float* delta_buf,
                               const QkRotation* rot, cudaStream_t stream);

// Number of SMs of the current device (queried once per device).
int device_sm_count();

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device).
cudaError_t set_max_dynamic_smem_once(const void* kernel, size_t bytes);
template <typename K>
inline cudaError_t set_max_dynamic_smem_once(K* kernel, size_t bytes) {
  return set_max_dynamic_smem_once(reinterpret_cast<const void*>(kernel), bytes);
}

}  // namespace frsa
